"""Test-side conversions between the numpy cases and torch device tensors."""

from __future__ import annotations

import numpy as np
import torch

TORCH_DTYPES = {"float32": torch.float32, "bfloat16": torch.bfloat16, "float16": torch.float16}


def to_dev(arr: np.ndarray, dtype: str, device="cuda") -> torch.Tensor:
    """fp32 numpy values (already representable in ``dtype``) -> device tensor, exactly."""
    return torch.from_numpy(np.ascontiguousarray(arr, dtype=np.float32)).to(device).to(TORCH_DTYPES[dtype])


def poison_unused(k_cache: np.ndarray, v_cache: np.ndarray, layer: int, tables, lens) -> tuple[np.ndarray, np.ndarray]:
    """Copies of the pools with NaN in every slot of ``layer`` outside the
    requests' first ``lens[b]`` positions (and in every other layer), so a
    kernel that reads outside the tables or lets masked rows leak produces NaN."""
    kc = np.full_like(k_cache, np.nan)
    vc = np.full_like(v_cache, np.nan)
    bs = k_cache.shape[3]
    blks, offs = [], []
    for table, n in zip(tables, lens):
        pos = np.arange(int(n))
        blks.append(np.asarray(table, dtype=np.int64)[pos // bs])
        offs.append(pos % bs)
    if blks:
        blk, off = np.concatenate(blks), np.concatenate(offs)
        kc[layer, blk, :, off, :] = k_cache[layer, blk, :, off, :]
        vc[layer, blk, :, off, :] = v_cache[layer, blk, :, off, :]
    return kc, vc


def err_stats(actual: torch.Tensor, expected: np.ndarray) -> tuple[float, float]:
    a = actual.detach().float().cpu().numpy().astype(np.float64)
    diff = np.abs(a - np.asarray(expected, dtype=np.float64))
    return float(np.max(diff)), float(np.mean(diff))


# bf16/f16 outputs vs the exact (float64) oracle: the bar the kernels are held to
TOL = {"bfloat16": (2e-2, 2e-3), "float16": (4e-3, 5e-4), "float32": (2e-4, 2e-5)}
