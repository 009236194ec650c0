"""Packed varlen causal prefill on the GPU vs the oracle and the reference's
golden ``paged_attention`` outputs (query_start_position 0)."""

from __future__ import annotations

import math
import os

import numpy as np
import pytest
import torch

from oracle import paged_attention as ora
from tests.golden.cases import prefill_case, varlen_case
from tests.helpers import TOL, err_stats, to_dev

pytestmark = pytest.mark.gpu

HERE = os.path.dirname(os.path.abspath(__file__))
GOLD = np.load(os.path.join(HERE, "golden", "reference_outputs.npz"))


def _run(c, hq=None):
    from pagedserve_b200 import ops
    q, k, v = (to_dev(c[x], c["dtype"]) for x in ("q", "k", "v"))
    cu = torch.from_numpy(np.asarray(c["cu_seqlens"], dtype=np.int32)).cuda()
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    out = ops.varlen_prefill(q, k, v, cu, max(c["lens"]), error_flag=err)
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    return out


@pytest.mark.parametrize("name", ["gqa_tiny", "qwen_fp32", "qwen_bf16"])
def test_prefill_matches_reference_golden(name):
    """The reference prefills one request through its paged cache; the packed
    kernel on the same rows must agree (reference tolerances)."""
    c = prefill_case(name)
    s = c["q"].shape[1]
    keys = ora.gather_context(c["k_cache"], 0, c["table"], s)  # [Hkv, S, D]
    vals = ora.gather_context(c["v_cache"], 0, c["table"], s)
    case = dict(dtype=c["dtype"], lens=[s], cu_seqlens=np.array([0, s], dtype=np.int32),
                q=np.transpose(c["q"], (1, 0, 2)), k=np.transpose(keys, (1, 0, 2)), v=np.transpose(vals, (1, 0, 2)))
    out = _run(case).float().cpu().permute(1, 0, 2)
    gold = torch.from_numpy(GOLD[f"prefill/{name}"])
    tol = 1e-4 if c["dtype"] == "float32" else 2e-2
    torch.testing.assert_close(out, gold, rtol=tol, atol=tol)


@pytest.mark.parametrize("dtype", ["bfloat16", "float16", "float32"])
@pytest.mark.parametrize("lens", [[1], [5, 1, 17], [128, 129, 127, 1, 256], [300, 64, 2048 // 4]])
def test_varlen_matches_oracle(dtype, lens):
    c = varlen_case(len(lens) * 7 + sum(lens), lens, dtype=dtype)
    out = _run(c)
    exact = ora.varlen_causal_attention(c["q"], c["k"], c["v"], c["cu_seqlens"])
    mx, mean = err_stats(out, exact)
    max_tol, mean_tol = TOL[dtype]
    assert mx <= max_tol and mean <= mean_tol, (mx, mean)


def test_varlen_packed_batch_lognormal():
    """A packed iteration shaped like the serving prefill workload: prompts
    lognormal(median 256, sigma 1.0) clipped to [32, 2048], ~4K tokens here."""
    rng = np.random.default_rng(4)
    lens = []
    while sum(lens) < 4096:
        lens.append(int(np.clip(round(rng.lognormal(math.log(256), 1.0)), 32, 2048)))
    c = varlen_case(77, lens)
    out = _run(c)
    # oracle on a stratified sub-sample of sequences (O(S^2) on the host)
    pick = sorted({0, len(lens) - 1, int(np.argmax(lens)), int(np.argmin(lens))})
    for i in pick:
        a, b = int(c["cu_seqlens"][i]), int(c["cu_seqlens"][i + 1])
        sub = ora.varlen_causal_attention(c["q"][a:b], c["k"][a:b], c["v"][a:b], [0, b - a])
        mx, mean = err_stats(out[a:b], sub)
        assert mx <= 2e-2 and mean <= 2e-3, (i, mx, mean)


@pytest.mark.parametrize("hq,hkv,d", [(4, 2, 64), (8, 1, 64), (14, 2, 128), (3, 3, 32)])
def test_varlen_other_geometries(hq, hkv, d):
    c = varlen_case(hq * 10 + d, [40, 130, 7], hq=hq, hkv=hkv, d=d)
    out = _run(c)
    exact = ora.varlen_causal_attention(c["q"], c["k"], c["v"], c["cu_seqlens"])
    mx, mean = err_stats(out, exact)
    assert mx <= 2e-2 and mean <= 2e-3, (mx, mean)


def test_malformed_cu_seqlens_reported():
    from pagedserve_b200 import ops
    c = varlen_case(3, [10, 10])
    q, k, v = (to_dev(c[x], c["dtype"]) for x in ("q", "k", "v"))
    cu = torch.tensor([0, 15, 12], dtype=torch.int32, device="cuda")
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    ops.varlen_prefill(q, k, v, cu, 15, error_flag=err)
    torch.cuda.synchronize()
    assert int(err.item()) & 32


@pytest.mark.parametrize("dtype", ["bfloat16", "float16"])
def test_varlen_strided_fused_qkv(dtype):
    """q, k and v as column slices of one fused QKV projection [T, (Hq + 2 Hkv) * D]
    (row stride 1152 elements), the layout the model's projection produces."""
    from pagedserve_b200 import ops
    lens = [200, 1, 130, 64]
    c = varlen_case(11, lens, dtype=dtype)
    t, hq, hkv, d = c["q"].shape[0], 14, 2, 64
    qkv = torch.zeros(t, (hq + 2 * hkv) * d, dtype=to_dev(c["q"], dtype).dtype, device="cuda")
    qkv[:, :hq * d] = to_dev(c["q"], dtype).reshape(t, hq * d)
    qkv[:, hq * d:(hq + hkv) * d] = to_dev(c["k"], dtype).reshape(t, hkv * d)
    qkv[:, (hq + hkv) * d:] = to_dev(c["v"], dtype).reshape(t, hkv * d)
    q = qkv[:, :hq * d].view(t, hq, d)
    k = qkv[:, hq * d:(hq + hkv) * d].view(t, hkv, d)
    v = qkv[:, (hq + hkv) * d:].view(t, hkv, d)
    assert q.stride(0) == (hq + 2 * hkv) * d
    cu = torch.from_numpy(np.asarray(c["cu_seqlens"], dtype=np.int32)).cuda()
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    out = ops.varlen_prefill(q, k, v, cu, max(lens), error_flag=err)
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    exact = ora.varlen_causal_attention(c["q"], c["k"], c["v"], c["cu_seqlens"])
    mx, mean = err_stats(out, exact)
    max_tol, mean_tol = TOL[dtype]
    assert mx <= max_tol and mean <= mean_tol, (mx, mean)


def test_varlen_longest_prompt():
    """A 2048-token prompt (16 query blocks, the heaviest tile streams 16 key
    tiles) packed with short ones; checked on its first, middle and last rows."""
    lens = [3, 2048, 129]
    c = varlen_case(5, lens)
    out = _run(c)
    a, b = int(c["cu_seqlens"][1]), int(c["cu_seqlens"][2])
    exact = ora.varlen_causal_attention(c["q"], c["k"], c["v"], c["cu_seqlens"])
    mx, mean = err_stats(out, exact)
    assert mx <= 2e-2 and mean <= 2e-3, (mx, mean)
    mx, _ = err_stats(out[b - 128:b], exact[b - 128:b])
    assert mx <= 2e-2


@pytest.mark.parametrize("pad", [2, 64])
def test_varlen_strided_output(pad):
    """Output rows in a wider buffer [T, Hq, 64 + pad]: pad 2 makes the head
    stride 132 bytes (the per-thread store path of the tensor-core epilogue),
    pad 64 keeps 16-byte rows (the path through the per-warp staging area);
    the padding columns must stay untouched."""
    from pagedserve_b200 import ops
    lens = [200, 1, 130, 64, 383]
    c = varlen_case(13, lens, dtype="bfloat16")
    q, k, v = (to_dev(c[x], "bfloat16") for x in ("q", "k", "v"))
    t, hq, d = q.shape
    wide = torch.full((t, hq, d + pad), 7.0, dtype=torch.bfloat16, device="cuda")
    out = wide[:, :, :d]
    cu = torch.from_numpy(np.asarray(c["cu_seqlens"], dtype=np.int32)).cuda()
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    res = ops.varlen_prefill(q, k, v, cu, max(lens), out=out, error_flag=err)
    torch.cuda.synchronize()
    assert int(err.item()) == 0 and res.data_ptr() == out.data_ptr()
    assert bool((wide[:, :, d:] == 7.0).all())
    exact = ora.varlen_causal_attention(c["q"], c["k"], c["v"], c["cu_seqlens"])
    mx, mean = err_stats(out, exact)
    max_tol, mean_tol = TOL["bfloat16"]
    assert mx <= max_tol and mean <= mean_tol, (mx, mean)
