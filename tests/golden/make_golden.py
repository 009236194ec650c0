"""Generate golden vectors by running the PagedServe reference itself.

Run in a container that has the reference checkout (read-only is fine):

    python tests/golden/make_golden.py --reference <PagedServe checkout>

For every case in ``cases.py`` it builds the reference's own ``PagedKVCache``
on the CPU, reproduces the case's block tables with the reference allocator,
loads the seeded pools, and calls the reference's public functions:

* ``vectorized_paged_attention`` (pagedserve/attention/vectorized_batched_attention.py:11)
* ``paged_attention``            (pagedserve/attention/paged_attention.py:10)
* ``PagedKVCache.write_token``   (pagedserve/engine/paged_kv_cache.py:148)

Outputs go to ``tests/golden/reference_outputs.npz`` plus a small JSON with
the tables the reference allocator produced and SHA-256 digests of the pools
after the token writes.  Nothing on the GPU box reads the reference: the
tests only read these files.
"""

from __future__ import annotations

import argparse
import hashlib
import json
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, REPO)

from tests.golden.cases import DECODE_CASES, PREFILL_CASES, decode_case, prefill_case, write_case  # noqa: E402
from oracle.paged_attention import bf16_bits  # noqa: E402


def _torch_dtype(torch, name):
    return {"float32": torch.float32, "bfloat16": torch.bfloat16, "float16": torch.float16}[name]


def _to_torch(torch, arr, dtype):
    return torch.from_numpy(np.ascontiguousarray(arr, dtype=np.float32)).to(_torch_dtype(torch, dtype))


def _force_tables(cache, tables, lens):
    """Allocate each request so the reference's FIFO allocator hands out ``tables``."""
    order = [b for t in tables for b in t]
    rest = [b for b in range(cache.num_blocks) if b not in set(order)]
    cache.block_manager._free_blocks = order + rest
    rids = []
    for i, n in enumerate(lens):
        rid = f"req-{i}"
        cache.allocate(rid, n)
        assert cache.get_block_table(rid).get_blocks() == list(tables[i])
        rids.append(rid)
    return rids


def pool_digest(arr: np.ndarray, dtype: str) -> str:
    data = bf16_bits(arr) if dtype == "bfloat16" else np.ascontiguousarray(arr, dtype=np.float32)
    return hashlib.sha256(data.tobytes()).hexdigest()


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True,
                    help="root of a PagedServe checkout (the directory holding the pagedserve package)")
    args = ap.parse_args()
    sys.path.insert(0, args.reference)

    import torch
    from pagedserve.attention.paged_attention import paged_attention
    from pagedserve.attention.vectorized_batched_attention import vectorized_paged_attention
    from pagedserve.engine.paged_kv_cache import PagedKVCache

    torch.set_num_threads(min(8, os.cpu_count() or 1))
    arrays: dict[str, np.ndarray] = {}
    meta: dict[str, object] = {"decode": {}, "prefill": {}, "write": {}}

    for name in DECODE_CASES:
        c = decode_case(name)
        dt = _torch_dtype(torch, c["dtype"])
        cache = PagedKVCache(num_blocks=c["num_blocks"], num_layers=c["num_layers"],
                             num_kv_heads=c["num_kv_heads"], head_dim=c["head_dim"],
                             block_size=c["block_size"], dtype=dt, device="cpu")
        lens = c["context_lens"]
        if c["alloc"] is not None:
            first, grow = c["alloc"]
            rids = [f"req-{i}" for i in range(len(lens))]
            for rid, n in zip(rids, first):
                cache.allocate(rid, n)
            for rid, n0, n1 in zip(rids, first, grow):
                if n1 > n0:
                    cache.append_tokens(rid, n1 - n0)
            got = [cache.get_block_table(r).get_blocks() for r in rids]
            assert got == c["tables"], (name, got, c["tables"])
        else:
            rids = _force_tables(cache, c["tables"], lens)
        cache.kv_cache.k_cache.copy_(_to_torch(torch, c["k_cache"], c["dtype"]))
        cache.kv_cache.v_cache.copy_(_to_torch(torch, c["v_cache"], c["dtype"]))
        q = _to_torch(torch, c["q"], c["dtype"]).unsqueeze(2)  # [B, Hq, 1, D]
        positions = [n - 1 for n in lens]
        out = vectorized_paged_attention(q, cache, rids, positions, layer=c["layer"])
        arrays[f"decode/{name}"] = out.squeeze(2).float().numpy()
        # the per-row causal path used by the reference's "pytorch" backend
        rows = [paged_attention(q[b], cache, rids[b], c["layer"], positions[b]) for b in range(len(lens))]
        arrays[f"decode_rows/{name}"] = torch.stack(rows).squeeze(2).float().numpy()
        meta["decode"][name] = {"tables": c["tables"], "context_lens": lens}

    for name in PREFILL_CASES:
        c = prefill_case(name)
        dt = _torch_dtype(torch, c["dtype"])
        cache = PagedKVCache(num_blocks=c["num_blocks"], num_layers=1, num_kv_heads=c["num_kv_heads"],
                             head_dim=c["head_dim"], block_size=c["block_size"], dtype=dt, device="cpu")
        total = c["start"] + c["q"].shape[1]
        if name == "gqa_tiny":
            # the reference test's fragmentation sequence (test_paged_attention.py:125-150)
            cache.allocate("request-A", 2)
            cache.allocate("request-B", 2)
            cache.allocate("request-C", 2)
            cache.free("request-B")
            cache.allocate("request-D", total)
            rid = "request-D"
            assert cache.get_block_table(rid).get_blocks() == c["table"] == [3, 4, 1]
        else:
            rid = _force_tables(cache, [c["table"]], [total])[0]
        cache.kv_cache.k_cache.copy_(_to_torch(torch, c["k_cache"], c["dtype"]))
        cache.kv_cache.v_cache.copy_(_to_torch(torch, c["v_cache"], c["dtype"]))
        q = _to_torch(torch, c["q"], c["dtype"])
        out = paged_attention(q, cache, rid, 0, c["start"])
        arrays[f"prefill/{name}"] = out.float().numpy()
        meta["prefill"][name] = {"table": c["table"], "start": c["start"]}

    for dtype in ("bfloat16", "float32"):
        c = write_case(dtype)
        dt = _torch_dtype(torch, dtype)
        cache = PagedKVCache(num_blocks=c["num_blocks"], num_layers=c["num_layers"],
                             num_kv_heads=c["num_kv_heads"], head_dim=c["head_dim"],
                             block_size=c["block_size"], dtype=dt, device="cpu")
        rids = [f"w-{i}" for i in range(len(c["lens"]))]
        for rid in rids:
            cache.allocate(rid, 1)
        for rid, n in zip(rids, c["lens"]):
            cache.append_tokens(rid, n - 1)
        assert [cache.get_block_table(r).get_blocks() for r in rids] == c["tables"]
        cache.kv_cache.k_cache.copy_(_to_torch(torch, c["base_k"], dtype))
        cache.kv_cache.v_cache.copy_(_to_torch(torch, c["base_v"], dtype))
        for r, rid in enumerate(rids):
            for i, pos in enumerate(c["positions"][r]):
                cache.write_token(rid, c["layer"], pos, _to_torch(torch, c["keys"][r][i], dtype),
                                  _to_torch(torch, c["values"][r][i], dtype))
        kc = cache.kv_cache.k_cache.float().numpy()
        vc = cache.kv_cache.v_cache.float().numpy()
        meta["write"][dtype] = {"tables": c["tables"], "k_sha256": pool_digest(kc, dtype),
                                "v_sha256": pool_digest(vc, dtype)}

    np.savez_compressed(os.path.join(HERE, "reference_outputs.npz"), **arrays)
    with open(os.path.join(HERE, "reference_meta.json"), "w") as fh:
        json.dump(meta, fh, indent=1, sort_keys=True)
    print(f"wrote {len(arrays)} arrays")


if __name__ == "__main__":
    main()
