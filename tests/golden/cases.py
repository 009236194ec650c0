"""Seeded input builders shared by the golden-vector generator and the tests.

Every case is rebuilt bit-identically from ``numpy.random.default_rng(seed)``
wherever it runs (this container, the GPU box), so the committed fixtures
only hold the reference's outputs, never the inputs.

Block tables are produced by ``fifo_tables`` - the reference allocator's
policy (pagedserve/engine/block_manager.py:71-139: take from the head of the
free list, append to a request's table on growth) - or as seeded random
permutation slices of the pool for the serving-scale shapes.
"""

from __future__ import annotations

import numpy as np

from oracle.paged_attention import bf16_round, f16_round


def _values(rng: np.random.Generator, shape, dtype: str) -> np.ndarray:
    x = rng.standard_normal(shape, dtype=np.float32)
    if dtype == "bfloat16":
        return bf16_round(x)
    if dtype == "float16":
        return f16_round(x)
    return x


def blocks_needed(n: int, block_size: int) -> int:
    return 0 if n <= 0 else -(-n // block_size)


def fifo_tables(first_counts, grow_to, num_blocks: int, block_size: int, free_list=None):
    """Tables after ``allocate(r, first_counts[r])`` for every request in order,
    then ``append_tokens(r, grow_to[r] - first_counts[r])`` in order.

    Mirrors PagedKVCache.allocate/append_tokens on top of BlockManager's FIFO
    free list (paged_kv_cache.py:47-105, block_manager.py:71-139).
    """
    free = list(range(num_blocks)) if free_list is None else list(free_list)
    tables = []
    for n in first_counts:
        need = blocks_needed(n, block_size)
        tables.append(free[:need])
        del free[:need]
    for r, (n0, n1) in enumerate(zip(first_counts, grow_to)):
        extra = blocks_needed(n1, block_size) - blocks_needed(n0, block_size)
        if extra > 0:
            tables[r] = tables[r] + free[:extra]
            del free[:extra]
    return tables


def decode_case(name: str) -> dict:
    """A decode case: pools, tables, lengths and queries.

    Returns a dict with keys ``dtype, num_layers, num_blocks, num_kv_heads,
    head_dim, block_size, q_heads, layer, tables, context_lens, q [B,Hq,D],
    k_cache, v_cache [L,NB,Hkv,BS,D]`` (fp32 arrays holding ``dtype`` values)
    and ``alloc`` (``(first_counts, grow_to)`` when the tables came from the
    FIFO allocator, else ``None``).
    """
    spec = dict(num_layers=1, num_kv_heads=2, head_dim=64, block_size=16, q_heads=4, layer=0)
    alloc = None
    if name.startswith("frag_"):
        # reference test_triton_paged_decode.py:20-62
        dtype = "float32" if name == "frag_fp32" else "bfloat16"
        seed, lens, nb = 7, [17, 32, 65], 32
        alloc = ([1] * 3, lens)
    elif name.startswith("boundary_"):
        # reference test_triton_paged_decode.py:80-137: B in {1,2,4,8}, layer in {0,1}
        _, b_str, l_str = name.split("_")
        bsz, layer = int(b_str[1:]), int(l_str[1:])
        dtype, nb = "bfloat16", 128
        seed = 1000 + layer * 100 + bsz
        lens = [1, 15, 16, 17, 31, 32, 33, 65][:bsz]
        spec.update(num_layers=2, layer=layer)
        alloc = ([1] * bsz, lens)
    elif name.startswith("layers_"):
        # reference test_triton_paged_decode.py:140-182
        layer = int(name[-1])
        dtype, seed, lens, nb = "float32", 2026, [17], 16
        spec.update(num_layers=2, layer=layer)
        alloc = ([1], lens)
    elif name == "config1":
        # CPU-runnable serving geometry: 8 seqs, ctx ~ U[1,512], Qwen 14q/2kv, fp32
        dtype, seed, nb = "float32", 11, 512
        spec.update(q_heads=14)
        lens = None
    elif name == "qwen_bf16":
        dtype, seed, nb = "bfloat16", 23, 400
        spec.update(q_heads=14)
        lens = None
    elif name == "qwen_f16":
        dtype, seed, nb = "float16", 29, 200
        spec.update(q_heads=14)
        lens = None
    else:
        raise KeyError(name)

    rng = np.random.default_rng(seed)
    bs = spec["block_size"]
    if alloc is not None:
        tables = fifo_tables(alloc[0], alloc[1], nb, bs)
    else:
        bsz = 8 if name == "config1" else 16
        hi = 512 if name == "config1" else 300
        lens = [int(x) for x in rng.integers(1, hi + 1, size=bsz)]
        perm = rng.permutation(nb)
        tables, at = [], 0
        for n in lens:
            need = blocks_needed(n, bs)
            tables.append([int(x) for x in perm[at:at + need]])
            at += need
        assert at <= nb
    shape = (spec["num_layers"], nb, spec["num_kv_heads"], bs, spec["head_dim"])
    k_cache = _values(rng, shape, dtype)
    v_cache = _values(rng, shape, dtype)
    q = _values(rng, (len(lens), spec["q_heads"], spec["head_dim"]), dtype)
    return dict(spec, dtype=dtype, num_blocks=nb, tables=tables, context_lens=list(lens), q=q,
                k_cache=k_cache, v_cache=v_cache, alloc=alloc, seed=seed)


DECODE_CASES = ["frag_fp32", "frag_bf16", "config1", "qwen_bf16", "qwen_f16", "layers_fp32_L0",
                "layers_fp32_L1"] + [f"boundary_B{b}_L{l}" for b in (1, 2, 4, 8) for l in (0, 1)]


def prefill_case(name: str) -> dict:
    """A causal case for ``paged_attention(query [Hq,S,D], cache, rid, layer, start)``.

    Keys ``dtype, q [Hq,S,D], start, table, k_cache, v_cache, block_size,
    num_kv_heads, head_dim, layer``.
    """
    if name == "gqa_tiny":
        # reference test_paged_attention.py:125-150: fragmentation leaves the
        # request's blocks at [3, 4, 1]
        dtype, seed, hq, hkv, d, bs, nb, s, start = "float32", 456, 4, 2, 4, 2, 5, 5, 0
        table = [3, 4, 1]
    elif name == "qwen_fp32":
        dtype, seed, hq, hkv, d, bs, nb, s, start = "float32", 31, 14, 2, 64, 16, 16, 40, 0
        table = None
    elif name == "qwen_bf16":
        dtype, seed, hq, hkv, d, bs, nb, s, start = "bfloat16", 37, 14, 2, 64, 16, 16, 33, 0
        table = None
    elif name == "prefix_bf16":
        dtype, seed, hq, hkv, d, bs, nb, s, start = "bfloat16", 41, 14, 2, 64, 16, 16, 8, 20
        table = None
    else:
        raise KeyError(name)
    rng = np.random.default_rng(seed)
    if table is None:
        table = [int(x) for x in rng.permutation(nb)[: blocks_needed(start + s, bs)]]
    shape = (1, nb, hkv, bs, d)
    k_cache = _values(rng, shape, dtype)
    v_cache = _values(rng, shape, dtype)
    q = _values(rng, (hq, s, d), dtype)
    return dict(dtype=dtype, q=q, start=start, table=table, k_cache=k_cache, v_cache=v_cache,
                block_size=bs, num_kv_heads=hkv, head_dim=d, layer=0, num_blocks=nb, seed=seed)


PREFILL_CASES = ["gqa_tiny", "qwen_fp32", "qwen_bf16", "prefix_bf16"]


def write_case(dtype: str = "bfloat16") -> dict:
    """Token writes through fragmented tables across block boundaries.

    Three requests allocated interleaved then grown (tables from the FIFO
    allocator), every position of every request written on layer 1 of a
    2-layer pool; positions 15/16 cross a block boundary
    (reference test_paged_kv_cache.py:229-245, test_cuda_integration.py:276-323).
    """
    rng = np.random.default_rng(99)
    nb, bs, hkv, d, layers = 16, 16, 2, 64, 2
    lens = [17, 40, 5]
    tables = fifo_tables([1, 1, 1], lens, nb, bs)
    positions = [list(range(n)) for n in lens]
    keys = [_values(rng, (n, hkv, d), dtype) for n in lens]
    values = [_values(rng, (n, hkv, d), dtype) for n in lens]
    base = _values(rng, (layers, nb, hkv, bs, d), dtype)
    return dict(dtype=dtype, num_blocks=nb, block_size=bs, num_kv_heads=hkv, head_dim=d,
                num_layers=layers, layer=1, lens=lens, tables=tables, positions=positions,
                keys=keys, values=values, base_k=base, base_v=base[::-1].copy())


def varlen_case(seed: int, lens, hq: int = 14, hkv: int = 2, d: int = 64, dtype: str = "bfloat16") -> dict:
    """Packed ragged prefill inputs: ``q [T,Hq,D]``, ``k, v [T,Hkv,D]``, ``cu_seqlens``."""
    rng = np.random.default_rng(seed)
    lens = [int(x) for x in lens]
    t = int(sum(lens))
    cu = np.zeros(len(lens) + 1, dtype=np.int32)
    cu[1:] = np.cumsum(lens)
    return dict(dtype=dtype, cu_seqlens=cu, lens=lens,
                q=_values(rng, (t, hq, d), dtype), k=_values(rng, (t, hkv, d), dtype),
                v=_values(rng, (t, hkv, d), dtype))
