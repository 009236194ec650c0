"""CPU oracle for the paged-attention hot path.  TEST INFRASTRUCTURE ONLY.

This module restates, in numpy, the arithmetic of PagedServe's own PyTorch
attention paths so that the CUDA kernels of ``pagedserve_b200`` can be checked
against it.  It is imported only by ``tests/``, by ``__graft_entry__.smoke()``
and by ``bench.py`` (its ``cpu_baseline`` leg and its ``--impl reference`` arm).
The product path never imports it: the CUDA library fails loudly when it is
missing instead of falling back here.

Parity is pinned: ``tests/golden/make_golden.py`` runs the reference's own
functions (``vectorized_paged_attention``, ``paged_attention``,
``PagedKVCache.write_token``) on seeded inputs and stores their outputs under
``tests/golden/``; ``tests/test_oracle_golden.py`` checks every function here
against those vectors.

Reference functions restated (paths inside the PagedServe project):

* ``decode_attention``   <- pagedserve/attention/vectorized_batched_attention.py:79-159
* ``causal_attention``   <- pagedserve/attention/paged_attention.py:94-145 (per-position causal
                            gather, fp32 softmax, probabilities cast to the query dtype
                            before P.V at :133-137)
* ``write_tokens``       <- pagedserve/engine/paged_kv_cache.py:187-200
* ``slot_for``           <- pagedserve/engine/paged_kv_cache.py:187-192
* ``padded_block_table`` <- pagedserve/attention/triton_paged_decode.py:134-154
* ``apply_rope``         <- pagedserve/attention/batched_paged_attention.py:105-112
                            (transformers Qwen2 ``apply_rotary_pos_emb``, imported at :8)

Two numeric modes are offered.  ``mode="exact"`` computes in float64 from the
stored values: this is the "fp32 reference" the bf16 kernels are held to
(max-abs 2e-2, mean-abs 2e-3).  ``mode="emulate"`` additionally rounds the
intermediate tensors the way the reference's bf16/f16 PyTorch path does
(scores after Q.K^T and after the 1/sqrt(D) division, probabilities before
P.V, and the output), so the oracle can be pinned tightly against golden
vectors produced by the reference in bf16.
"""

from __future__ import annotations

import math
from typing import Sequence

import numpy as np

__all__ = [
    "bf16_round",
    "f16_round",
    "round_to",
    "bf16_bits",
    "bf16_from_bits",
    "slot_for",
    "slot_mapping",
    "padded_block_table",
    "gather_context",
    "decode_attention",
    "causal_attention",
    "paged_causal_attention",
    "varlen_causal_attention",
    "varlen_causal_attention_blocked",
    "write_tokens",
    "reshape_and_cache",
    "pack_step",
]


# --------------------------------------------------------------------------
# low-precision rounding helpers (round-to-nearest-even, as torch's .to() does)
# --------------------------------------------------------------------------

def bf16_bits(x: np.ndarray) -> np.ndarray:
    """fp32 -> bfloat16 bit patterns (uint16), round-to-nearest-even; NaN stays NaN."""
    f = np.ascontiguousarray(x, dtype=np.float32)
    u = f.view(np.uint32).astype(np.uint64)
    lsb = (u >> 16) & 1
    rounded = ((u + 0x7FFF + lsb) >> 16).astype(np.uint16)
    nan = np.isnan(f)
    if nan.any():
        rounded = rounded.copy()
        rounded[nan] = ((u[nan] >> 16) | 0x40).astype(np.uint16)  # keep it a quiet NaN
    return rounded


def bf16_from_bits(b: np.ndarray) -> np.ndarray:
    """bfloat16 bit patterns (uint16) -> fp32 values."""
    return (np.ascontiguousarray(b, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def bf16_round(x: np.ndarray) -> np.ndarray:
    """Round to the nearest bfloat16 value, returned as fp32."""
    return bf16_from_bits(bf16_bits(x))


def f16_round(x: np.ndarray) -> np.ndarray:
    """Round to the nearest IEEE half value, returned as fp32."""
    return np.asarray(x, dtype=np.float32).astype(np.float16).astype(np.float32)


def round_to(x: np.ndarray, dtype: str) -> np.ndarray:
    """Round ``x`` to storage ``dtype`` ("float32", "bfloat16" or "float16")."""
    if dtype == "bfloat16":
        return bf16_round(x)
    if dtype == "float16":
        return f16_round(x)
    if dtype == "float32":
        return np.asarray(x, dtype=np.float32)
    raise ValueError(f"unsupported dtype {dtype!r}")


# --------------------------------------------------------------------------
# block-table arithmetic
# --------------------------------------------------------------------------

def slot_for(table: Sequence[int], position: int, block_size: int) -> int:
    """Physical slot of logical ``position``: ``table[pos // BS] * BS + pos % BS``.

    Restates PagedKVCache.write_token's addressing
    (pagedserve/engine/paged_kv_cache.py:187-192).
    """
    if position < 0:
        raise IndexError(f"negative position {position}")
    logical = position // block_size
    if logical >= len(table):
        raise IndexError(f"position {position} beyond the block table ({len(table)} blocks)")
    return int(table[logical]) * block_size + position % block_size


def slot_mapping(tables: Sequence[Sequence[int]], positions: Sequence[Sequence[int]] | Sequence[int],
                 block_size: int) -> np.ndarray:
    """int64 slot for each (request, position) pair, requests in order."""
    out = []
    for table, pos in zip(tables, positions):
        if np.isscalar(pos):
            pos = [pos]
        out.extend(slot_for(table, int(p), block_size) for p in pos)
    return np.asarray(out, dtype=np.int64)


def padded_block_table(tables: Sequence[Sequence[int]], width: int | None = None) -> np.ndarray:
    """Zero-padded int32 ``[B, max_blocks]`` table, as the reference's Triton
    wrapper builds it on the host (pagedserve/attention/triton_paged_decode.py:143-150)."""
    width = max((len(t) for t in tables), default=0) if width is None else width
    out = np.zeros((len(tables), width), dtype=np.int32)
    for row, table in enumerate(tables):
        out[row, : len(table)] = np.asarray(table, dtype=np.int32)
    return out


def gather_context(cache: np.ndarray, layer: int, table: Sequence[int], length: int) -> np.ndarray:
    """``[Hkv, length, D]`` view of one request's history through its block table.

    ``cache`` is one pool tensor ``[L, NB, Hkv, BS, D]``
    (layout of pagedserve/engine/kv_cache.py:51-69).  Equivalent to calling
    PagedKVCache.read_token for positions ``0..length-1``
    (pagedserve/engine/paged_kv_cache.py:202-233).
    """
    block_size = cache.shape[3]
    pos = np.arange(length)
    blocks = np.asarray(table, dtype=np.int64)[pos // block_size]
    rows = cache[layer, blocks, :, pos % block_size, :]  # [length, Hkv, D]
    return np.transpose(rows, (1, 0, 2))


# --------------------------------------------------------------------------
# attention
# --------------------------------------------------------------------------

def _softmax_rows(scores: np.ndarray) -> np.ndarray:
    m = np.max(scores, axis=-1, keepdims=True)
    e = np.exp(scores - m)
    return e / np.sum(e, axis=-1, keepdims=True)


def _attend(q: np.ndarray, k: np.ndarray, v: np.ndarray, dtype: str, mode: str) -> np.ndarray:
    """Attention of queries ``q [G, D]`` over ``k, v [n, D]`` (one kv head).

    ``mode="exact"``: float64 throughout.  ``mode="emulate"``: the rounding
    steps of the reference's PyTorch arithmetic for a low-precision ``dtype``
    (vectorized_batched_attention.py:141-159 / paged_attention.py:121-143):
    scores = round(round(Q.K^T) / sqrt(D)); probabilities = round(softmax_fp32);
    output = round(P.V).
    """
    d = q.shape[-1]
    if mode == "exact" or dtype == "float32":
        scores = (q.astype(np.float64) @ k.astype(np.float64).T) / math.sqrt(d)
        probs = _softmax_rows(scores)
        out = probs @ v.astype(np.float64)
        return out if mode == "exact" else out.astype(np.float32)
    if mode != "emulate":
        raise ValueError(f"unknown mode {mode!r}")
    raw = round_to((q.astype(np.float32) @ k.astype(np.float32).T), dtype)
    scores = round_to(raw / np.float32(math.sqrt(d)), dtype).astype(np.float32)
    probs = round_to(_softmax_rows(scores.astype(np.float64)).astype(np.float32), dtype)
    return round_to(probs.astype(np.float32) @ v.astype(np.float32), dtype)


def decode_attention(q: np.ndarray, k_cache: np.ndarray, v_cache: np.ndarray,
                     tables: Sequence[Sequence[int]], context_lens: Sequence[int], layer: int,
                     dtype: str = "float32", mode: str = "exact") -> np.ndarray:
    """Single-token paged GQA decode, ``q [B, Hq, D]`` -> ``[B, Hq, D]``.

    Restates vectorized_paged_attention (vectorized_batched_attention.py:79-159):
    request ``b`` attends to its first ``context_lens[b]`` (= position + 1)
    cached tokens; q head ``h`` reads kv head ``h // (Hq // Hkv)``; scores are
    scaled by ``1/sqrt(D)``; softmax in fp32.
    """
    bsz, hq, d = q.shape
    hkv = k_cache.shape[2]
    group = hq // hkv
    out = np.zeros((bsz, hq, d), dtype=np.float64 if mode == "exact" else np.float32)
    for b in range(bsz):
        n = int(context_lens[b])
        if n <= 0:
            continue
        keys = gather_context(k_cache, layer, tables[b], n)
        vals = gather_context(v_cache, layer, tables[b], n)
        for kh in range(hkv):
            heads = slice(kh * group, (kh + 1) * group)
            out[b, heads] = _attend(q[b, heads], keys[kh], vals[kh], dtype, mode)
    return out


def causal_attention(q: np.ndarray, keys: np.ndarray, values: np.ndarray, start: int,
                     dtype: str = "float32", mode: str = "exact") -> np.ndarray:
    """Causal attention of ``q [Hq, S, D]`` whose first row sits at ``start``.

    Query row ``i`` (position ``start + i``) sees keys ``0 .. start + i`` of
    ``keys, values [Hkv, >= start + S, D]``.  Restates paged_attention
    (paged_attention.py:94-145).
    """
    hq, s, d = q.shape
    hkv = keys.shape[0]
    group = hq // hkv
    out = np.zeros((hq, s, d), dtype=np.float64 if mode == "exact" else np.float32)
    for i in range(s):
        visible = start + i + 1
        for kh in range(hkv):
            heads = slice(kh * group, (kh + 1) * group)
            out[heads, i] = _attend(q[heads, i], keys[kh, :visible], values[kh, :visible], dtype, mode)
    return out


def paged_causal_attention(q: np.ndarray, k_cache: np.ndarray, v_cache: np.ndarray,
                           table: Sequence[int], layer: int, start: int,
                           dtype: str = "float32", mode: str = "exact") -> np.ndarray:
    """``paged_attention(query [Hq,S,D], cache, request, layer, start)`` on a numpy pool."""
    s = q.shape[1]
    keys = gather_context(k_cache, layer, table, start + s)
    vals = gather_context(v_cache, layer, table, start + s)
    return causal_attention(q, keys, vals, start, dtype, mode)


def varlen_causal_attention(q: np.ndarray, k: np.ndarray, v: np.ndarray, cu_seqlens: Sequence[int],
                            dtype: str = "float32", mode: str = "exact") -> np.ndarray:
    """Packed ragged causal prefill: ``q [T, Hq, D]``, ``k, v [T, Hkv, D]``.

    Sequence ``i`` owns rows ``cu_seqlens[i] .. cu_seqlens[i+1]`` and is causal
    within itself.  Per sequence this is exactly ``paged_attention`` with
    ``query_start_position = 0`` (paged_attention.py:94-145), which the
    reference runs one request at a time (qwen_paged_attention.py:110-128).
    """
    t, hq, d = q.shape
    out = np.zeros((t, hq, d), dtype=np.float64 if mode == "exact" else np.float32)
    for i in range(len(cu_seqlens) - 1):
        a, b = int(cu_seqlens[i]), int(cu_seqlens[i + 1])
        if b <= a:
            continue
        qs = np.transpose(q[a:b], (1, 0, 2))
        ks = np.transpose(k[a:b], (1, 0, 2))
        vs = np.transpose(v[a:b], (1, 0, 2))
        out[a:b] = np.transpose(causal_attention(qs, ks, vs, 0, dtype, mode), (1, 0, 2))
    return out


# --------------------------------------------------------------------------
# KV scatter
# --------------------------------------------------------------------------

def varlen_causal_attention_blocked(q: np.ndarray, k: np.ndarray, v: np.ndarray, cu_seqlens: Sequence[int],
                                    rows: int = 256) -> np.ndarray:
    """``varlen_causal_attention`` in ``mode="exact"`` (float64), evaluated
    ``rows`` query rows and one kv head at a time as matrix products instead
    of one row at a time: the same arithmetic (paged_attention.py:94-145 per
    sequence), fast enough for full 16K-token packs.  Pinned to the per-row
    form by the oracle tests."""
    t, hq, d = q.shape
    hkv = k.shape[1]
    group = hq // hkv
    out = np.zeros((t, hq, d), dtype=np.float64)
    scale = 1.0 / math.sqrt(d)
    for i in range(len(cu_seqlens) - 1):
        a, b = int(cu_seqlens[i]), int(cu_seqlens[i + 1])
        n = b - a
        for kh in range(hkv):
            keys = k[a:b, kh].astype(np.float64)          # [n, D]
            vals = v[a:b, kh].astype(np.float64)
            heads = slice(kh * group, (kh + 1) * group)
            for r0 in range(0, n, rows):
                r1 = min(n, r0 + rows)
                qq = q[a + r0:a + r1, heads].astype(np.float64)          # [r, G, D]
                sc = np.einsum("rgd,kd->rgk", qq, keys[:r1]) * scale     # keys 0 .. r1 - 1
                vis = np.arange(r1)[None, :] <= np.arange(r0, r1)[:, None]  # [r, k] causal
                sc = np.where(vis[:, None, :], sc, -np.inf)
                sc -= sc.max(axis=-1, keepdims=True)
                e = np.exp(sc)
                p = e / e.sum(axis=-1, keepdims=True)
                out[a + r0:a + r1, heads] = np.einsum("rgk,kd->rgd", p, vals[:r1])
    return out


def write_tokens(k_cache: np.ndarray, v_cache: np.ndarray, layer: int, table: Sequence[int],
                 positions: Sequence[int], keys: np.ndarray, values: np.ndarray) -> None:
    """In-place ``write_token`` for several positions of one request.

    ``keys, values [n, Hkv, D]``; restates pagedserve/engine/paged_kv_cache.py:187-200:
    ``cache[layer, table[pos // BS], :, pos % BS, :] = key``.
    """
    bs = k_cache.shape[3]
    for i, pos in enumerate(positions):
        blk = int(table[pos // bs])
        k_cache[layer, blk, :, pos % bs, :] = keys[i]
        v_cache[layer, blk, :, pos % bs, :] = values[i]


def reshape_and_cache(key: np.ndarray, value: np.ndarray, k_cache: np.ndarray, v_cache: np.ndarray,
                      slots: np.ndarray, layer: int) -> None:
    """Slot-mapped scatter of ``key, value [T, Hkv, D]`` into the pools, in place.

    Slot ``s`` addresses block ``s // BS`` offset ``s % BS`` (the addressing of
    paged_kv_cache.py:187-200).  A negative slot means "no write" (padding rows).
    """
    bs = k_cache.shape[3]
    for t, s in enumerate(np.asarray(slots, dtype=np.int64)):
        if s < 0:
            continue
        k_cache[layer, s // bs, :, s % bs, :] = key[t]
        v_cache[layer, s // bs, :, s % bs, :] = value[t]


def apply_rope(x: np.ndarray, cos: np.ndarray, sin: np.ndarray, dtype: str) -> np.ndarray:
    """Rotary position embedding of ``x [T, H, D]`` with per-token ``cos, sin
    [T, D]``, as the reference's decode glue applies it
    (pagedserve/attention/batched_paged_attention.py:105-112, the transformers
    Qwen2 ``apply_rotary_pos_emb``: ``x * cos + rotate_half(x) * sin`` with
    ``rotate_half(x) = cat(-x2, x1)``), rounded as PyTorch does for ``dtype``
    tensors: each product and the sum are computed in fp32 and rounded to
    ``dtype``.
    """
    x = np.asarray(x, dtype=np.float32)
    c = np.asarray(cos, dtype=np.float32)[:, None, :]
    s = np.asarray(sin, dtype=np.float32)[:, None, :]
    half = x.shape[-1] // 2
    rot = np.concatenate([-x[..., half:], x[..., :half]], axis=-1)
    a = round_to(x * c, dtype)
    b = round_to(rot * s, dtype)
    return round_to(a + b, dtype)


def rope_reshape_and_cache(query: np.ndarray, key: np.ndarray, value: np.ndarray, cos: np.ndarray, sin: np.ndarray,
                           k_cache: np.ndarray, v_cache: np.ndarray, slots: np.ndarray, layer: int,
                           dtype: str) -> tuple[np.ndarray, np.ndarray]:
    """The decode glue's RoPE followed by its per-row ``write_token`` loop
    (batched_paged_attention.py:105-124), over a slot mapping: returns the
    rotated ``(query, key)`` and writes the rotated key and the value into the
    pools in place (negative slot = no write)."""
    q_rot = apply_rope(query, cos, sin, dtype)
    k_rot = apply_rope(key, cos, sin, dtype)
    reshape_and_cache(k_rot, np.asarray(value, dtype=np.float32), k_cache, v_cache, slots, layer)
    return q_rot, k_rot


# --------------------------------------------------------------------------
# ragged-batch metadata
# --------------------------------------------------------------------------

def pack_step(tables: Sequence[Sequence[int]], starts: Sequence[int], query_lens: Sequence[int],
              block_size: int, width: int | None = None):
    """Metadata for one engine step over ``B`` requests.

    Request ``b`` contributes ``query_lens[b]`` new tokens at positions
    ``starts[b] .. starts[b] + query_lens[b] - 1``.  Returns
    ``(cu_seqlens int32 [B+1], slot_mapping int64 [T], context_lens int32 [B],
    block_tables int32 [B, width])`` where ``context_lens = starts + query_lens``
    (the reference's "length = position + 1", triton_paged_decode.py:140) and the
    table is zero padded (triton_paged_decode.py:143-150).
    """
    ql = np.asarray(query_lens, dtype=np.int64)
    cu = np.zeros(len(ql) + 1, dtype=np.int32)
    cu[1:] = np.cumsum(ql)
    positions = [list(range(int(s), int(s) + int(n))) for s, n in zip(starts, ql)]
    slots = slot_mapping(tables, positions, block_size)
    ctx = (np.asarray(starts, dtype=np.int64) + ql).astype(np.int32)
    return cu, slots, ctx, padded_block_table(tables, width)
