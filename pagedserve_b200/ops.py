"""Tensor-level API over the C ABI: the batched hot path the engine calls.

* ``reshape_and_cache``  one launch per layer for all new tokens (replaces the
  per-token ``PagedKVCache.write_token`` loop,
  pagedserve/attention/batched_paged_attention.py:115-124)
* ``paged_decode``       split-K GQA decode over the paged pool (replaces
  pagedserve/attention/triton_paged_decode.py:10-95)
* ``varlen_prefill``     packed ragged causal prefill (replaces the per-request
  prefill of pagedserve/attention/qwen_paged_attention.py:121-128)
* ``pack_step``          GPU-side ragged-batch metadata for one engine step
  (replaces pagedserve/attention/triton_paged_decode.py:134-154)
* ``select_tokens``      greedy next token + stop check of every row on the
  device (replaces ``logits[:, -1, :].argmax`` and the per-row ``.item()``
  loop of pagedserve/engine/continuous_batcher.py:333-360)

Every function requires CUDA tensors, launches on the current stream and
returns without synchronising.  There is no CPU path.
"""

from __future__ import annotations

import ctypes
import functools
import math
import threading

import torch

from . import _native

_DTYPES = {torch.float32: _native.PSB_F32, torch.float16: _native.PSB_F16, torch.bfloat16: _native.PSB_BF16}


def dtype_code(dtype: torch.dtype) -> int:
    try:
        return _DTYPES[dtype]
    except KeyError:
        raise ValueError(f"Unsupported dtype {dtype}") from None


try:  # the raw handle of the current stream, without building a Stream object (as torch's own codegen does)
    from torch._C import _cuda_getCurrentRawStream as _raw_stream
except ImportError:  # pragma: no cover - older torch
    _raw_stream = None


def _stream(device: torch.device) -> int:
    if _raw_stream is not None:
        return _raw_stream(device.index if device.index is not None else torch.cuda.current_device())
    return torch.cuda.current_stream(device).cuda_stream


def _ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def _require_cuda(*tensors: torch.Tensor) -> None:
    for t in tensors:
        if not t.is_cuda:
            raise ValueError("B200 paged attention requires CUDA tensors")


def _pool_geometry(k_cache: torch.Tensor, v_cache: torch.Tensor):
    if k_cache.ndim != 5 or v_cache.shape != k_cache.shape:
        raise ValueError("k_cache/v_cache must be [num_layers, num_blocks, num_kv_heads, block_size, head_dim]")
    if not (k_cache.is_contiguous() and v_cache.is_contiguous()):
        raise ValueError("KV pools must be contiguous")
    if k_cache.dtype != v_cache.dtype:
        raise ValueError("k_cache and v_cache dtypes differ")
    return tuple(int(x) for x in k_cache.shape)


def reshape_and_cache(key: torch.Tensor, value: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor,
                      slot_mapping: torch.Tensor, layer: int, error_flag: torch.Tensor | None = None) -> None:
    """Scatter ``key, value [T, Hkv, D]`` into ``k_cache/v_cache[layer]`` at ``slot_mapping [T]`` (int64).

    Bit-exact with ``PagedKVCache.write_token`` (paged_kv_cache.py:187-200); a
    negative slot writes nothing.
    """
    _require_cuda(key, value, k_cache, v_cache, slot_mapping)
    nl, nb, hkv, bs, d = _pool_geometry(k_cache, v_cache)
    if key.ndim != 3 or key.shape[1:] != (hkv, d) or value.shape != key.shape:
        raise ValueError(f"key/value must be [T, {hkv}, {d}]")
    if key.dtype != k_cache.dtype or value.dtype != k_cache.dtype:
        raise ValueError("key/value dtype must match the cache dtype")
    if key.stride(2) != 1 or value.stride(2) != 1:
        raise ValueError("key/value need unit stride along head_dim")
    if slot_mapping.dtype != torch.int64 or slot_mapping.ndim != 1 or slot_mapping.shape[0] != key.shape[0]:
        raise ValueError("slot_mapping must be int64 [T]")
    if not slot_mapping.is_contiguous():
        slot_mapping = slot_mapping.contiguous()
    if not 0 <= layer < nl:
        raise ValueError("Invalid layer")
    lib = _native.load()
    _native.check(lib.psb_reshape_and_cache(
        key.data_ptr(), key.stride(0), key.stride(1), value.data_ptr(), value.stride(0), value.stride(1),
        k_cache.data_ptr(), v_cache.data_ptr(), slot_mapping.data_ptr(), key.shape[0], layer, nl, nb, hkv, bs, d,
        dtype_code(k_cache.dtype), _ptr(error_flag), _stream(key.device)), "reshape_and_cache")


def rope_reshape_and_cache(query: torch.Tensor, key: torch.Tensor, value: torch.Tensor, cos: torch.Tensor,
                           sin: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor, slot_mapping: torch.Tensor,
                           layer: int, query_out: torch.Tensor | None = None,
                           key_out: torch.Tensor | None | bool = None,
                           error_flag: torch.Tensor | None = None) -> tuple[torch.Tensor, torch.Tensor | None]:
    """Rotary embedding of ``query [T, Hq, D]`` and ``key [T, Hkv, D]`` with
    the per-token ``cos, sin [T, D]`` rows, fused with the slot-mapped write
    of the rotated keys and of ``value`` into ``k_cache/v_cache[layer]``
    (psb_rope_reshape_and_cache; bit-exact with the reference's
    ``apply_rotary_pos_emb`` then ``write_token``).

    Returns ``(query_out, key_out)``: ``query_out`` defaults to a new tensor
    (pass ``query`` to rotate in place); ``key_out`` defaults to a new tensor
    holding the rotated keys, ``False`` skips it (the pool still gets them).
    """
    _require_cuda(query, key, value, cos, sin, k_cache, v_cache, slot_mapping)
    nl, nb, hkv, bs, d = _pool_geometry(k_cache, v_cache)
    if query.ndim != 3 or query.shape[2] != d:
        raise ValueError(f"query must be [T, Hq, {d}]")
    t = query.shape[0]
    if key.shape != (t, hkv, d) or value.shape != (t, hkv, d):
        raise ValueError(f"key/value must be [{t}, {hkv}, {d}]")
    cos = cos.reshape(-1, d)
    sin = sin.reshape(-1, d)
    if cos.shape[0] != t or sin.shape != cos.shape:
        raise ValueError(f"cos/sin must hold one [{d}] row per token")
    if cos.stride(1) != 1 or sin.stride(1) != 1 or cos.stride(0) != sin.stride(0):
        cos, sin = cos.contiguous(), sin.contiguous()
    for x in (query, key, value, cos, sin):
        if x.dtype != k_cache.dtype:
            raise ValueError("query/key/value/cos/sin dtype must match the cache dtype")
        if x.stride(-1) != 1:
            raise ValueError("unit stride along head_dim is required")
    if slot_mapping.dtype != torch.int64 or slot_mapping.shape != (t,):
        raise ValueError("slot_mapping must be int64 [T]")
    slot_mapping = slot_mapping.contiguous()
    if not 0 <= layer < nl:
        raise ValueError("Invalid layer")
    if query_out is None:
        query_out = torch.empty_like(query)
    if query_out.shape != query.shape or query_out.dtype != query.dtype or query_out.stride(2) != 1:
        raise ValueError("query_out must match query's shape and dtype with unit stride along head_dim")
    if key_out is None:
        key_out = torch.empty_like(key)
    elif key_out is False:
        key_out = None
    if key_out is not None and (key_out.shape != key.shape or key_out.dtype != key.dtype or key_out.stride(2) != 1):
        raise ValueError("key_out must match key's shape and dtype with unit stride along head_dim")
    lib = _native.load()
    _native.check(lib.psb_rope_reshape_and_cache(
        query.data_ptr(), query.stride(0), query.stride(1), query_out.data_ptr(), query_out.stride(0),
        query_out.stride(1), key.data_ptr(), key.stride(0), key.stride(1), _ptr(key_out),
        key_out.stride(0) if key_out is not None else 0, key_out.stride(1) if key_out is not None else 0,
        value.data_ptr(), value.stride(0), value.stride(1), cos.data_ptr(), sin.data_ptr(), cos.stride(0),
        k_cache.data_ptr(), v_cache.data_ptr(), slot_mapping.data_ptr(), t, query.shape[1], layer, nl, nb, hkv, bs, d,
        dtype_code(k_cache.dtype), _ptr(error_flag), _stream(query.device)), "rope_reshape_and_cache")
    return query_out, key_out


class DecodeWorkspace:
    """Split-K scratch for ``paged_decode``: one growable buffer per device.

    The first bytes hold per-(sequence, kv head) arrival counters that must be
    zero before a launch; every launch leaves them zero, so the buffer is
    zeroed only when it is (re)allocated.  Launches sharing a workspace must be
    ordered (same stream), which is what the per-device default gives.
    """

    _lock = threading.Lock()
    _per_device: dict[int, "DecodeWorkspace"] = {}

    def __init__(self, device: torch.device):
        self.device = device
        self.buffer = torch.empty(0, dtype=torch.uint8, device=device)

    @classmethod
    def for_device(cls, device: torch.device) -> "DecodeWorkspace":
        idx = device.index if device.index is not None else torch.cuda.current_device()
        with cls._lock:
            ws = cls._per_device.get(idx)
            if ws is None:
                ws = cls._per_device[idx] = DecodeWorkspace(torch.device("cuda", idx))
            return ws

    def get(self, nbytes: int, batch: int, hkv: int) -> torch.Tensor:
        if self.buffer.numel() < nbytes:
            self.buffer = torch.empty(max(nbytes, 2 * self.buffer.numel()), dtype=torch.uint8, device=self.device)
            lib = _native.load()
            # zero the whole buffer once: covers the counters of any later, larger batch too
            self.buffer.zero_()
        return self.buffer


@functools.lru_cache(maxsize=256)
def decode_workspace_bytes(batch: int, q_heads: int, hkv: int, head_dim: int, block_size: int, max_context: int,
                           dtype: torch.dtype) -> int:
    lib = _native.load()
    return int(lib.psb_paged_decode_workspace_size(batch, q_heads, hkv, head_dim, block_size, max_context,
                                                   dtype_code(dtype)))


def paged_decode(query: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor, block_tables: torch.Tensor,
                 context_lens: torch.Tensor, layer: int, scale: float | None = None, out: torch.Tensor | None = None,
                 max_context: int | None = None, workspace: torch.Tensor | None = None,
                 error_flag: torch.Tensor | None = None, new_key: torch.Tensor | None = None,
                 new_value: torch.Tensor | None = None) -> torch.Tensor:
    """Decode attention for ``query [B, Hq, D]`` (or ``[B, Hq, 1, D]``) over the paged pool.

    ``block_tables [B, M]`` int32 and ``context_lens [B]`` int32 live on the
    device; ``max_context`` (default ``M * block_size``) bounds every length.
    With ``new_key`` / ``new_value`` (``[B, Hkv, D]`` or ``[B, Hkv, 1, D]``)
    the same launch first stores row b's new token at position
    ``context_lens[b] - 1`` through its block table (psb_paged_decode_append).
    Returns ``out`` with ``query``'s shape and dtype.
    """
    _require_cuda(query, k_cache, v_cache, block_tables, context_lens)
    nl, nb, hkv, bs, d = _pool_geometry(k_cache, v_cache)
    q3 = query.squeeze(2) if query.ndim == 4 else query
    if q3.ndim != 3 or q3.shape[2] != d:
        raise ValueError("query must be [B, Hq, D] or [B, Hq, 1, D]")
    bsz, hq, _ = q3.shape
    if bsz == 0:
        raise ValueError("Batch must not be empty")
    if hq % hkv:
        raise ValueError("Query heads must be divisible by KV heads")
    if q3.dtype != k_cache.dtype:
        raise ValueError("Query dtype must match cache dtype")
    if q3.stride(2) != 1:
        q3 = q3.contiguous()
    if block_tables.dtype != torch.int32 or block_tables.ndim != 2 or block_tables.shape[0] != bsz:
        raise ValueError("block_tables must be int32 [B, max_blocks]")
    if block_tables.stride(1) != 1:
        block_tables = block_tables.contiguous()
    if context_lens.dtype != torch.int32 or context_lens.shape != (bsz,):
        raise ValueError("context_lens must be int32 [B]")
    context_lens = context_lens.contiguous()
    if not 0 <= layer < nl:
        raise ValueError("Invalid layer")
    if max_context is None:
        max_context = block_tables.shape[1] * bs
    scale = 1.0 / math.sqrt(d) if scale is None else float(scale)
    if out is None:
        out = torch.empty_like(query)
    o3 = out.squeeze(2) if out.ndim == 4 else out
    if o3.shape != q3.shape or o3.stride(2) != 1 or o3.dtype != q3.dtype:
        raise ValueError("out must match query's shape/dtype with unit stride along head_dim")
    need = decode_workspace_bytes(bsz, hq, hkv, d, bs, max_context, q3.dtype)
    if workspace is None:
        workspace = DecodeWorkspace.for_device(query.device).get(need, bsz, hkv)
    lib = _native.load()
    if (new_key is None) != (new_value is None):
        raise ValueError("new_key and new_value go together")
    if new_key is not None:
        _require_cuda(new_key, new_value)
        nk = new_key.squeeze(2) if new_key.ndim == 4 else new_key
        nv = new_value.squeeze(2) if new_value.ndim == 4 else new_value
        for t in (nk, nv):
            if t.shape != (bsz, hkv, d) or t.dtype != q3.dtype or t.stride(2) != 1:
                raise ValueError(f"new K/V must be [{bsz}, {hkv}, {d}] {q3.dtype} with unit stride along head_dim")
        _native.check(lib.psb_paged_decode_append(
            q3.data_ptr(), q3.stride(0), q3.stride(1), o3.data_ptr(), o3.stride(0), o3.stride(1), k_cache.data_ptr(),
            v_cache.data_ptr(), nk.data_ptr(), nk.stride(0), nk.stride(1), nv.data_ptr(), nv.stride(0), nv.stride(1),
            block_tables.data_ptr(), block_tables.stride(0), context_lens.data_ptr(), bsz, hq, layer, nl, nb, hkv, bs,
            d, dtype_code(q3.dtype), int(max_context), scale, workspace.data_ptr(),
            workspace.numel() * workspace.element_size(), _ptr(error_flag), _stream(query.device)),
            "paged_decode_append")
        return out
    _native.check(lib.psb_paged_decode(
        q3.data_ptr(), q3.stride(0), q3.stride(1), o3.data_ptr(), o3.stride(0), o3.stride(1), k_cache.data_ptr(),
        v_cache.data_ptr(), block_tables.data_ptr(), block_tables.stride(0), context_lens.data_ptr(), bsz, hq, layer,
        nl, nb, hkv, bs, d, dtype_code(q3.dtype), int(max_context), scale, workspace.data_ptr(),
        workspace.numel() * workspace.element_size(), _ptr(error_flag), _stream(query.device)), "paged_decode")
    return out


class DecodeLaunch:
    """The launch arguments of one decode batch that stay the same for all
    the layer calls of an iteration (pools, device table and lengths,
    geometry, workspace), kept by the reference-facing wrappers next to the
    batch's metadata as one ``psb_decode_args`` struct, so a repeat layer call
    passes only the query, output, new rows, layer and stream
    (``psb_paged_decode_args``).

    Built from arguments the wrappers have already checked: pools contiguous
    and of the query's dtype, device table ``[B, M]`` int32 with unit inner
    stride and contiguous int32 lengths.  The workspace it sized, and the
    table and lengths, are held here, so a later growth of the per-device
    workspace never leaves this launch pointing at freed memory."""

    __slots__ = ("lib", "k_ptr", "v_ptr", "batch", "q_heads", "dtype", "dev", "ws", "keep", "args", "args_ptr")

    def __init__(self, k_cache: torch.Tensor, v_cache: torch.Tensor, tables: torch.Tensor, lengths: torch.Tensor,
                 batch: int, q_heads: int, max_context: int, dtype: torch.dtype):
        nl, nb, hkv, bs, d = (int(x) for x in k_cache.shape)
        if not (k_cache.is_contiguous() and v_cache.is_contiguous()):
            raise ValueError("KV pools must be contiguous")
        self.lib = _native.load()
        self.k_ptr, self.v_ptr = k_cache.data_ptr(), v_cache.data_ptr()
        self.batch, self.q_heads, self.dtype = int(batch), int(q_heads), dtype
        self.dev = k_cache.device.index if k_cache.device.index is not None else torch.cuda.current_device()
        need = decode_workspace_bytes(self.batch, self.q_heads, hkv, d, bs, int(max_context), dtype)
        self.ws = DecodeWorkspace.for_device(k_cache.device).get(need, self.batch, hkv)
        self.keep = (tables, lengths)
        self.args = _native.DecodeArgs(
            k_cache=self.k_ptr, v_cache=self.v_ptr, block_tables=tables.data_ptr(), table_stride=tables.stride(0),
            context_lens=lengths.data_ptr(), num_blocks=nb, workspace=self.ws.data_ptr(),
            workspace_bytes=self.ws.numel() * self.ws.element_size(), error_flag=None, batch=self.batch,
            q_heads=self.q_heads, num_layers=nl, num_kv_heads=hkv, block_size=bs, head_dim=d,
            dtype=_DTYPES[dtype], max_context=int(max_context), scale=1.0 / math.sqrt(d), reserved=0)
        self.args_ptr = ctypes.addressof(self.args)

    def with_lengths(self, lengths: torch.Tensor) -> "DecodeLaunch":
        """The same launch over another lengths array (contiguous int32 [B]
        on the same device) with the same table and bound."""
        new = object.__new__(DecodeLaunch)
        for name in ("lib", "k_ptr", "v_ptr", "batch", "q_heads", "dtype", "dev", "ws"):
            setattr(new, name, getattr(self, name))
        new.keep = (self.keep[0], lengths)
        new.args = _native.DecodeArgs.from_buffer_copy(self.args)
        new.args.context_lens = lengths.data_ptr()
        new.args_ptr = ctypes.addressof(new.args)
        return new

    def matches(self, k_cache: torch.Tensor, v_cache: torch.Tensor, query: torch.Tensor) -> bool:
        return (k_cache.data_ptr() == self.k_ptr and v_cache.data_ptr() == self.v_ptr
                and query.shape[0] == self.batch and query.shape[1] == self.q_heads and query.dtype == self.dtype)

    def __call__(self, query: torch.Tensor, layer: int, new_key: torch.Tensor | None = None,
                 new_value: torch.Tensor | None = None) -> torch.Tensor:
        """Decode (with ``new_key``/``new_value``: the fused write + decode)
        for ``query [B, Hq, (1,) D]``; returns a new output of its shape."""
        if query.stride(-1) != 1:
            query = query.contiguous()
        out = torch.empty_like(query)
        stream = _raw_stream(self.dev) if _raw_stream is not None else torch.cuda.current_stream(self.dev).cuda_stream
        if new_key is None:
            _native.check(self.lib.psb_paged_decode_args(
                self.args_ptr, query.data_ptr(), query.stride(0), query.stride(1), out.data_ptr(), out.stride(0),
                out.stride(1), None, 0, 0, None, 0, 0, layer, stream), "paged_decode")
            return out
        if new_key.stride(-1) != 1:
            new_key = new_key.contiguous()
        if new_value.stride(-1) != 1:
            new_value = new_value.contiguous()
        _native.check(self.lib.psb_paged_decode_args(
            self.args_ptr, query.data_ptr(), query.stride(0), query.stride(1), out.data_ptr(), out.stride(0),
            out.stride(1), new_key.data_ptr(), new_key.stride(0), new_key.stride(1), new_value.data_ptr(),
            new_value.stride(0), new_value.stride(1), layer, stream), "paged_decode_append")
        return out


def varlen_prefill(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, cu_seqlens: torch.Tensor, max_seqlen: int,
                   scale: float | None = None, out: torch.Tensor | None = None,
                   error_flag: torch.Tensor | None = None) -> torch.Tensor:
    """Packed causal prefill: ``q [T, Hq, D]``, ``k, v [T, Hkv, D]``, ``cu_seqlens [B+1]`` int32."""
    _require_cuda(q, k, v, cu_seqlens)
    if q.ndim != 3 or k.ndim != 3 or v.shape != k.shape or q.shape[0] != k.shape[0] or q.shape[2] != k.shape[2]:
        raise ValueError("q must be [T, Hq, D] and k, v [T, Hkv, D]")
    t, hq, d = q.shape
    hkv = k.shape[1]
    if hq % hkv:
        raise ValueError("Query heads must be divisible by KV heads")
    if not (q.dtype == k.dtype == v.dtype):
        raise ValueError("q, k, v dtypes differ")
    if cu_seqlens.dtype != torch.int32 or cu_seqlens.ndim != 1 or cu_seqlens.shape[0] < 1:
        raise ValueError("cu_seqlens must be int32 [B+1]")
    q, k, v = (x if x.stride(2) == 1 else x.contiguous() for x in (q, k, v))
    cu_seqlens = cu_seqlens.contiguous()
    if out is None:
        out = torch.empty_like(q)
    if out.shape != q.shape or out.stride(2) != 1:
        raise ValueError("out must match q with unit stride along head_dim")
    scale = 1.0 / math.sqrt(d) if scale is None else float(scale)
    lib = _native.load()
    _native.check(lib.psb_varlen_prefill(
        q.data_ptr(), q.stride(0), q.stride(1), k.data_ptr(), k.stride(0), k.stride(1), v.data_ptr(), v.stride(0),
        v.stride(1), out.data_ptr(), out.stride(0), out.stride(1), cu_seqlens.data_ptr(), cu_seqlens.shape[0] - 1,
        t, int(max_seqlen), hq, hkv, d, dtype_code(q.dtype), scale, _ptr(error_flag), _stream(q.device)),
        "varlen_prefill")
    return out


def paged_prefill(q: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor, block_tables: torch.Tensor,
                  context_lens: torch.Tensor, cu_seqlens: torch.Tensor, max_seqlen: int, layer: int,
                  scale: float | None = None, out: torch.Tensor | None = None, max_context: int | None = None,
                  error_flag: torch.Tensor | None = None) -> torch.Tensor:
    """Prefix-aware (chunked) causal prefill over the paged pool.

    ``q [T, Hq, D]`` packs each sequence's new rows (``cu_seqlens [B+1]``
    int32); sequence ``b`` holds ``context_lens[b]`` tokens in the pool,
    read through ``block_tables[b]``, its query rows being the last
    ``cu_seqlens[b+1] - cu_seqlens[b]`` of them (their K/V already written,
    e.g. by ``rope_reshape_and_cache``).  Row ``i`` of sequence ``b`` attends
    to positions ``0 .. context_lens[b] - n_b + i``: the reference's
    ``paged_attention(query, cache, request, layer, query_start_position)``
    (pagedserve/attention/paged_attention.py:10-146) for a whole batch.
    """
    _require_cuda(q, k_cache, v_cache, block_tables, context_lens, cu_seqlens)
    nl, nb, hkv, bs, d = _pool_geometry(k_cache, v_cache)
    if q.ndim != 3 or q.shape[2] != d:
        raise ValueError(f"q must be [T, Hq, {d}]")
    t, hq, _ = q.shape
    if hq % hkv:
        raise ValueError("Query heads must be divisible by KV heads")
    if q.dtype != k_cache.dtype:
        raise ValueError("q dtype must match the cache dtype")
    if cu_seqlens.dtype != torch.int32 or cu_seqlens.ndim != 1 or cu_seqlens.shape[0] < 1:
        raise ValueError("cu_seqlens must be int32 [B+1]")
    batch = cu_seqlens.shape[0] - 1
    if block_tables.dtype != torch.int32 or block_tables.ndim != 2 or block_tables.shape[0] != batch:
        raise ValueError("block_tables must be int32 [B, max_blocks]")
    if context_lens.dtype != torch.int32 or context_lens.shape != (batch,):
        raise ValueError("context_lens must be int32 [B]")
    if not 0 <= layer < nl:
        raise ValueError("Invalid layer")
    if q.stride(2) != 1:
        q = q.contiguous()
    if block_tables.stride(1) != 1:
        block_tables = block_tables.contiguous()
    cu_seqlens, context_lens = cu_seqlens.contiguous(), context_lens.contiguous()
    if max_context is None:
        max_context = block_tables.shape[1] * bs
    if out is None:
        out = torch.empty_like(q)
    if out.shape != q.shape or out.stride(2) != 1 or out.dtype != q.dtype:
        raise ValueError("out must match q with unit stride along head_dim")
    scale = 1.0 / math.sqrt(d) if scale is None else float(scale)
    lib = _native.load()
    _native.check(lib.psb_paged_prefill(
        q.data_ptr(), q.stride(0), q.stride(1), k_cache.data_ptr(), v_cache.data_ptr(), block_tables.data_ptr(),
        block_tables.stride(0), context_lens.data_ptr(), out.data_ptr(), out.stride(0), out.stride(1),
        cu_seqlens.data_ptr(), batch, t, int(max_seqlen), int(max_context), hq, layer, nl, nb, hkv, bs, d,
        dtype_code(q.dtype), scale, _ptr(error_flag), _stream(q.device)), "paged_prefill")
    return out


def pack_step(table_store: torch.Tensor, req_rows: torch.Tensor, starts: torch.Tensor, query_lens: torch.Tensor,
              total: int, block_size: int, out_width: int | None = None, error_flag: torch.Tensor | None = None,
              out: tuple | None = None):
    """Build one step's ragged-batch metadata on the GPU.

    ``table_store [R, W]`` int32 holds every live request's block table (one
    row each); ``req_rows, starts, query_lens [B]`` int32 are the scheduler's
    step plan.  Returns ``(cu_seqlens, context_lens, slot_mapping, positions,
    block_tables)``, written into ``out`` (the same five tensors, e.g. the
    static buffers of a captured step) when given.
    """
    _require_cuda(table_store, req_rows, starts, query_lens)
    for name, x in (("req_rows", req_rows), ("starts", starts), ("query_lens", query_lens)):
        if x.dtype != torch.int32 or x.ndim != 1:
            raise ValueError(f"{name} must be int32 [B]")
    if table_store.dtype != torch.int32 or table_store.ndim != 2 or table_store.stride(1) != 1:
        raise ValueError("table_store must be int32 [R, W] with unit column stride")
    bsz = req_rows.shape[0]
    out_width = table_store.shape[1] if out_width is None else int(out_width)
    dev = table_store.device
    if out is None:
        cu = torch.empty(bsz + 1, dtype=torch.int32, device=dev)
        ctx = torch.empty(bsz, dtype=torch.int32, device=dev)
        slots = torch.empty(total, dtype=torch.int64, device=dev)
        pos = torch.empty(total, dtype=torch.int64, device=dev)
        tables = torch.empty((bsz, out_width), dtype=torch.int32, device=dev)
    else:
        cu, ctx, slots, pos, tables = out
        ok = (cu.shape == (bsz + 1,) and cu.dtype == torch.int32 and ctx.shape == (bsz,) and ctx.dtype == torch.int32
              and slots.shape == (total,) and slots.dtype == torch.int64 and pos.shape == (total,)
              and pos.dtype == torch.int64 and tables.shape == (bsz, out_width) and tables.dtype == torch.int32
              and all(t.is_contiguous() for t in out))
        if not ok:
            raise ValueError("out must be contiguous (cu_seqlens [B+1] i32, context_lens [B] i32, slot_mapping [T] "
                             "i64, positions [T] i64, block_tables [B, out_width] i32)")
    lib = _native.load()
    _native.check(lib.psb_pack_step(
        table_store.data_ptr(), table_store.stride(0), table_store.shape[0], req_rows.contiguous().data_ptr(),
        starts.contiguous().data_ptr(), query_lens.contiguous().data_ptr(), bsz, int(total), int(block_size),
        cu.data_ptr(), ctx.data_ptr(), slots.data_ptr(), pos.data_ptr(), tables.data_ptr(), out_width,
        _ptr(error_flag), _stream(dev)), "pack_step")
    return cu, ctx, slots, pos, tables


def add_rms_norm(x: torch.Tensor, weight: torch.Tensor, eps: float, residual: torch.Tensor | None = None,
                 out: torch.Tensor | None = None) -> torch.Tensor:
    """RMSNorm of ``x [R, H]`` (Qwen2RMSNorm), or, with ``residual [R, H]``,
    ``residual += x`` (rounded, in place) followed by RMSNorm of the sum, in
    one launch (psb_add_rms_norm).  Returns ``out``."""
    _require_cuda(x, weight)
    if x.ndim != 2 or weight.shape != (x.shape[1],):
        raise ValueError("x must be [R, H] and weight [H]")
    if x.stride(1) != 1 or weight.stride(0) != 1:
        raise ValueError("x and weight need unit stride along H")
    if out is None:
        out = torch.empty_like(x)
    for t in (out,) + ((residual,) if residual is not None else ()):
        if t.shape != x.shape or t.dtype != x.dtype or t.stride(1) != 1:
            raise ValueError("out / residual must match x's shape and dtype with unit stride along H")
    if weight.dtype != x.dtype:
        raise ValueError("weight dtype must match x")
    lib = _native.load()
    _native.check(lib.psb_add_rms_norm(
        x.data_ptr(), x.stride(0), _ptr(residual), residual.stride(0) if residual is not None else 0,
        weight.data_ptr(), out.data_ptr(), out.stride(0), x.shape[0], x.shape[1], float(eps), dtype_code(x.dtype),
        _stream(x.device)), "add_rms_norm")
    return out


def silu_and_mul(gate_up: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
    """``silu(gate) * up`` of a fused ``gate_up [R, 2I]`` projection -> ``[R, I]`` (psb_silu_and_mul)."""
    _require_cuda(gate_up)
    if gate_up.ndim != 2 or gate_up.shape[1] % 2 or gate_up.stride(1) != 1:
        raise ValueError("gate_up must be [R, 2 * I] with unit column stride")
    rows, inter = gate_up.shape[0], gate_up.shape[1] // 2
    if out is None:
        out = torch.empty((rows, inter), dtype=gate_up.dtype, device=gate_up.device)
    if out.shape != (rows, inter) or out.dtype != gate_up.dtype or out.stride(1) != 1:
        raise ValueError(f"out must be [{rows}, {inter}] of gate_up's dtype with unit column stride")
    lib = _native.load()
    _native.check(lib.psb_silu_and_mul(gate_up.data_ptr(), gate_up.stride(0), out.data_ptr(), out.stride(0), rows,
                                       inter, dtype_code(gate_up.dtype), _stream(gate_up.device)), "silu_and_mul")
    return out


SELECT_DONE, SELECT_EOS, SELECT_LIMIT = 1, 2, 4


def select_tokens(logits: torch.Tensor, eos_ids: torch.Tensor, remaining: torch.Tensor,
                  tokens: torch.Tensor | None = None, status: torch.Tensor | None = None,
                  error_flag: torch.Tensor | None = None, ctas_per_row: int = 0) -> tuple[torch.Tensor, torch.Tensor]:
    """Greedy next token of every row and the reference's stop test, in one launch.

    ``logits`` is ``[B, V]`` or the model's ``[B, S, V]`` (the last position is
    used, as ``logits[:, -1, :]``), unit stride along V.  ``eos_ids`` int64
    ``[E]`` (E <= 64), ``remaining`` int32 ``[B]``: tokens each request may
    still generate, decremented in place.  Returns ``(tokens [B] int64,
    status [B] uint8)``: ``tokens`` is ``argmax(dim=-1)`` with torch's rules
    (first maximum, NaN largest); ``status`` holds SELECT_DONE (the request
    finishes: EOS or its last allowed token), SELECT_EOS, and SELECT_LIMIT
    (no tokens were left: the reference's add_generated_token raises; the
    row is also flagged in ``error_flag`` with 64).
    """
    _require_cuda(logits, eos_ids, remaining)
    if logits.ndim == 3:
        logits = logits[:, -1, :]
    if logits.ndim != 2:
        raise ValueError("logits must be [B, V] or [B, S, V]")
    b, v = int(logits.shape[0]), int(logits.shape[1])
    if v == 0:
        raise ValueError("logits have an empty vocabulary axis")
    if logits.stride(1) != 1:
        logits = logits.contiguous()
    if eos_ids.dtype != torch.int64 or eos_ids.ndim != 1 or eos_ids.shape[0] > 64:
        raise ValueError("eos_ids must be int64 [E] with E <= 64")
    if not eos_ids.is_contiguous():
        eos_ids = eos_ids.contiguous()
    if remaining.dtype != torch.int32 or remaining.shape != (b,) or not remaining.is_contiguous():
        raise ValueError("remaining must be a contiguous int32 [B] tensor (updated in place)")
    if tokens is None:
        tokens = torch.empty(b, dtype=torch.int64, device=logits.device)
    if status is None:
        status = torch.empty(b, dtype=torch.uint8, device=logits.device)
    if tokens.dtype != torch.int64 or tokens.shape != (b,) or not tokens.is_contiguous():
        raise ValueError("tokens must be a contiguous int64 [B] tensor")
    if status.dtype != torch.uint8 or status.shape != (b,) or not status.is_contiguous():
        raise ValueError("status must be a contiguous uint8 [B] tensor")
    if not 0 <= ctas_per_row <= 8:
        raise ValueError("ctas_per_row must be 0 (auto) or 1..8")
    if b == 0:
        return tokens, status
    row_stride = int(logits.stride(0)) if b > 1 else v
    lib = _native.load()
    _native.check(lib.psb_select_tokens(
        logits.data_ptr(), row_stride, b, v, dtype_code(logits.dtype), eos_ids.data_ptr() if eos_ids.numel() else None,
        int(eos_ids.shape[0]), remaining.data_ptr(), tokens.data_ptr(), status.data_ptr(), ctas_per_row,
        _ptr(error_flag), _stream(logits.device)), "select_tokens")
    return tokens, status
