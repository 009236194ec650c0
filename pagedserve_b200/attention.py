"""Reference-facing attention entry points (the drop-in boundary).

``paged_decode_attention`` has exactly the signature, argument meaning and
``ValueError`` conditions/messages of the reference's Triton wrapper
``triton_paged_decode_attention`` (pagedserve/attention/triton_paged_decode.py:98-173),
so PagedServe's decode glue can call it in place of the Triton kernel:

    pagedserve.attention.batched_paged_attention.triton_paged_decode_attention = paged_decode_attention

Differences are internal: the per-row host loop that builds the padded table
is one numpy pass and one host->device copy of (table, lengths), and the
attention runs in the sm_100a split-K kernel of ``libpagedserve_b200.so``.
``write_tokens`` replaces the per-row ``write_token`` loop
(pagedserve/attention/batched_paged_attention.py:115-124) with one
``reshape_and_cache`` launch.

The reference rebuilds the table for every layer of every decode iteration
(triton_paged_decode.py:134-154) although all layers of one iteration see the
same requests, positions and blocks.  With this package's ``PagedKVCache``,
whose ``metadata_epoch`` changes on every allocation, growth or release, the
device copies (table, lengths, slots) are kept on the cache object and reused
while the epoch, the request ids and the positions are unchanged; any other
cache object is rebuilt on every call, as in the reference.
"""

from __future__ import annotations

from collections import OrderedDict
from collections.abc import Sequence

import numpy as np
import torch

from . import ops


_KEEP = 4  # metadata entries kept per cache (one per live batch shape)

# triton_paged_decode.py:106-107 raises exactly this text for a host query
_CUDA_REQUIRED = "Triton paged attention requires CUDA"
_QUERY_DTYPES = (torch.float32, torch.float16, torch.bfloat16)


def _memo(cache, kind: str, request_ids, positions, device, build):
    """``build()``, or its result from an earlier call at the same cache
    epoch for the same requests, positions and device.

    The layer calls of one decode iteration pass the same lists: the last
    result per kind is checked first with two list comparisons (C speed),
    before the keyed store."""
    epoch = getattr(cache, "metadata_epoch", None)
    if epoch is None:
        return build()
    dev = _dev_key(device)
    lists = type(request_ids) is list and type(positions) is list
    last = getattr(cache, "_psb_last", None)
    if last is None:
        last = cache._psb_last = {}
    if lists:
        hit = last.get(kind)
        if hit is not None and hit[0] == epoch and hit[1] == dev and hit[2] == request_ids and hit[3] == positions:
            return hit[4]
    store = getattr(cache, "_psb_metadata", None)
    if store is None:
        store = cache._psb_metadata = OrderedDict()
    # tuples built at C speed (numpy and Python integers hash alike)
    key = (kind, epoch, tuple(request_ids), tuple(positions), dev)
    value = store.get(key)
    if value is not None:
        store.move_to_end(key)
    else:
        value = build()
        store[key] = value
        while len(store) > _KEEP:
            store.popitem(last=False)
    if lists:
        last[kind] = (epoch, dev, list(request_ids), list(positions), value)
    return value


def _dev_key(device) -> int:
    """A device as a plain integer (CUDA index, -1 for the CPU): cheap to compare."""
    if isinstance(device, int):
        return device
    return device.index if device.type == "cuda" and device.index is not None else (
        torch.cuda.current_device() if device.type == "cuda" else -1)


def _last_hit(cache, kind: str, request_ids, positions, dev: int):
    """The metadata the last call of this kind built for the same epoch,
    request list and positions on device index ``dev``, or None (two list
    comparisons)."""
    last = getattr(cache, "_psb_last", None)
    if last is None or type(request_ids) is not list or type(positions) is not list:
        return None
    hit = last.get(kind)
    if (hit is not None and hit[0] == getattr(cache, "metadata_epoch", None) and hit[1] == dev
            and hit[2] == request_ids and hit[3] == positions):
        return hit[4]
    return None


def clear_metadata_cache(cache) -> None:
    """Drop the device copies of block tables, lengths and slots kept on ``cache``."""
    store = getattr(cache, "_psb_metadata", None)
    if store is not None:
        store.clear()
    last = getattr(cache, "_psb_last", None)
    if last is not None:
        last.clear()
    if getattr(cache, "_psb_table", None) is not None:
        cache._psb_table = None
    cache._psb_fast = None


def _host_metadata(cache, request_ids, positions, device):
    """(table [B, M] int32, lengths [B] int32) as one device tensor pair.

    Raises the reference's position error (triton_paged_decode.py:134-141).
    """
    return _memo(cache, "table", request_ids, positions, device,
                 lambda: _build_metadata(cache, request_ids, positions, device))


def _build_metadata(cache, request_ids, positions, device):
    if hasattr(cache, "gather_tables"):
        # this package's PagedKVCache: vectorised over its table store, the
        # table gathered straight into pinned memory as [table (B x W) | lengths (B)]
        b = len(request_ids)
        table = _table_for(cache, request_ids, device)
        if table is not None:
            tables, width, rows, counts, holder = table
            return _Meta(tables, _upload_lengths(cache, holder, positions, counts, request_ids, device), width,
                         holder)
        # the batch's device table, kept per (epoch, request list): within an
        # epoch the blocks do not change (the scheduler reserves a request's
        # whole capacity when it admits it), so the decode iterations that
        # follow upload only the lengths
        pos = np.fromiter(positions, dtype=np.int64, count=b)
        rows = cache.table_store_rows(request_ids)
        counts = cache.store_token_counts(rows)
        _check_positions(pos, counts, positions, request_ids)
        width = cache.table_width(rows)
        host, done = _staging(cache, b * (width + 1), device)
        flat = host.numpy()
        cache.gather_tables(rows, flat, width)
        flat[b * width:] = pos + 1
        dev = host.to(device, non_blocking=True)
        done()
        tables = dev[: b * width].view(b, width)
        # [launch struct of the first call over this table (a template for
        # the next), lengths ring (added by the first new-positions upload)]
        holder = [None]
        cache._psb_table = (cache.metadata_epoch, device, list(request_ids), tables, width, rows, counts, holder)
        return _Meta(tables, dev[b * width:], width, holder)
    else:
        # any cache with the reference's interface
        lengths = np.empty(len(request_ids), dtype=np.int32)
        tables = []
        for row, (rid, pos) in enumerate(zip(request_ids, positions)):
            count = cache.token_count(rid)
            if not 0 <= pos < count:
                raise ValueError(f"Invalid position {pos} for {rid}")
            lengths[row] = pos + 1
            tables.append(cache.get_block_table(rid).get_blocks())
        width = max(len(t) for t in tables)
        packed = np.zeros((len(tables), width + 1), dtype=np.int32)  # [table | length]
        for row, t in enumerate(tables):
            packed[row, : len(t)] = t
        packed[:, width] = lengths
    host = torch.from_numpy(packed)
    if device.type == "cuda":
        host = host.pin_memory()
    dev = host.to(device, non_blocking=True)
    return _Meta(dev[:, :width], dev[:, width].contiguous(), width)


def _staging(cache, n: int, device):
    """An int32 host buffer of ``n`` elements for a metadata upload, and the
    function to call once its copy has been issued.

    For a CUDA device: pinned memory from a ring of two buffers kept on the
    cache object (pinning memory costs far more than the copy); a buffer is
    reused only after the copy issued from it has completed (an event)."""
    if device.type != "cuda":
        return torch.empty(n, dtype=torch.int32), (lambda: None)
    ring = getattr(cache, "_psb_staging", None)
    if ring is None:
        # [buffer, event, event recorded] x 2, next slot; an event per slot, made once
        ring = cache._psb_staging = [[None, torch.cuda.Event(), False], [None, torch.cuda.Event(), False], 0]
    slot = ring[2]
    ring[2] = 1 - slot
    entry = ring[slot]
    buf, ev = entry[0], entry[1]
    if entry[2]:
        ev.synchronize()  # normally long complete: the slot was used an iteration ago
    if buf is None or buf.numel() < n:
        buf = torch.empty(max(n, 2 * (buf.numel() if buf is not None else 0)), dtype=torch.int32, pin_memory=True)
        entry[0] = buf

    def done():
        ev.record(torch.cuda.current_stream(device))
        entry[2] = True

    return buf[:n], done


def _table_for(cache, request_ids, device):
    """(tables, width, store rows, token counts, launch template holder)
    built earlier in this epoch for this request list on this device, or None."""
    kept = getattr(cache, "_psb_table", None)
    if kept is None or kept[0] != cache.metadata_epoch or kept[1] != device or kept[2] != request_ids:
        return None
    return kept[3:]


_LEN_SLOTS = 4  # pinned lengths rows per device table, filled in turn


def _upload_lengths(cache, holder, positions, counts, request_ids, device):
    """The device lengths (``positions[b] + 1``, int32) of a new decode
    iteration over a device table kept for this epoch, after the reference's
    position check.

    Each table keeps a ring of ``_LEN_SLOTS`` pinned host rows: the positions
    are written straight into the next row, checked with one unsigned
    comparison against the token counts (a negative position wraps above
    every count), turned into lengths in place and copied on the current
    stream to a device array of their own (kept metadata may outlive any
    number of later iterations).  A host row is refilled only after its
    previous copy has completed (an event per row)."""
    b = len(request_ids)
    if device.type != "cuda":  # host metadata (tests of the table logic): no ring
        pos = np.fromiter(positions, dtype=np.int64, count=b)
        _check_positions(pos, counts, positions, request_ids)
        return torch.from_numpy((pos + 1).astype(np.int32))
    ring = holder[1] if len(holder) > 1 else None
    if ring is None:
        host = torch.empty((_LEN_SLOTS, b), dtype=torch.int32, pin_memory=True)
        ring = [host, host.numpy(), None, [torch.cuda.Event() for _ in range(_LEN_SLOTS)], [False] * _LEN_SLOTS, 0,
                np.asarray(counts, dtype=np.int64).clip(0, 2 ** 31 - 1).astype(np.uint32)]
        holder.append(ring)
    host, host_np, _, events, recorded, slot, counts_u32 = ring
    ring[5] = (slot + 1) % _LEN_SLOTS
    if recorded[slot]:
        events[slot].synchronize()  # normally long complete: the row was used several iterations ago
    row = host_np[slot]
    try:
        row[:] = positions
    except (OverflowError, TypeError, ValueError):
        row = None
    if row is None or bool((row.view(np.uint32) >= counts_u32).any()):
        for i, (rid, p) in enumerate(zip(request_ids, positions)):  # the first bad row, as the reference reports it
            if not 0 <= p < int(counts[i]):
                raise ValueError(f"Invalid position {p} for {rid}")
        raise ValueError("Invalid positions")
    row += 1
    out = torch.empty(b, dtype=torch.int32, device=device)
    out.copy_(host[slot], non_blocking=True)
    events[slot].record(torch.cuda.current_stream(device))
    recorded[slot] = True
    return out


def _unique_known(cache, request_ids) -> bool:
    """True when ``request_ids`` is the list the table kept for this epoch
    was built for (a table is built only after the ids passed the uniqueness
    check)."""
    kept = getattr(cache, "_psb_table", None)
    return (kept is not None and kept[0] == getattr(cache, "metadata_epoch", None) and type(request_ids) is list
            and kept[2] == request_ids)


def _check_positions(pos: np.ndarray, counts: np.ndarray, positions, request_ids) -> None:
    """The reference's position check (triton_paged_decode.py:136-139), vectorised."""
    bad = np.flatnonzero((pos < 0) | (pos >= counts))
    if bad.size:
        row = int(bad[0])
        raise ValueError(f"Invalid position {positions[row]} for {request_ids[row]}")


class _Meta:
    """A decode batch's device table and lengths, and the launch arguments
    that stay the same for all layer calls over them (``ops.DecodeLaunch``,
    built on the first call)."""

    __slots__ = ("tables", "lengths", "width", "launch", "holder")

    def __init__(self, tables, lengths, width, holder=None):
        self.tables, self.lengths, self.width = tables, lengths, width
        self.launch = None
        self.holder = holder  # a one-element list shared by the metadata built over the same device table

    def __iter__(self):  # (tables, lengths, width)
        return iter((self.tables, self.lengths, self.width))

    def __getitem__(self, i):
        return (self.tables, self.lengths, self.width)[i]


def paged_decode_attention(query: torch.Tensor, cache, request_ids: Sequence[str], positions: Sequence[int],
                           layer: int) -> torch.Tensor:
    """Decode attention for query ``[B, Hq, 1, D]``, returning the same shape.

    Drop-in for ``triton_paged_decode_attention`` (triton_paged_decode.py:98-104).
    """
    sig = (query.shape, query.dtype, query.get_device())
    meta = _repeat(cache, sig, request_ids, positions, layer)
    if meta is not None:
        return meta.launch(query, layer)
    meta = _validated_metadata(query, cache, request_ids, positions, layer)
    out = _launch(meta, cache, query, layer)
    _remember(cache, sig, meta)
    return out


# The layer calls of one decode iteration repeat the same lists and tensors of
# the same shapes, dtypes and devices.  After a call passed every check, the
# cache keeps (signature of its tensors, its metadata, device, layers, pools);
# a later call whose signature is equal and whose lists hit that same
# metadata has passed the same checks, all but the layer index, which is
# checked here.  Anything else takes the full path and its error messages.
def _repeat(cache, sig, request_ids, positions, layer):
    fast = getattr(cache, "_psb_fast", None)
    if fast is None or fast[0] != sig or not 0 <= layer < fast[3]:
        return None
    kv = cache.kv_cache
    if kv.k_cache is not fast[4] or kv.v_cache is not fast[5]:
        return None
    meta = _last_hit(cache, "table", request_ids, positions, fast[2])
    return meta if meta is fast[1] and meta.launch is not None else None


def _remember(cache, sig, meta) -> None:
    kv = cache.kv_cache
    cache._psb_fast = (sig, meta, sig[2], kv.k_cache.shape[0], kv.k_cache, kv.v_cache)


def _launch(meta: "_Meta", cache, query, layer, new_key=None, new_value=None):
    kv = cache.kv_cache
    launch = meta.launch
    if launch is None or not launch.matches(kv.k_cache, kv.v_cache, query):
        tmpl = meta.holder[0] if meta.holder is not None else None
        if tmpl is not None and tmpl.matches(kv.k_cache, kv.v_cache, query):
            # the same device table: only the lengths differ
            launch = meta.launch = tmpl.with_lengths(meta.lengths)
        else:
            launch = meta.launch = ops.DecodeLaunch(kv.k_cache, kv.v_cache, meta.tables, meta.lengths,
                                                    query.shape[0], query.shape[1], meta.width * cache.block_size,
                                                    query.dtype)
            if meta.holder is not None:
                meta.holder[0] = launch
    return launch(query, layer, new_key, new_value)


def _validated_metadata(query, cache, request_ids, positions, layer):
    """The reference wrapper's checks, in its order and with its messages
    (triton_paged_decode.py:106-141), then the device table and lengths."""
    if not query.is_cuda:
        # the reference wrapper's message, word for word: callers that match
        # on it keep working when this backend replaces the Triton one
        raise ValueError(_CUDA_REQUIRED)
    shape = query.shape
    if len(shape) != 4 or shape[2] != 1:
        raise ValueError("query must have shape [B, Hq, 1, D]")
    dtype = query.dtype
    if dtype not in _QUERY_DTYPES:
        raise ValueError("Unsupported query dtype")
    batch, q_heads, _, head_dim = shape
    kv = cache.kv_cache
    if batch == 0:
        raise ValueError("Batch must not be empty")
    if len(request_ids) != batch or len(positions) != batch:
        raise ValueError("Request IDs and positions must match batch size")
    dev = query.get_device()
    # the metadata of an earlier call with these very lists was built only
    # after they passed every check here, uniqueness included
    meta = _last_hit(cache, "table", request_ids, positions, dev)
    if meta is None and not _unique_known(cache, request_ids) and len(set(request_ids)) != batch:
        raise ValueError("Request IDs must be unique")
    if head_dim != kv.head_dim:
        raise ValueError("Head dimension mismatch")
    if q_heads % kv.num_kv_heads:
        raise ValueError("Query heads must be divisible by KV heads")
    if dtype != kv.dtype:
        raise ValueError("Query dtype must match cache dtype")
    k_cache = kv.k_cache
    if dev != k_cache.get_device():
        raise ValueError("Query and cache must be on the same device")
    if not 0 <= layer < k_cache.shape[0]:
        raise ValueError("Invalid layer")
    if meta is None:
        meta = _host_metadata(cache, request_ids, positions, query.device)
    return meta


def paged_decode_attention_with_write(query: torch.Tensor, key: torch.Tensor, value: torch.Tensor, cache,
                                      request_ids: Sequence[str], positions: Sequence[int],
                                      layer: int) -> torch.Tensor:
    """The decode step's cache write and attention in one launch.

    Same result, and the same pool bytes, as the reference's per-row
    ``write_token(request_id, layer, position, key[b], value[b])`` loop
    (pagedserve/attention/batched_paged_attention.py:115-124) followed by
    ``triton_paged_decode_attention(query, cache, request_ids, positions,
    layer)`` (:126-135): ``key``/``value`` are ``[B, Hkv, D]`` (or
    ``[B, Hkv, 1, D]``) and row b lands at ``positions[b]``, the last position
    the query attends to.  Runs as ``psb_paged_decode_append``.
    """
    sig = (query.shape, query.dtype, query.get_device(), key.shape, key.dtype, key.get_device(), value.shape,
           value.dtype, value.get_device())
    meta = _repeat(cache, sig, request_ids, positions, layer)
    if meta is not None:
        return meta.launch(query, layer, key, value)
    if not query.is_cuda:
        raise ValueError(_CUDA_REQUIRED)
    kv = cache.kv_cache
    shape = (kv.num_kv_heads, kv.head_dim)
    # [B, Hkv, 1, D] as the glue holds them, or [B, Hkv, D]; the launch reads
    # the batch and head strides, which are the same either way
    if _rows_shape(key) != shape or _rows_shape(value) != shape:
        raise ValueError(f"Expected K/V shape {shape}; got key={tuple(key.shape)}, value={tuple(value.shape)}")
    if key.dtype != kv.dtype or value.dtype != kv.dtype:
        raise ValueError(f"K/V tensors must have dtype {kv.dtype}")
    if key.shape[0] != query.shape[0] or value.shape[0] != query.shape[0]:
        raise ValueError("Request IDs and positions must match batch size")
    meta = _validated_metadata(query, cache, request_ids, positions, layer)
    dev = query.get_device()
    if key.get_device() != dev or value.get_device() != dev:
        raise ValueError("new K/V must be on the query's device")
    out = _launch(meta, cache, query, layer, key, value)
    _remember(cache, sig, meta)
    return out


def _rows_shape(t: torch.Tensor) -> tuple:
    """(heads, head_dim) of new rows given as [B, H, D] or [B, H, 1, D] (else a shape that matches nothing)."""
    shp = t.shape
    if len(shp) == 3:
        return (shp[1], shp[2])
    if len(shp) == 4 and shp[2] == 1:
        return (shp[1], shp[3])
    return tuple(shp)


def write_tokens(cache, request_ids: Sequence[str], positions: Sequence[int], layer: int, key: torch.Tensor,
                 value: torch.Tensor) -> None:
    """Write row ``b``'s ``key[b], value[b] [Hkv, D]`` at ``positions[b]`` of
    ``request_ids[b]``, for every row in one launch.

    Same validation as ``PagedKVCache.write_token`` (paged_kv_cache.py:158-185)
    per row, same bytes written (paged_kv_cache.py:187-200).
    """
    kv = cache.kv_cache
    if key.ndim == 4:  # [B, Hkv, 1, D] as produced by the decode glue
        key, value = key.squeeze(2), value.squeeze(2)
    shape = (kv.num_kv_heads, kv.head_dim)
    if tuple(key.shape[1:]) != shape or tuple(value.shape[1:]) != shape:
        raise ValueError(f"Expected K/V shape {shape}; got key={tuple(key.shape)}, value={tuple(value.shape)}")
    if key.dtype != kv.dtype or value.dtype != kv.dtype:
        raise ValueError(f"K/V tensors must have dtype {kv.dtype}")

    slot_t = _slots(cache, request_ids, positions, key.device)
    ops.reshape_and_cache(key, value, kv.k_cache, kv.v_cache, slot_t, layer)


def rope_and_write_tokens(query: torch.Tensor, key: torch.Tensor, value: torch.Tensor, cos: torch.Tensor,
                          sin: torch.Tensor, cache, request_ids: Sequence[str], positions: Sequence[int],
                          layer: int) -> torch.Tensor:
    """The decode glue's rotary embedding and KV write in one launch.

    Replaces ``apply_rotary_pos_emb(query, key, cos, sin)`` followed by the
    per-row ``write_token`` loop (pagedserve/attention/batched_paged_attention.py:105-124):
    ``query [B, Hq, 1, D]``, ``key``/``value [B, Hkv, 1, D]`` as the glue
    holds them, ``cos``/``sin`` the engine's position embeddings (one
    ``[D]`` row per batch row).  Writes the rotated key and the value of row b
    at ``positions[b]`` and returns the rotated query, bit-identical to the
    reference's (psb_rope_reshape_and_cache).
    """
    kv = cache.kv_cache
    if query.ndim != 4 or query.shape[2] != 1:
        raise ValueError("query must have shape [B, Hq, 1, D]")
    batch = query.shape[0]
    if key.ndim == 4:
        key, value = key.squeeze(2), value.squeeze(2)
    shape = (kv.num_kv_heads, kv.head_dim)
    if tuple(key.shape[1:]) != shape or tuple(value.shape[1:]) != shape or key.shape[0] != batch:
        raise ValueError(f"Expected K/V shape {shape}; got key={tuple(key.shape)}, value={tuple(value.shape)}")
    if len(request_ids) != batch or len(positions) != batch:
        raise ValueError("Request IDs and positions must match batch size")
    slot_t = _slots(cache, request_ids, positions, key.device)
    q_rot, _ = ops.rope_reshape_and_cache(query.squeeze(2), key, value, cos.reshape(batch, -1),
                                          sin.reshape(batch, -1), kv.k_cache, kv.v_cache, slot_t, layer,
                                          key_out=False)
    return q_rot.unsqueeze(2)


def _slots(cache, request_ids, positions, device):
    """Device int64 slots of (request, position) pairs, reused within an epoch."""
    def build():
        slots = np.fromiter((cache.slot_of(r, p) if hasattr(cache, "slot_of") else _slot(cache, r, p)
                             for r, p in zip(request_ids, positions)), dtype=np.int64, count=len(request_ids))
        host = torch.from_numpy(slots)
        if device.type == "cuda":
            host = host.pin_memory()
        return host.to(device, non_blocking=True)

    return _memo(cache, "slots", request_ids, positions, device, build)


def _slot(cache, request_id: str, position: int) -> int:
    """Slot of a position for a reference ``PagedKVCache`` (paged_kv_cache.py:187-192)."""
    count = cache.token_count(request_id)
    if not 0 <= position < count:
        raise IndexError(f"Invalid token position: {position}; valid range is [0, {count})")
    bs = cache.block_size
    return cache.get_block_table(request_id).get_physical_block(position // bs) * bs + position % bs
