"""Host-side paged-KV bookkeeping with PagedServe's interface.

The B200 kernels address the pool through block tables; this module owns
them.  Class names, method names, argument meaning and the exception types
raised follow the reference so callers can switch without edits:

* ``BlockManager``  - pagedserve/engine/block_manager.py:6-155 (FIFO free list:
  allocation takes from the head, ``free`` returns blocks to the tail)
* ``BlockTable``    - pagedserve/engine/block_table.py:4-49
* ``KVCache``       - pagedserve/engine/kv_cache.py:6-164, layout
  ``[layer, physical_block, kv_head, token_in_block, head_dim]``
* ``PagedKVCache``  - pagedserve/engine/paged_kv_cache.py:10-233

Added for the batched path: ``PagedKVCache.table_rows`` (a padded int32
table for a list of requests, built in one numpy pass) and
``PagedKVCache.slot_of`` (the int64 slot a position maps to).
"""

from __future__ import annotations

from collections import deque

import numpy as np
import torch


class BlockManager:
    """Ownership of physical KV blocks; allocates no tensors."""

    def __init__(self, num_blocks: int, block_size: int = 16, free_order=None):
        if num_blocks <= 0:
            raise ValueError("num_blocks must be positive")
        if block_size <= 0:
            raise ValueError("block_size must be positive")
        self.num_blocks = num_blocks
        self.block_size = block_size
        # ``free_order`` (a permutation of the block ids) seeds the free list in
        # another order, e.g. a shuffled pool for fragmentation studies.
        order = range(num_blocks) if free_order is None else [int(b) for b in free_order]
        if free_order is not None and sorted(order) != list(range(num_blocks)):
            raise ValueError("free_order must be a permutation of range(num_blocks)")
        self._free: deque[int] = deque(order)
        self._owned: dict[str, list[int]] = {}

    @property
    def free_blocks(self) -> int:
        return len(self._free)

    @property
    def used_blocks(self) -> int:
        return self.num_blocks - len(self._free)

    def blocks_needed(self, num_tokens: int) -> int:
        """ceil(num_tokens / block_size); 0 tokens need 0 blocks."""
        if num_tokens < 0:
            raise ValueError("num_tokens cannot be negative")
        return -(-num_tokens // self.block_size)

    def _take(self, count: int) -> list[int]:
        if count > len(self._free):
            raise RuntimeError(f"Not enough KV blocks: required={count}, free={len(self._free)}")
        return [self._free.popleft() for _ in range(count)]

    def allocate(self, request_id: str, num_tokens: int) -> list[int]:
        """Blocks for a new request, taken from the head of the free list."""
        if request_id in self._owned:
            raise ValueError(f"Request {request_id!r} already has blocks")
        blocks = self._take(self.blocks_needed(num_tokens))
        self._owned[request_id] = blocks
        return list(blocks)

    def allocate_blocks(self, request_id: str, num_blocks: int) -> list[int]:
        """Additional blocks for an existing request."""
        if request_id not in self._owned:
            raise KeyError(f"Unknown request: {request_id!r}")
        if num_blocks <= 0:
            raise ValueError("num_blocks must be positive")
        blocks = self._take(num_blocks)
        self._owned[request_id].extend(blocks)
        return list(blocks)

    def free(self, request_id: str) -> None:
        """Return all of a request's blocks to the tail of the free list."""
        if request_id not in self._owned:
            raise KeyError(f"Unknown request: {request_id!r}")
        self._free.extend(self._owned.pop(request_id))

    def get_blocks(self, request_id: str) -> list[int]:
        if request_id not in self._owned:
            raise KeyError(f"Unknown request: {request_id!r}")
        return list(self._owned[request_id])

    def has_request(self, request_id: str) -> bool:
        return request_id in self._owned


class BlockTable:
    """Logical -> physical block map of one request."""

    def __init__(self) -> None:
        self._blocks: list[int] = []
        self._owner: "PagedKVCache | None" = None  # told of every change (metadata epoch, table store)
        self._row = -1                              # this table's row in the owner's table store

    @property
    def num_blocks(self) -> int:
        return len(self._blocks)

    def append(self, physical_block_id: int) -> None:
        if physical_block_id < 0:
            raise ValueError("physical_block_id cannot be negative")
        self._blocks.append(physical_block_id)
        if self._owner is not None:
            self._owner._store_put(self._row, len(self._blocks) - 1, physical_block_id)
            self._owner._epoch += 1

    def get_physical_block(self, logical_block_id: int) -> int:
        if not 0 <= logical_block_id < len(self._blocks):
            raise IndexError(f"Invalid logical block: {logical_block_id}; valid range is [0, {len(self._blocks)})")
        return self._blocks[logical_block_id]

    def get_blocks(self) -> list[int]:
        return list(self._blocks)

    def clear(self) -> None:
        self._blocks.clear()
        if self._owner is not None:
            self._owner._store_clear(self._row)
            self._owner._epoch += 1


class KVCache:
    """The K and V pools, ``[num_layers, num_blocks, num_kv_heads, block_size, head_dim]`` each."""

    def __init__(self, num_blocks: int, num_layers: int, num_kv_heads: int, head_dim: int, block_size: int = 16,
                 dtype: torch.dtype = torch.bfloat16, device: str | torch.device = "cuda"):
        for name, val in (("num_blocks", num_blocks), ("num_layers", num_layers), ("num_kv_heads", num_kv_heads),
                          ("head_dim", head_dim), ("block_size", block_size)):
            if val <= 0:
                raise ValueError(f"{name} must be positive")
        self.num_blocks = num_blocks
        self.num_layers = num_layers
        self.num_kv_heads = num_kv_heads
        self.head_dim = head_dim
        self.block_size = block_size
        self.dtype = dtype
        self.device = torch.device(device)
        shape = (num_layers, num_blocks, num_kv_heads, block_size, head_dim)
        self.k_cache = torch.empty(shape, dtype=dtype, device=self.device)
        self.v_cache = torch.empty(shape, dtype=dtype, device=self.device)

    @property
    def block_shape(self) -> tuple[int, ...]:
        return (self.num_kv_heads, self.block_size, self.head_dim)

    @property
    def block_bytes(self) -> int:
        """K+V bytes of one physical block across all layers."""
        esz = torch.empty((), dtype=self.dtype).element_size()
        return self.num_layers * 2 * self.num_kv_heads * self.block_size * self.head_dim * esz

    @property
    def total_bytes(self) -> int:
        return self.num_blocks * self.block_bytes

    def _check_layer(self, layer: int) -> None:
        if not 0 <= layer < self.num_layers:
            raise IndexError(f"Invalid layer: {layer}; valid range is [0, {self.num_layers})")

    def _check_block(self, block_id: int) -> None:
        if not 0 <= block_id < self.num_blocks:
            raise IndexError(f"Invalid block ID: {block_id}; valid range is [0, {self.num_blocks})")

    def write_block(self, layer: int, block_id: int, key: torch.Tensor, value: torch.Tensor) -> None:
        self._check_layer(layer)
        self._check_block(block_id)
        for name, t in (("key", key), ("value", value)):
            if tuple(t.shape) != self.block_shape:
                raise ValueError(f"Invalid {name} shape: expected {self.block_shape}, got {tuple(t.shape)}")
            if t.dtype != self.dtype:
                raise ValueError(f"Invalid {name} dtype: expected {self.dtype}, got {t.dtype}")
        self.k_cache[layer, block_id].copy_(key)
        self.v_cache[layer, block_id].copy_(value)

    def read_block(self, layer: int, block_id: int) -> tuple[torch.Tensor, torch.Tensor]:
        self._check_layer(layer)
        self._check_block(block_id)
        return self.k_cache[layer, block_id], self.v_cache[layer, block_id]


class PagedKVCache:
    """Block allocation + per-request tables + the pools, behind one object."""

    def __init__(self, num_blocks: int, num_layers: int, num_kv_heads: int, head_dim: int, block_size: int = 16,
                 dtype: torch.dtype = torch.bfloat16, device: str | torch.device = "cuda", free_order=None):
        self.block_manager = BlockManager(num_blocks=num_blocks, block_size=block_size, free_order=free_order)
        self.kv_cache = KVCache(num_blocks=num_blocks, num_layers=num_layers, num_kv_heads=num_kv_heads,
                                head_dim=head_dim, block_size=block_size, dtype=dtype, device=device)
        self._tables: dict[str, BlockTable] = {}
        self._counts: dict[str, int] = {}
        self._epoch = 0
        # Table store: one zero-padded int32 row of block ids per live
        # request, kept in step with the BlockTables, so a batch's block table
        # is one gather instead of a list-to-array copy per request.
        self._store = np.zeros((16, 16), dtype=np.int32)
        self._store_blocks = np.zeros(16, dtype=np.int64)   # blocks per store row
        self._store_tokens = np.zeros(16, dtype=np.int64)   # token count per store row
        self._free_rows: list[int] = []
        self._rows_used = 0
        self._row_of: dict[str, int] = {}  # live request -> its table-store row

    # -- allocation ---------------------------------------------------------
    def allocate(self, request_id: str, num_tokens: int) -> None:
        if request_id in self._tables:
            raise ValueError(f"Request {request_id!r} already exists")
        if num_tokens < 0:
            raise ValueError("num_tokens cannot be negative")
        blocks = self.block_manager.allocate(request_id=request_id, num_tokens=num_tokens)
        table = BlockTable()
        table._owner = self
        table._row = self._store_row()
        self._row_of[request_id] = table._row
        for blk in blocks:
            table.append(blk)
        self._tables[request_id] = table
        self._counts[request_id] = num_tokens
        self._store_tokens[table._row] = num_tokens
        self._epoch += 1

    def append_tokens(self, request_id: str, num_tokens: int) -> None:
        """Grow a request's capacity; new blocks only when a block boundary is crossed."""
        self._validate_request(request_id)
        if num_tokens < 0:
            raise ValueError("num_tokens cannot be negative")
        if num_tokens == 0:
            return
        old = self._counts[request_id]
        extra = self.block_manager.blocks_needed(old + num_tokens) - self.block_manager.blocks_needed(old)
        if extra > 0:
            for blk in self.block_manager.allocate_blocks(request_id=request_id, num_blocks=extra):
                self._tables[request_id].append(blk)
        self._counts[request_id] = old + num_tokens
        self._store_tokens[self._tables[request_id]._row] = old + num_tokens
        self._epoch += 1

    def free(self, request_id: str) -> None:
        self._validate_request(request_id)
        table = self._tables.pop(request_id)
        self._store_clear(table._row)
        self._free_rows.append(table._row)
        del self._row_of[request_id]
        table._owner, table._row = None, -1
        del self._counts[request_id]
        self.block_manager.free(request_id)
        self._epoch += 1

    # -- table store -------------------------------------------------------------
    def _store_row(self) -> int:
        if self._free_rows:
            return self._free_rows.pop()
        row = self._rows_used
        self._rows_used += 1
        if row >= self._store.shape[0]:
            grow = self._store.shape[0]
            self._store = np.concatenate([self._store, np.zeros_like(self._store[:grow])])
            self._store_blocks = np.concatenate([self._store_blocks, np.zeros(grow, dtype=np.int64)])
            self._store_tokens = np.concatenate([self._store_tokens, np.zeros(grow, dtype=np.int64)])
        return row

    def _store_put(self, row: int, index: int, block: int) -> None:
        if index >= self._store.shape[1]:
            width = max(2 * self._store.shape[1], index + 1)
            wider = np.zeros((self._store.shape[0], width), dtype=np.int32)
            wider[:, : self._store.shape[1]] = self._store
            self._store = wider
        self._store[row, index] = block
        self._store_blocks[row] = index + 1

    def _store_clear(self, row: int) -> None:
        self._store[row, :] = 0
        self._store_blocks[row] = 0
        self._store_tokens[row] = 0

    def _rows_of(self, request_ids) -> np.ndarray:
        try:  # one C-level pass over the id -> row map
            return np.fromiter(map(self._row_of.__getitem__, request_ids), dtype=np.int64, count=len(request_ids))
        except KeyError as e:
            raise KeyError(f"Unknown request: {e.args[0]!r}") from None

    # -- queries ---------------------------------------------------------------
    def get_block_table(self, request_id: str) -> BlockTable:
        self._validate_request(request_id)
        return self._tables[request_id]

    def token_count(self, request_id: str) -> int:
        self._validate_request(request_id)
        return self._counts[request_id]

    @property
    def metadata_epoch(self) -> int:
        """Changes whenever a request's blocks or token count change; the
        batched path reuses device copies of block tables built at the same
        epoch for the same requests and positions."""
        return self._epoch

    @property
    def free_blocks(self) -> int:
        return self.block_manager.free_blocks

    @property
    def used_blocks(self) -> int:
        return self.block_manager.used_blocks

    @property
    def num_blocks(self) -> int:
        return self.block_manager.num_blocks

    @property
    def block_size(self) -> int:
        return self.block_manager.block_size

    def _validate_request(self, request_id: str) -> None:
        if request_id not in self._tables:
            raise KeyError(f"Unknown request: {request_id!r}")

    # -- per-token access (reference semantics) -------------------------------
    def _locate(self, request_id: str, token_position: int) -> tuple[int, int]:
        self._validate_request(request_id)
        count = self._counts[request_id]
        if not 0 <= token_position < count:
            raise IndexError(f"Invalid token position: {token_position}; valid range is [0, {count})")
        bs = self.block_size
        return self._tables[request_id].get_physical_block(token_position // bs), token_position % bs

    def write_token(self, request_id: str, layer: int, token_position: int, key: torch.Tensor,
                    value: torch.Tensor) -> None:
        """Write one token's ``[Hkv, D]`` K/V at its logical position."""
        self._validate_request(request_id)
        block, offset = self._locate(request_id, token_position)
        shape = (self.kv_cache.num_kv_heads, self.kv_cache.head_dim)
        if tuple(key.shape) != shape or tuple(value.shape) != shape:
            raise ValueError(f"Expected K/V shape {shape}; got key={tuple(key.shape)}, value={tuple(value.shape)}")
        if key.dtype != self.kv_cache.dtype or value.dtype != self.kv_cache.dtype:
            raise ValueError(f"K/V tensors must have dtype {self.kv_cache.dtype}")
        if key.device != self.kv_cache.k_cache.device or value.device != self.kv_cache.v_cache.device:
            raise ValueError("K/V tensors must be on the same devices as their respective cache tensors")
        self.kv_cache.k_cache[layer, block, :, offset, :].copy_(key)
        self.kv_cache.v_cache[layer, block, :, offset, :].copy_(value)

    def read_token(self, request_id: str, layer: int, token_position: int) -> tuple[torch.Tensor, torch.Tensor]:
        block, offset = self._locate(request_id, token_position)
        return (self.kv_cache.k_cache[layer, block, :, offset, :], self.kv_cache.v_cache[layer, block, :, offset, :])

    # -- batched helpers for the B200 path -----------------------------------
    def slot_of(self, request_id: str, token_position: int) -> int:
        """int64 slot (``block * block_size + offset``) of a logical position."""
        block, offset = self._locate(request_id, token_position)
        return block * self.block_size + offset

    def table_rows(self, request_ids, width: int | None = None) -> np.ndarray:
        """Zero-padded int32 ``[B, width]`` block table of ``request_ids``
        (width: the longest of their tables by default)."""
        rows = self._rows_of(request_ids)
        if width is None:
            width = int(self._store_blocks[rows].max()) if len(rows) else 0
        width = max(width, 1)
        have = min(width, self._store.shape[1])
        if have == width:
            return self._store[rows, :width]
        out = np.zeros((len(rows), width), dtype=np.int32)
        out[:, :have] = self._store[rows, :have]
        return out

    def table_store_rows(self, request_ids) -> np.ndarray:
        """int64 ``[B]`` rows of ``request_ids`` in the table store (for
        ``gather_tables``; raises KeyError for an unknown request)."""
        return self._rows_of(request_ids)

    def table_width(self, rows: np.ndarray) -> int:
        """Blocks in the longest table of store ``rows`` (at least 1)."""
        return max(int(self._store_blocks[rows].max()), 1) if len(rows) else 1

    def gather_tables(self, rows: np.ndarray, out: np.ndarray, width: int) -> None:
        """Write the block tables of store ``rows``, zero padded to ``width``
        (>= ``table_width(rows)``), into the first ``len(rows) * width``
        elements of ``out`` (int32, C-contiguous) as ``[B, width]``."""
        dst = out[: len(rows) * width].reshape(len(rows), width)
        have = min(width, self._store.shape[1])
        np.take(self._store[:, :have], rows, axis=0, out=dst[:, :have] if have == width else None, mode="clip")
        if have < width:
            dst[:, :have] = self._store[rows, :have]
            dst[:, have:] = 0

    def store_token_counts(self, rows: np.ndarray) -> np.ndarray:
        """int64 token counts of store ``rows``."""
        return self._store_tokens[rows]

    def token_counts(self, request_ids) -> np.ndarray:
        """int64 ``[B]`` token counts of ``request_ids``."""
        return self._store_tokens[self._rows_of(request_ids)]
