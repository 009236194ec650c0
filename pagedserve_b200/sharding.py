"""Sequence sharding across the GPUs of one node.

Requests are independent, so a node with N GPUs serves them as N replicas:
one process per GPU, each with its own ``PagedKVCache`` pool, and every
request placed on exactly one rank for its whole life.  Nothing on the
attention path crosses GPUs; the only cross-rank traffic is host-side
bookkeeping (the end-of-run counter aggregation below, and the max-over-ranks
step time a benchmark reports).

The reference serves from one process on one device (pagedserve/engine/
engine.py, pagedserve/engine/continuous_batcher.py:33-65) and has no
dispatcher; this module is the placement rule that sits in front of N such
engines.  It is deterministic: every rank that runs ``SequenceDispatcher``
over the same arrival sequence computes the same placement, so the ranks need
not exchange it.
"""

from __future__ import annotations

from typing import Iterable, Sequence

import torch


class SequenceDispatcher:
    """Places each arriving request on the rank with the most free KV blocks.

    ``blocks_per_rank`` is each rank's pool size in blocks (an int for equal
    pools, or one entry per rank).  ``assign`` reserves the blocks a request
    needs for ``num_tokens`` tokens (prompt plus the decode budget the caller
    plans for) on the chosen rank; ``release`` returns them.  Ties go to the
    lowest rank.  A request that fits on no rank raises ``RuntimeError``, the
    error ``BlockManager.allocate`` raises for an exhausted pool
    (pagedserve/engine/block_manager.py:71-90).
    """

    def __init__(self, world_size: int, blocks_per_rank, block_size: int = 16):
        if world_size <= 0:
            raise ValueError("world_size must be positive")
        if block_size <= 0:
            raise ValueError("block_size must be positive")
        if isinstance(blocks_per_rank, int):
            blocks_per_rank = [blocks_per_rank] * world_size
        blocks_per_rank = [int(b) for b in blocks_per_rank]
        if len(blocks_per_rank) != world_size:
            raise ValueError("blocks_per_rank needs one entry per rank")
        if any(b < 0 for b in blocks_per_rank):
            raise ValueError("blocks_per_rank cannot be negative")
        self.world_size = world_size
        self.block_size = block_size
        self._free = list(blocks_per_rank)
        self._tokens = [0] * world_size
        self._placed: dict[str, tuple[int, int, int]] = {}

    def blocks_needed(self, num_tokens: int) -> int:
        if num_tokens < 0:
            raise ValueError("num_tokens cannot be negative")
        return -(-num_tokens // self.block_size)

    def free_blocks(self, rank: int) -> int:
        return self._free[rank]

    def running_tokens(self, rank: int) -> int:
        return self._tokens[rank]

    def assign(self, request_id: str, num_tokens: int) -> int:
        if request_id in self._placed:
            raise ValueError(f"request {request_id} is already placed")
        need = self.blocks_needed(num_tokens)
        best = -1
        for r in range(self.world_size):
            if self._free[r] >= need and (best < 0 or self._free[r] > self._free[best]):
                best = r
        if best < 0:
            raise RuntimeError(f"no rank has {need} free KV blocks for request {request_id}")
        self._free[best] -= need
        self._tokens[best] += num_tokens
        self._placed[request_id] = (best, need, num_tokens)
        return best

    def rank_of(self, request_id: str) -> int:
        if request_id not in self._placed:
            raise KeyError(f"request {request_id} is not placed")
        return self._placed[request_id][0]

    def release(self, request_id: str) -> None:
        if request_id not in self._placed:
            raise KeyError(f"request {request_id} is not placed")
        rank, need, tokens = self._placed.pop(request_id)
        self._free[rank] += need
        self._tokens[rank] -= tokens

    def shard(self, rank: int) -> list[str]:
        """Request ids placed on ``rank``, in placement order."""
        return [rid for rid, (r, _, _) in self._placed.items() if r == rank]


def shard_sequences(lengths: Sequence[int], world_size: int, blocks_per_rank: int, block_size: int = 16
                    ) -> list[list[int]]:
    """Indices of ``lengths`` that each rank serves, placing them in order
    with ``SequenceDispatcher`` (most free blocks first)."""
    d = SequenceDispatcher(world_size, blocks_per_rank, block_size)
    for i, n in enumerate(lengths):
        d.assign(str(i), int(n))
    return [[int(rid) for rid in d.shard(r)] for r in range(world_size)]


def aggregate_counters(counters: dict[str, float], device: torch.device | str = "cpu", op: str = "sum",
                       group=None) -> dict[str, float]:
    """Combine per-rank counters over ``group`` (default: the default process group).

    ``op`` is ``"sum"`` (tokens served, bytes moved) or ``"max"`` (step time:
    the job is as slow as its slowest rank).  ``device`` is where the staging
    tensor lives: ``"cpu"`` for a gloo group, the rank's GPU for NCCL.  Every
    rank must pass the same keys.  Without an initialised process group the
    counters come back unchanged.
    """
    import torch.distributed as dist
    if op not in ("sum", "max"):
        raise ValueError("op must be 'sum' or 'max'")
    keys = sorted(counters)
    if not (dist.is_available() and dist.is_initialized()):
        return {k: float(counters[k]) for k in keys}
    t = torch.tensor([float(counters[k]) for k in keys], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.SUM if op == "sum" else dist.ReduceOp.MAX, group=group)
    return {k: float(v) for k, v in zip(keys, t.tolist())}


def gather_counters(counters: dict[str, float], group=None) -> list[dict[str, float]]:
    """Every rank's counters, in rank order, over a gloo ``group`` (host
    tensors).  Every rank must pass the same keys; without an initialised
    process group this is ``[counters]``."""
    import torch.distributed as dist
    keys = sorted(counters)
    if not (dist.is_available() and dist.is_initialized()):
        return [{k: float(counters[k]) for k in keys}]
    world = dist.get_world_size(group)
    t = torch.tensor([float(counters[k]) for k in keys], dtype=torch.float64)
    out = [torch.empty_like(t) for _ in range(world)]
    dist.all_gather(out, t, group=group)
    return [{k: float(v) for k, v in zip(keys, o.tolist())} for o in out]


def balanced(shards: Iterable[Sequence[int]], lengths: Sequence[int]) -> list[int]:
    """Tokens per rank for a placement (a convenience for reports)."""
    return [int(sum(int(lengths[i]) for i in s)) for s in shards]
