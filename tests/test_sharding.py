"""Sequence sharding across ranks: placement rule and the host-side
aggregation, including a two-rank gloo run on CPU."""

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from pagedserve_b200 import PagedKVCache
from pagedserve_b200.sharding import SequenceDispatcher, aggregate_counters, balanced, shard_sequences


def test_most_free_blocks_wins_ties_lowest():
    d = SequenceDispatcher(3, [10, 10, 10], block_size=16)
    assert d.assign("a", 40) == 0          # 3 blocks: [7, 10, 10]
    assert d.assign("b", 16) == 1          # [7, 9, 10]
    assert d.assign("c", 1) == 2           # [7, 9, 9]
    assert d.assign("d", 0) == 1           # zero blocks; 9 == 9, lowest rank
    assert [d.free_blocks(r) for r in range(3)] == [7, 9, 9]
    assert [d.running_tokens(r) for r in range(3)] == [40, 16, 1]
    assert d.shard(1) == ["b", "d"]


def test_release_and_errors():
    d = SequenceDispatcher(2, 4, block_size=16)
    assert d.assign("x", 64) == 0
    assert d.assign("y", 64) == 1
    with pytest.raises(RuntimeError):
        d.assign("z", 17)                   # needs 2 blocks, both ranks have 0
    with pytest.raises(ValueError):
        d.assign("x", 1)
    d.release("x")
    assert d.free_blocks(0) == 4
    assert d.assign("z", 17) == 0
    with pytest.raises(KeyError):
        d.release("nope")
    with pytest.raises(KeyError):
        d.rank_of("x")
    with pytest.raises(ValueError):
        SequenceDispatcher(0, 1)
    with pytest.raises(ValueError):
        SequenceDispatcher(2, [1])
    with pytest.raises(ValueError):
        d.blocks_needed(-1)


def test_shards_partition_and_balance():
    rng = np.random.default_rng(5)
    lens = np.clip(np.round(rng.lognormal(np.log(1024), 0.8, 2048)), 16, 8192).astype(np.int64)
    for world in (1, 2, 4, 8):
        blocks = int(np.ceil(1.25 * np.sum(-(-lens // 16)) / world))
        shards = shard_sequences(lens, world, blocks)
        flat = sorted(i for s in shards for i in s)
        assert flat == list(range(len(lens)))
        toks = balanced(shards, lens)
        assert sum(toks) == int(lens.sum())
        # the greedy placement keeps every rank within one longest request of the mean
        assert max(toks) - min(toks) <= 8192


def test_aggregate_without_process_group_is_identity():
    assert aggregate_counters({"b": 2, "a": 1.5}) == {"a": 1.5, "b": 2.0}
    with pytest.raises(ValueError):
        aggregate_counters({"a": 1}, op="min")


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank: int, world: int, port: int, lens: list[int], out_dir: str) -> None:
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world)
    try:
        blocks = int(np.ceil(1.25 * sum(-(-n // 16) for n in lens) / world))
        shards = shard_sequences(lens, world, blocks)
        # every rank computes the placement alone; all must agree
        gathered = [None] * world
        dist.all_gather_object(gathered, shards)
        assert all(g == shards for g in gathered)
        mine = shards[rank]
        # this rank's pool holds only its own requests
        cache = PagedKVCache(num_blocks=blocks, num_layers=1, num_kv_heads=2, head_dim=8, block_size=16,
                             dtype=torch.float32, device="cpu")
        for i in mine:
            cache.allocate(f"r{i}", lens[i])
        rows = cache.table_rows([f"r{i}" for i in mine])
        assert rows.shape[0] == len(mine)
        used = cache.used_blocks
        total = aggregate_counters({"seqs": len(mine), "tokens": sum(lens[i] for i in mine), "blocks": used})
        slowest = aggregate_counters({"step_ms": 1.0 + rank}, op="max")
        np.save(os.path.join(out_dir, f"rank{rank}.npy"),
                np.array([total["seqs"], total["tokens"], total["blocks"], slowest["step_ms"]]))
    finally:
        dist.destroy_process_group()


def test_two_rank_gloo_sharding(tmp_path):
    rng = np.random.default_rng(11)
    lens = [int(x) for x in np.clip(np.round(rng.lognormal(np.log(256), 0.8, 96)), 16, 4096)]
    world = 2
    mp.start_processes(_rank_main, args=(world, _free_port(), lens, str(tmp_path)), nprocs=world,
                       start_method="spawn", join=True)
    blocks_total = sum(-(-n // 16) for n in lens)
    for r in range(world):
        seqs, tokens, blocks, step_ms = np.load(tmp_path / f"rank{r}.npy")
        assert seqs == len(lens)
        assert tokens == sum(lens)
        assert blocks == blocks_total
        assert step_ms == 2.0
