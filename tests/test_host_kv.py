"""Host-side block bookkeeping: the reference's unit tests, run against the
mirror in ``pagedserve_b200.paged_kv`` (CPU, fp32).

Ported from tests/unit/test_block_manager.py, test_block_table.py,
test_kv_cache.py and test_paged_kv_cache.py of PagedServe.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from pagedserve_b200.paged_kv import BlockManager, BlockTable, KVCache, PagedKVCache
from tests.golden.cases import fifo_tables


# ---- BlockManager (test_block_manager.py) ---------------------------------
def test_block_manager_counts_and_ceil():
    m = BlockManager(num_blocks=8, block_size=16)
    assert (m.free_blocks, m.used_blocks) == (8, 0)
    assert [m.blocks_needed(n) for n in (0, 1, 16, 17, 32, 33)] == [0, 1, 1, 2, 2, 3]
    blocks = m.allocate("A", 40)
    assert len(blocks) == 3 and m.used_blocks == 3 and m.free_blocks == 5
    assert m.get_blocks("A") == blocks
    b = m.allocate("B", 30)
    assert set(blocks).isdisjoint(b)
    m.free("A")
    assert not m.has_request("A") and m.free_blocks == 6


def test_block_manager_errors():
    m = BlockManager(num_blocks=2, block_size=16)
    m.allocate("A", 32)
    with pytest.raises(RuntimeError):
        m.allocate("B", 1)
    with pytest.raises(ValueError):
        m.allocate("A", 1)
    with pytest.raises(KeyError):
        m.get_blocks("nope")
    with pytest.raises(KeyError):
        m.free("nope")
    with pytest.raises(ValueError):
        BlockManager(0)
    with pytest.raises(ValueError):
        m.blocks_needed(-1)


# ---- BlockTable (test_block_table.py) --------------------------------------
def test_block_table():
    t = BlockTable()
    assert t.num_blocks == 0 and t.get_blocks() == []
    for b in (7, 2, 9):
        t.append(b)
    assert t.get_blocks() == [7, 2, 9] and [t.get_physical_block(i) for i in range(3)] == [7, 2, 9]
    with pytest.raises(IndexError):
        t.get_physical_block(3)
    with pytest.raises(ValueError):
        t.append(-1)
    copy = t.get_blocks()
    copy.append(99)
    assert t.get_blocks() == [7, 2, 9]
    t.clear()
    assert t.num_blocks == 0


# ---- KVCache (test_kv_cache.py) -------------------------------------------
def test_kv_cache_layout_and_bytes():
    c = KVCache(num_blocks=4, num_layers=2, num_kv_heads=2, head_dim=4, block_size=16, dtype=torch.float32,
                device="cpu")
    assert c.k_cache.shape == c.v_cache.shape == (2, 4, 2, 16, 4)
    assert c.block_shape == (2, 16, 4)
    assert c.block_bytes == 2 * 2 * 2 * 16 * 4 * 4 and c.total_bytes == 4 * c.block_bytes
    key, value = torch.randn(c.block_shape), torch.randn(c.block_shape)
    c.write_block(0, 1, key, value)
    k, v = c.read_block(0, 1)
    assert torch.equal(k, key) and torch.equal(v, value)
    with pytest.raises(IndexError):
        c.write_block(2, 0, key, value)
    with pytest.raises(IndexError):
        c.read_block(0, 4)
    with pytest.raises(ValueError):
        c.write_block(0, 0, torch.randn(1, 16, 4), value)
    with pytest.raises(ValueError):
        c.write_block(0, 0, key.double(), value)


def test_qwen_kv_bytes_per_token():
    """12288 bytes per token for Qwen2.5-0.5B in bf16 (bench/baselines/model_config.json)."""
    c = KVCache(num_blocks=1, num_layers=24, num_kv_heads=2, head_dim=64, block_size=16, dtype=torch.bfloat16,
                device="cpu")
    assert c.block_bytes == 196608 and c.block_bytes // 16 == 12288


# ---- PagedKVCache (test_paged_kv_cache.py) --------------------------------
def _cache():
    return PagedKVCache(num_blocks=4, num_layers=2, num_kv_heads=2, head_dim=4, block_size=16, dtype=torch.float32,
                        device="cpu")


def test_paged_allocation():
    c = _cache()
    c.allocate("r1", 40)
    assert c.get_block_table("r1").get_blocks() == [0, 1, 2]
    assert (c.used_blocks, c.free_blocks) == (3, 1)
    c.free("r1")
    assert (c.used_blocks, c.free_blocks) == (0, 4)
    c.allocate("again", 16)  # freed blocks went to the tail of the free list
    assert c.get_block_table("again").get_blocks() == [3]
    c = _cache()
    c.allocate("a", 16)
    c.allocate("b", 16)
    assert c.get_block_table("a").get_blocks() == [0] and c.get_block_table("b").get_blocks() == [1]


@pytest.mark.parametrize("initial,appended,tokens,blocks",
                         [(15, 1, 16, 1), (16, 1, 17, 2), (31, 1, 32, 2), (32, 1, 33, 3), (40, 8, 48, 3),
                          (48, 1, 49, 4)])
def test_dynamic_block_growth(initial, appended, tokens, blocks):
    c = _cache()
    c.allocate("A", initial)
    c.append_tokens("A", appended)
    assert c.token_count("A") == tokens
    assert c.get_block_table("A").num_blocks == blocks
    assert (c.used_blocks, c.free_blocks) == (blocks, 4 - blocks)


def test_growth_errors_preserve_state():
    c = _cache()
    c.allocate("A", 64)
    before = c.get_block_table("A").get_blocks()
    with pytest.raises(RuntimeError):
        c.append_tokens("A", 1)
    assert c.token_count("A") == 64 and c.get_block_table("A").get_blocks() == before
    with pytest.raises(ValueError):
        c.append_tokens("A", -1)
    with pytest.raises(KeyError):
        c.append_tokens("unknown", 1)
    with pytest.raises(ValueError):
        c.allocate("A", 1)
    c.append_tokens("A", 0)
    assert c.token_count("A") == 64


def test_write_read_across_block_boundary():
    c = _cache()
    c.allocate("A", 17)
    key = torch.full((2, 4), 3.0)
    value = torch.full((2, 4), 4.0)
    c.write_token("A", 1, 15, key, value)
    c.write_token("A", 1, 16, key * 2, value * 2)
    k15, v15 = c.read_token("A", 1, 15)
    k16, v16 = c.read_token("A", 1, 16)
    assert torch.equal(k15, key) and torch.equal(v15, value)
    assert torch.equal(k16, key * 2) and torch.equal(v16, value * 2)
    with pytest.raises(IndexError):
        c.read_token("A", 0, 17)
    with pytest.raises(IndexError):
        c.read_token("A", 0, -1)
    with pytest.raises(KeyError):
        c.read_token("unknown", 0, 0)
    with pytest.raises(ValueError):
        c.write_token("A", 0, 0, torch.zeros(3, 4), value)
    with pytest.raises(ValueError):
        c.write_token("A", 0, 0, key.double(), value)


def test_fragmentation_known_answer():
    """alloc A,B,C; free B; alloc D(5 tokens, block size 2) -> [3, 4, 1]
    (test_paged_attention.py:125-150)."""
    c = PagedKVCache(num_blocks=5, num_layers=1, num_kv_heads=2, head_dim=4, block_size=2, dtype=torch.float32,
                     device="cpu")
    for r in ("A", "B", "C"):
        c.allocate(r, 2)
    c.free("B")
    c.allocate("D", 5)
    assert c.get_block_table("D").get_blocks() == [3, 4, 1]


def test_interleaved_growth_matches_reference_allocator():
    c = PagedKVCache(num_blocks=32, num_layers=1, num_kv_heads=2, head_dim=64, block_size=16, dtype=torch.float32,
                     device="cpu")
    lens = [17, 32, 65]
    for r in "abc":
        c.allocate(r, 1)
    for r, n in zip("abc", lens):
        c.append_tokens(r, n - 1)
    assert [c.get_block_table(r).get_blocks() for r in "abc"] == fifo_tables([1] * 3, lens, 32, 16)


def test_batched_helpers():
    c = PagedKVCache(num_blocks=32, num_layers=1, num_kv_heads=2, head_dim=64, block_size=16, dtype=torch.float32,
                     device="cpu")
    for r in "abc":
        c.allocate(r, 1)
    for r, n in zip("abc", [17, 32, 65]):
        c.append_tokens(r, n - 1)
    rows = c.table_rows(["c", "a"])
    assert rows.dtype == np.int32 and rows.tolist() == [[2, 5, 6, 7, 8], [0, 3, 0, 0, 0]]
    assert c.slot_of("a", 16) == 3 * 16 and c.slot_of("c", 64) == 8 * 16
    with pytest.raises(IndexError):
        c.slot_of("a", 17)


def test_metadata_epoch_tracks_every_change():
    c = PagedKVCache(num_blocks=16, num_layers=1, num_kv_heads=2, head_dim=8, block_size=4, dtype=torch.float32,
                     device="cpu")
    seen = [c.metadata_epoch]

    def changed():
        seen.append(c.metadata_epoch)
        return seen[-1] != seen[-2]

    c.allocate("a", 3)
    assert changed()
    c.append_tokens("a", 1)      # same block, more tokens: positions valid now differ
    assert changed()
    c.append_tokens("a", 0)      # no change
    assert not changed()
    c.get_block_table("a").append(9)  # direct table edit by a caller
    assert changed()
    c.token_count("a")
    assert not changed()
    c.free("a")
    assert changed()


def test_host_metadata_reused_within_an_epoch():
    from pagedserve_b200 import attention
    c = PagedKVCache(num_blocks=32, num_layers=2, num_kv_heads=2, head_dim=8, block_size=4, dtype=torch.float32,
                     device="cpu")
    for rid, n in (("x", 5), ("y", 9)):
        c.allocate(rid, n)
    dev = torch.device("cpu")
    t1, l1, w1 = attention._host_metadata(c, ["x", "y"], [4, 8], dev)
    t2, l2, w2 = attention._host_metadata(c, ["x", "y"], [4, 8], dev)
    assert t1 is t2 and l1 is l2 and w1 == w2 == 3
    assert l1.tolist() == [5, 9]
    assert t1.tolist() == [c.get_block_table("x").get_blocks() + [0], c.get_block_table("y").get_blocks()]
    t3, l3, _ = attention._host_metadata(c, ["x", "y"], [3, 8], dev)   # other positions, same epoch:
    assert t3 is t1 and l3 is not l1 and l3.tolist() == [4, 9]          # the table is kept, lengths rebuilt
    c.append_tokens("x", 4)                                             # new epoch
    t4, l4, w4 = attention._host_metadata(c, ["x", "y"], [8, 8], dev)
    assert t4 is not t1 and w4 == 3 and l4.tolist() == [9, 9]
    assert t4.tolist()[0] == c.get_block_table("x").get_blocks()
    t5, _, _ = attention._host_metadata(c, ["y", "x"], [8, 8], dev)    # another request list
    assert t5 is not t4 and t5.tolist()[1] == t4.tolist()[0]
    with pytest.raises(ValueError, match="Invalid position"):
        attention._host_metadata(c, ["x", "y"], [9, 8], dev)
    attention.clear_metadata_cache(c)
    assert len(c._psb_metadata) == 0


def test_host_metadata_without_epoch_rebuilds():
    """A cache object without ``metadata_epoch`` (the reference's) is rebuilt every call."""
    from pagedserve_b200 import attention
    inner = PagedKVCache(num_blocks=8, num_layers=1, num_kv_heads=1, head_dim=8, block_size=4, dtype=torch.float32,
                         device="cpu")
    inner.allocate("r", 6)

    class Plain:
        block_size = 4
        kv_cache = inner.kv_cache

        def token_count(self, rid):
            return inner.token_count(rid)

        def get_block_table(self, rid):
            return inner.get_block_table(rid)

    plain = Plain()
    a = attention._host_metadata(plain, ["r"], [5], torch.device("cpu"))
    b = attention._host_metadata(plain, ["r"], [5], torch.device("cpu"))
    assert a[0] is not b[0] and torch.equal(a[0], b[0])
    assert not hasattr(plain, "_psb_metadata")


def test_table_store_follows_every_change():
    """table_rows / token_counts (the vectorised store) equal the per-request
    BlockTables through allocation, growth past the store's width, frees,
    row reuse and direct table edits."""
    rng = np.random.default_rng(7)
    c = PagedKVCache(num_blocks=4096, num_layers=1, num_kv_heads=1, head_dim=8, block_size=4, dtype=torch.float32,
                     device="cpu", free_order=rng.permutation(4096))
    live: dict[str, int] = {}
    for step in range(400):
        op = rng.integers(0, 3)
        if op == 0 or not live:
            rid = f"r{step}"
            n = int(rng.integers(0, 70))
            c.allocate(rid, n)
            live[rid] = n
        elif op == 1:
            rid = list(live)[int(rng.integers(0, len(live)))]
            k = int(rng.integers(0, 90))
            c.append_tokens(rid, k)
            live[rid] += k
        else:
            rid = list(live)[int(rng.integers(0, len(live)))]
            c.free(rid)
            del live[rid]
        if live and step % 7 == 0:
            ids = list(live)
            rng.shuffle(ids)
            rows = c.table_rows(ids)
            width = max(1, max(c.get_block_table(r).num_blocks for r in ids))
            want = np.zeros((len(ids), width), dtype=np.int32)
            for i, r in enumerate(ids):
                b = c.get_block_table(r).get_blocks()
                want[i, : len(b)] = b
            assert np.array_equal(rows, want)
            assert c.token_counts(ids).tolist() == [live[r] for r in ids]
            assert np.array_equal(c.table_rows(ids, width=width + 3)[:, :width], want)
            assert not c.table_rows(ids, width=width + 3)[:, width:].any()
    rid = next(iter(live))
    c.get_block_table(rid).append(4000)                # a caller's direct edit reaches the store
    assert c.table_rows([rid])[0, c.get_block_table(rid).num_blocks - 1] == 4000
    with pytest.raises(KeyError, match="Unknown request"):
        c.table_rows([rid, "nope"])


def test_host_metadata_fast_path_sees_list_changes():
    """The last-call shortcut compares list contents, so an id list or a
    position list changed in place between calls is never served stale."""
    from pagedserve_b200 import attention
    c = PagedKVCache(num_blocks=32, num_layers=1, num_kv_heads=1, head_dim=8, block_size=4, dtype=torch.float32,
                     device="cpu")
    for rid, n in (("x", 5), ("y", 9), ("z", 2)):
        c.allocate(rid, n)
    dev = torch.device("cpu")
    ids, pos = ["x", "y"], [4, 8]
    t1, l1, _ = attention._host_metadata(c, ids, pos, dev)
    assert attention._host_metadata(c, ids, pos, dev)[0] is t1          # same lists: reused
    pos[0] = 2
    _, l2, _ = attention._host_metadata(c, ids, pos, dev)
    assert l2.tolist() == [3, 9]
    ids[1] = "z"
    pos[1] = 1
    t3, l3, _ = attention._host_metadata(c, ids, pos, dev)
    assert l3.tolist() == [3, 2] and t3.tolist()[1][: 1] == c.get_block_table("z").get_blocks()
    with pytest.raises(ValueError, match="Invalid position 7 for z"):
        attention._host_metadata(c, ["x", "z"], [0, 7], dev)
