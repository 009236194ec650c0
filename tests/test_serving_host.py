"""Host-side parts of the serving loop, on the CPU: FIFO admission with KV
reservations (the reference Scheduler's rules), the synthetic trace, and the
rotary tables the runner gathers from (against transformers' own rotary
embedding)."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from pagedserve_b200.paged_kv import PagedKVCache
from pagedserve_b200.serving import FifoScheduler, ServeRequest, poisson_trace, prompt_tokens


def _cache(blocks=64):
    return PagedKVCache(num_blocks=blocks, num_layers=1, num_kv_heads=1, head_dim=4, block_size=16,
                        dtype=torch.float32, device="cpu")


def _req(rid, prompt, new):
    return ServeRequest(rid, np.zeros(prompt, dtype=np.int64), new)


def test_admission_is_strict_fifo_with_reservations():
    """scheduler.py:68-109: the head is admitted while capacity and its
    prompt + max_new_tokens blocks allow; a head that does not fit blocks
    the queue (nothing behind it is admitted)."""
    cache = _cache(blocks=10)
    s = FifoScheduler(cache, max_running=8, max_prefill_tokens=10_000, max_prefill_seqs=8)
    s.submit(_req("a", 40, 8))    # 3 blocks
    s.submit(_req("b", 90, 10))   # 7 blocks -> 10 used
    s.submit(_req("c", 1, 1))     # 1 block: no room
    s.submit(_req("d", 1, 0))
    assert [r.request_id for r in s.schedule()] == ["a", "b"]
    assert cache.free_blocks == 0
    assert s.schedule() == []
    s.complete("a")
    assert [r.request_id for r in s.schedule()] == ["c", "d"]
    assert cache.free_blocks == 1


def test_admission_caps():
    cache = _cache(blocks=1000)
    s = FifoScheduler(cache, max_running=3, max_prefill_tokens=100, max_prefill_seqs=2)
    for i, n in enumerate([30, 30, 30, 60, 10]):
        s.submit(_req(f"r{i}", n, 4))
    assert [r.request_id for r in s.schedule()] == ["r0", "r1"]          # two per step
    assert [r.request_id for r in s.schedule()] == ["r2"]                # running cap 3
    s.complete("r0")
    s.complete("r1")
    assert [r.request_id for r in s.schedule()] == ["r3", "r4"]          # 60 + 10 prompt tokens <= 100
    s.complete("r2")
    s.submit(_req("r5", 95, 1))
    s.submit(_req("r6", 10, 1))
    assert [r.request_id for r in s.schedule()] == ["r5"]                # 95 + 10 > 100: r6 waits
    with pytest.raises(ValueError, match="prefill budget"):
        s.submit(_req("big", 101, 1))
    with pytest.raises(ValueError, match="empty"):
        s.submit(_req("empty", 0, 1))


def test_request_positions_follow_the_reference():
    """continuous_batcher.py:316-319: the decode step feeds the last
    generated token at num_prompt + num_generated - 1."""
    r = _req("x", 7, 5)
    r.generated = 1
    assert r.position == 7 and r.capacity == 12
    r.generated = 3
    assert r.position == 9


def test_poisson_trace_shapes():
    tr = poisson_trace(20000, rate=1000.0, seed=1)
    arr = np.array([a for a, _, _ in tr])
    prompts = np.array([p for _, p, _ in tr])
    outs = np.array([o for _, _, o in tr])
    assert np.all(np.diff(arr) >= 0) and abs(arr[-1] / len(tr) - 1e-3) < 1e-4
    assert prompts.min() >= 16 and prompts.max() <= 8192 and abs(np.median(prompts) - 512) < 25
    assert outs.min() >= 1 and abs(outs.mean() - 256) < 8
    assert np.all(prompts + outs <= 32768)
    assert poisson_trace(5, 10.0, seed=1) == tr[:0] + poisson_trace(5, 10.0, seed=1)
    a, b = prompt_tokens(3, 50, 1000, 9), prompt_tokens(3, 50, 1000, 9)
    assert np.array_equal(a, b) and a.min() >= 0 and a.max() < 1000


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_rope_tables_equal_transformers_rotary(dtype):
    """Row p of the runner's tables is transformers' Qwen2 rotary embedding
    for position p (engine.py:572-575), bit for bit."""
    from transformers import Qwen2Config
    from transformers.models.qwen2.modeling_qwen2 import Qwen2RotaryEmbedding

    from pagedserve_b200.model_runner import QwenConfig, rope_tables
    cfg = Qwen2Config(hidden_size=896, num_attention_heads=14, num_key_value_heads=2, rope_theta=1e6,
                      max_position_embeddings=32768)
    rot = Qwen2RotaryEmbedding(cfg)
    pos = torch.tensor([[0, 1, 2, 15, 16, 511, 4097, 32767]])
    x = torch.zeros(1, pos.shape[1], 896, dtype=dtype)
    cos, sin = rot(x, pos)
    tc, ts = rope_tables(QwenConfig.from_hf(cfg), "cpu", dtype)
    assert torch.equal(tc[pos[0]], cos[0]) and torch.equal(ts[pos[0]], sin[0])
