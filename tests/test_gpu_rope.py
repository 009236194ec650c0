"""Fused RoPE + KV write on the GPU (psb_rope_reshape_and_cache): bit-exact
against the reference's own apply_rotary_pos_emb outputs (golden vectors
made by tests/golden/make_golden_rope.py) and against the oracle's
restatement at larger sizes, on the 16-byte and the element-wise paths."""

from __future__ import annotations

import os

import numpy as np
import pytest
import torch

from oracle import paged_attention as ora
from tests.helpers import TORCH_DTYPES

pytestmark = pytest.mark.gpu

HERE = os.path.dirname(os.path.abspath(__file__))
ROPE = np.load(os.path.join(HERE, "golden", "rope_outputs.npz"))


@pytest.fixture(scope="module", autouse=True)
def _cuda():
    if not torch.cuda.is_available():
        pytest.fail("CUDA device required for -m gpu tests")
    import pagedserve_b200._native as native
    native.load()


def _dev(a, dtype):
    return torch.from_numpy(np.ascontiguousarray(a, dtype=np.float32)).cuda().to(TORCH_DTYPES[dtype])


def _pool(nb, hkv, d, bs, dtype, layers=2, seed=0):
    g = torch.Generator(device="cuda").manual_seed(seed)
    k = torch.randn(layers, nb, hkv, bs, d, generator=g, device="cuda").to(TORCH_DTYPES[dtype])
    v = torch.randn(layers, nb, hkv, bs, d, generator=g, device="cuda").to(TORCH_DTYPES[dtype])
    return k, v


@pytest.mark.parametrize("name,dtype", [("decode_bf16", "bfloat16"), ("prefill_bf16", "bfloat16"),
                                        ("prefill_f16", "float16"), ("prefill_f32", "float32")])
def test_rope_matches_reference_outputs_bit_exact(name, dtype):
    from pagedserve_b200 import ops
    q, k = ROPE[f"{name}/q"], ROPE[f"{name}/k"]
    t, hkv, d = k.shape
    v = ora.round_to(np.random.default_rng(1).standard_normal(k.shape).astype(np.float32), dtype)
    kc, vc = _pool(t + 3, hkv, d, 16, dtype)
    kc_np, vc_np = kc.float().cpu().numpy(), vc.float().cpu().numpy()
    slots = np.random.default_rng(2).permutation((t + 3) * 16)[:t].astype(np.int64)
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    qo, ko = ops.rope_reshape_and_cache(_dev(q, dtype), _dev(k, dtype), _dev(v, dtype), _dev(ROPE[f"{name}/cos"], dtype),
                                        _dev(ROPE[f"{name}/sin"], dtype), kc, vc, torch.from_numpy(slots).cuda(), 1,
                                        error_flag=err)
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    assert np.array_equal(qo.float().cpu().numpy(), ROPE[f"{name}/q_embed"])
    assert np.array_equal(ko.float().cpu().numpy(), ROPE[f"{name}/k_embed"])
    ora.reshape_and_cache(ROPE[f"{name}/k_embed"], v, kc_np, vc_np, slots, 1)
    assert np.array_equal(kc.float().cpu().numpy(), kc_np) and np.array_equal(vc.float().cpu().numpy(), vc_np)


def _random_case(t, hq, hkv, d, dtype, seed):
    rng = np.random.default_rng(seed)
    q = ora.round_to(rng.standard_normal((t, hq, d)).astype(np.float32), dtype)
    k = ora.round_to(rng.standard_normal((t, hkv, d)).astype(np.float32), dtype)
    v = ora.round_to(rng.standard_normal((t, hkv, d)).astype(np.float32), dtype)
    pos = rng.integers(0, 32768, t)
    inv = 1.0 / (1e6 ** (np.arange(0, d, 2, dtype=np.float32) / d))
    ang = np.concatenate([pos[:, None] * inv[None]] * 2, axis=1).astype(np.float32)
    cos, sin = ora.round_to(np.cos(ang), dtype), ora.round_to(np.sin(ang), dtype)
    return q, k, v, cos, sin


@pytest.mark.parametrize("dtype,hq,hkv,d,bs", [("bfloat16", 14, 2, 64, 16), ("float16", 8, 4, 128, 16),
                                               ("float32", 14, 2, 64, 16), ("bfloat16", 6, 2, 40, 8),
                                               ("float32", 4, 1, 6, 4)])
def test_rope_matches_oracle(dtype, hq, hkv, d, bs):
    """16-byte path (bf16/f16 halves of 32/64 elements, fp32 halves of 32) and
    element-wise path (halves of 20 or 3 elements), with padding and
    out-of-pool slots."""
    from pagedserve_b200 import ops
    t = 301
    q, k, v, cos, sin = _random_case(t, hq, hkv, d, dtype, 7)
    nb = t // bs + 8
    kc, vc = _pool(nb, hkv, d, bs, dtype, seed=3)
    kc_np, vc_np = kc.float().cpu().numpy(), vc.float().cpu().numpy()
    slots = np.random.default_rng(5).permutation(nb * bs)[:t].astype(np.int64)
    slots[[0, 10, 200]] = -1
    slots[50] = nb * bs + 3   # outside the pool: flagged, skipped
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    qo, ko = ops.rope_reshape_and_cache(_dev(q, dtype), _dev(k, dtype), _dev(v, dtype), _dev(cos, dtype),
                                        _dev(sin, dtype), kc, vc, torch.from_numpy(slots).cuda(), 0, error_flag=err)
    torch.cuda.synchronize()
    assert int(err.item()) == 2
    q_want, k_want = ora.apply_rope(q, cos, sin, dtype), ora.apply_rope(k, cos, sin, dtype)
    assert np.array_equal(qo.float().cpu().numpy(), q_want)
    assert np.array_equal(ko.float().cpu().numpy(), k_want)
    ok = slots < nb * bs
    ora.reshape_and_cache(k_want[ok], v[ok], kc_np, vc_np, slots[ok], 0)
    assert np.array_equal(kc.float().cpu().numpy(), kc_np) and np.array_equal(vc.float().cpu().numpy(), vc_np)


def test_rope_in_place_strided_fused_qkv():
    """q, k, v as views of one fused projection [T, Hq + 2 Hkv, D]; q rotated
    in place; no key output (pool only)."""
    from pagedserve_b200 import ops
    dtype, t, hq, hkv, d, bs = "bfloat16", 77, 14, 2, 64, 16
    q, k, v, cos, sin = _random_case(t, hq, hkv, d, dtype, 9)
    qkv = _dev(np.concatenate([q, k, v], axis=1), dtype)
    qd, kd, vd = qkv[:, :hq], qkv[:, hq:hq + hkv], qkv[:, hq + hkv:]
    nb = 16
    kc, vc = _pool(nb, hkv, d, bs, dtype, seed=4)
    kc_np, vc_np = kc.float().cpu().numpy(), vc.float().cpu().numpy()
    slots = np.arange(t, dtype=np.int64) + 5
    qo, ko = ops.rope_reshape_and_cache(qd, kd, vd, _dev(cos, dtype), _dev(sin, dtype), kc, vc,
                                        torch.from_numpy(slots).cuda(), 1, query_out=qd, key_out=False)
    torch.cuda.synchronize()
    assert ko is None and qo.data_ptr() == qd.data_ptr()
    assert np.array_equal(qd.float().cpu().numpy(), ora.apply_rope(q, cos, sin, dtype))
    assert np.array_equal(kd.float().cpu().numpy(), k)  # the key input is left alone
    ora.reshape_and_cache(ora.apply_rope(k, cos, sin, dtype), v, kc_np, vc_np, slots, 1)
    assert np.array_equal(kc.float().cpu().numpy(), kc_np) and np.array_equal(vc.float().cpu().numpy(), vc_np)


def test_reference_facing_rope_write_then_decode():
    """rope_and_write_tokens + paged_decode_attention == the reference's
    apply_rotary_pos_emb + write_token loop + decode, through the oracle."""
    from pagedserve_b200 import PagedKVCache, paged_decode_attention, rope_and_write_tokens
    dtype, hq, hkv, d = "bfloat16", 14, 2, 64
    lens = [1, 17, 40, 200]
    cache = PagedKVCache(num_blocks=40, num_layers=2, num_kv_heads=hkv, head_dim=d, block_size=16,
                         dtype=torch.bfloat16, device="cuda", free_order=np.random.default_rng(3).permutation(40))
    ids = [f"r{i}" for i in range(len(lens))]
    for rid, n in zip(ids, lens):
        cache.allocate(rid, n)
    g = torch.Generator(device="cuda").manual_seed(11)
    cache.kv_cache.k_cache.copy_(torch.randn(cache.kv_cache.k_cache.shape, generator=g, device="cuda"))
    cache.kv_cache.v_cache.copy_(torch.randn(cache.kv_cache.v_cache.shape, generator=g, device="cuda"))
    kc0, vc0 = cache.kv_cache.k_cache.float().cpu().numpy(), cache.kv_cache.v_cache.float().cpu().numpy()
    q, k, v, cos, sin = _random_case(len(lens), hq, hkv, d, dtype, 13)
    pos = [n - 1 for n in lens]
    q_rot = rope_and_write_tokens(_dev(q, dtype).unsqueeze(2), _dev(k, dtype).unsqueeze(2),
                                  _dev(v, dtype).unsqueeze(2), _dev(cos, dtype).unsqueeze(1),
                                  _dev(sin, dtype).unsqueeze(1), cache, ids, pos, 1)
    out = paged_decode_attention(q_rot, cache, ids, pos, 1)
    torch.cuda.synchronize()
    q_want, k_want = ora.apply_rope(q, cos, sin, dtype), ora.apply_rope(k, cos, sin, dtype)
    assert np.array_equal(q_rot.squeeze(2).float().cpu().numpy(), q_want)
    tables = [cache.get_block_table(r).get_blocks() for r in ids]
    for b, rid in enumerate(ids):
        ora.write_tokens(kc0, vc0, 1, tables[b], [pos[b]], k_want[b:b + 1], v[b:b + 1])
    assert np.array_equal(cache.kv_cache.k_cache.float().cpu().numpy(), kc0)
    assert np.array_equal(cache.kv_cache.v_cache.float().cpu().numpy(), vc0)
    exact = ora.decode_attention(q_want, kc0, vc0, tables, np.asarray(lens), 1)
    diff = np.abs(out.squeeze(2).float().cpu().numpy().astype(np.float64) - exact)
    assert diff.max() <= 2e-2 and diff.mean() <= 2e-3
