"""Fused decode step (psb_paged_decode_append): the new token's cache write
and the attention in one launch must equal reshape_and_cache followed by
paged_decode - the same pool bytes and the same outputs - and, through the
oracle, the reference's write_token loop followed by its decode.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import paged_attention as ora
from tests.helpers import TOL, TORCH_DTYPES, err_stats

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module", autouse=True)
def _cuda():
    if not torch.cuda.is_available():
        pytest.fail("CUDA device required for -m gpu tests")
    import pagedserve_b200._native as native
    native.load()


def _case(seed, lens, hq, hkv, d, bs, layers=2, dtype="bfloat16"):
    """Fragmented tables over a shuffled pool, pools and new rows drawn in
    ``dtype``; returns device tensors plus the int64 slot of each row's last
    position (-1 for an empty row)."""
    rng = np.random.default_rng(seed)
    lens = np.asarray(lens, dtype=np.int64)
    need = [max(1, -(-int(n) // bs)) for n in lens]
    nb = int(sum(need) * 1.5) + 4
    perm = rng.permutation(nb)
    tables, at = [], 0
    for k in need:
        tables.append(perm[at:at + k])
        at += k
    width = max(need) + 1
    table = np.zeros((len(lens), width), dtype=np.int32)
    for i, t in enumerate(tables):
        table[i, :len(t)] = t
    slots = np.array([-1 if n == 0 else tables[i][(n - 1) // bs] * bs + (n - 1) % bs for i, n in enumerate(lens)],
                     dtype=np.int64)
    td = TORCH_DTYPES[dtype]
    g = torch.Generator(device="cuda").manual_seed(seed)
    k = torch.randn(layers, nb, hkv, bs, d, generator=g, device="cuda").to(td)
    v = torch.randn(layers, nb, hkv, bs, d, generator=g, device="cuda").to(td)
    q = torch.randn(len(lens), hq, d, generator=g, device="cuda").to(td)
    nk = torch.randn(len(lens), hkv, d, generator=g, device="cuda").to(td)
    nv = torch.randn(len(lens), hkv, d, generator=g, device="cuda").to(td)
    return dict(k=k, v=v, q=q, nk=nk, nv=nv, table=torch.from_numpy(table).cuda(),
                lens=torch.from_numpy(lens.astype(np.int32)).cuda(), slots=torch.from_numpy(slots).cuda(),
                tables=tables, lens_np=lens, max_context=width * bs)


def _both(c, layer):
    """(pools, out) of the two-launch sequence and of the fused launch."""
    from pagedserve_b200 import ops
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    k1, v1 = c["k"].clone(), c["v"].clone()
    ops.reshape_and_cache(c["nk"], c["nv"], k1, v1, c["slots"], layer, error_flag=err)
    o1 = ops.paged_decode(c["q"], k1, v1, c["table"], c["lens"], layer, max_context=c["max_context"],
                          error_flag=err)
    k2, v2 = c["k"].clone(), c["v"].clone()
    o2 = ops.paged_decode(c["q"], k2, v2, c["table"], c["lens"], layer, max_context=c["max_context"],
                          error_flag=err, new_key=c["nk"], new_value=c["nv"])
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    return (k1, v1, o1), (k2, v2, o2)


BOUNDARY = [1, 2, 15, 16, 17, 31, 32, 33, 64, 65, 129, 1000, 4097]


@pytest.mark.parametrize("dtype", ["bfloat16", "float16"])
@pytest.mark.parametrize("hq,hkv", [(14, 2), (8, 1), (16, 4)])
def test_append_equals_write_then_decode(dtype, hq, hkv):
    c = _case(11, BOUNDARY + [0, 300, 17], hq, hkv, 64, 16, dtype=dtype)
    for layer in (0, 1):
        (k1, v1, o1), (k2, v2, o2) = _both(c, layer)
        assert torch.equal(k1, k2) and torch.equal(v1, v2)
        assert torch.equal(o1, o2)


def test_append_serving_batch_split_across_warps():
    rng = np.random.default_rng(3)
    lens = np.clip(np.round(rng.lognormal(np.log(1024), 0.8, 256)), 16, 8192).astype(np.int64)
    c = _case(12, lens, 14, 2, 64, 16)
    (k1, v1, o1), (k2, v2, o2) = _both(c, 1)
    assert torch.equal(k1, k2) and torch.equal(v1, v2)
    assert torch.equal(o1, o2)


@pytest.mark.parametrize("dtype,d,bs", [("float32", 64, 16), ("bfloat16", 128, 16), ("float16", 64, 8)])
def test_append_generic_path(dtype, d, bs):
    c = _case(13, [1, 7, 8, 9, 40, 0, 100], 4, 2, d, bs, dtype=dtype)
    (k1, v1, o1), (k2, v2, o2) = _both(c, 0)
    assert torch.equal(k1, k2) and torch.equal(v1, v2)
    assert torch.equal(o1, o2)


def test_append_matches_oracle_write_then_decode():
    """The fused launch against the reference algorithm: write_token at each
    row's last position, then decode (oracle, float64)."""
    c = _case(14, [1, 16, 17, 200, 33], 14, 2, 64, 16)
    from pagedserve_b200 import ops
    k, v = c["k"].clone(), c["v"].clone()
    out = ops.paged_decode(c["q"], k, v, c["table"], c["lens"], 1, max_context=c["max_context"],
                           new_key=c["nk"], new_value=c["nv"])
    kc = c["k"].float().cpu().numpy()
    vc = c["v"].float().cpu().numpy()
    nk, nv = c["nk"].float().cpu().numpy(), c["nv"].float().cpu().numpy()
    for b, n in enumerate(c["lens_np"]):
        pos = int(n) - 1
        blk, off = c["tables"][b][pos // 16], pos % 16
        kc[1, blk, :, off, :] = nk[b]
        vc[1, blk, :, off, :] = nv[b]
    exact = ora.decode_attention(c["q"].float().cpu().numpy(), kc, vc, c["tables"], c["lens_np"], 1)
    mx, mean = err_stats(out, exact)
    assert mx <= TOL["bfloat16"][0] and mean <= TOL["bfloat16"][1], (mx, mean)
    assert np.array_equal(k.float().cpu().numpy(), kc) and np.array_equal(v.float().cpu().numpy(), vc)


def test_reference_facing_write_and_attend():
    """paged_decode_attention_with_write == write_tokens + paged_decode_attention."""
    from pagedserve_b200 import PagedKVCache, paged_decode_attention, paged_decode_attention_with_write, write_tokens
    torch.manual_seed(5)
    lens = [3, 16, 17, 40, 1]
    caches = []
    for _ in range(2):
        cache = PagedKVCache(num_blocks=64, num_layers=2, num_kv_heads=2, head_dim=64, block_size=16,
                             dtype=torch.bfloat16, device="cuda", free_order=np.random.default_rng(2).permutation(64))
        for i, n in enumerate(lens):
            cache.allocate(f"r{i}", n)
        caches.append(cache)
    g = torch.Generator(device="cuda").manual_seed(9)
    pool_k = torch.randn(caches[0].kv_cache.k_cache.shape, generator=g, device="cuda").to(torch.bfloat16)
    pool_v = torch.randn(caches[0].kv_cache.v_cache.shape, generator=g, device="cuda").to(torch.bfloat16)
    for cache in caches:
        cache.kv_cache.k_cache.copy_(pool_k)
        cache.kv_cache.v_cache.copy_(pool_v)
    ids = [f"r{i}" for i in range(len(lens))]
    pos = [n - 1 for n in lens]
    q = torch.randn(len(lens), 14, 1, 64, generator=g, device="cuda").to(torch.bfloat16)
    nk = torch.randn(len(lens), 2, 1, 64, generator=g, device="cuda").to(torch.bfloat16)
    nv = torch.randn(len(lens), 2, 1, 64, generator=g, device="cuda").to(torch.bfloat16)
    write_tokens(caches[0], ids, pos, 1, nk, nv)
    o1 = paged_decode_attention(q, caches[0], ids, pos, 1)
    o2 = paged_decode_attention_with_write(q, nk, nv, caches[1], ids, pos, 1)
    torch.cuda.synchronize()
    assert torch.equal(o1, o2)
    assert torch.equal(caches[0].kv_cache.k_cache, caches[1].kv_cache.k_cache)
    assert torch.equal(caches[0].kv_cache.v_cache, caches[1].kv_cache.v_cache)
    with pytest.raises(ValueError, match="Expected K/V shape"):
        paged_decode_attention_with_write(q, nk[:, :1], nv[:, :1], caches[1], ids, pos, 1)


def test_repeat_calls_keep_every_check():
    """Layer calls that repeat the last call's lists and tensor signature skip
    the re-validation; the result is the full path's, and a call that differs
    in anything the reference wrapper checks still raises its error."""
    from pagedserve_b200 import PagedKVCache, paged_decode_attention, paged_decode_attention_with_write
    from pagedserve_b200.attention import clear_metadata_cache
    lens = [5, 40, 17]
    cache = PagedKVCache(num_blocks=32, num_layers=3, num_kv_heads=2, head_dim=64, block_size=16,
                         dtype=torch.bfloat16, device="cuda", free_order=np.random.default_rng(4).permutation(32))
    ids = [f"r{i}" for i in range(len(lens))]
    for rid, n in zip(ids, lens):
        cache.allocate(rid, n)
    g = torch.Generator(device="cuda").manual_seed(3)
    cache.kv_cache.k_cache.copy_(torch.randn(cache.kv_cache.k_cache.shape, generator=g, device="cuda"))
    cache.kv_cache.v_cache.copy_(torch.randn(cache.kv_cache.v_cache.shape, generator=g, device="cuda"))
    pos = [n - 1 for n in lens]
    q = torch.randn(len(lens), 14, 1, 64, generator=g, device="cuda").to(torch.bfloat16)
    nk = torch.randn(len(lens), 2, 64, generator=g, device="cuda").to(torch.bfloat16)
    nv = torch.randn(len(lens), 2, 64, generator=g, device="cuda").to(torch.bfloat16)
    first = [paged_decode_attention_with_write(q, nk, nv, cache, ids, pos, layer) for layer in range(3)]
    again = [paged_decode_attention_with_write(q, nk, nv, cache, ids, pos, layer) for layer in range(3)]
    plain = paged_decode_attention(q, cache, ids, pos, 2)
    clear_metadata_cache(cache)
    full = paged_decode_attention_with_write(q, nk, nv, cache, ids, pos, 2)
    torch.cuda.synchronize()
    for a, b in zip(first, again):
        assert torch.equal(a, b)
    assert torch.equal(full, again[2]) and torch.equal(plain, again[2])
    with pytest.raises(ValueError, match="Invalid layer"):
        paged_decode_attention_with_write(q, nk, nv, cache, ids, pos, 3)
    with pytest.raises(ValueError, match="Invalid layer"):
        paged_decode_attention(q, cache, ids, pos, -1)
    with pytest.raises(ValueError, match="Invalid position"):
        paged_decode_attention_with_write(q, nk, nv, cache, ids, [pos[0], pos[1] + 1, pos[2]], 0)
    with pytest.raises(ValueError, match="unique"):
        paged_decode_attention_with_write(q, nk, nv, cache, [ids[0], ids[0], ids[2]], pos, 0)
    with pytest.raises(ValueError, match="dtype"):
        paged_decode_attention_with_write(q.float(), nk, nv, cache, ids, pos, 0)
    with pytest.raises(ValueError, match="Expected K/V shape"):
        paged_decode_attention_with_write(q, nk[:, :1], nv[:, :1], cache, ids, pos, 0)
    # after the errors, the repeat path still returns the full path's result
    again2 = paged_decode_attention_with_write(q, nk, nv, cache, ids, pos, 2)
    torch.cuda.synchronize()
    assert torch.equal(again2, full)


def test_kept_metadata_survives_many_new_iterations():
    """A position list kept in the metadata store (hit between every new
    iteration, so it never ages out) still decodes with its own lengths after
    many more iterations over the same device table have uploaded theirs."""
    from pagedserve_b200 import PagedKVCache, paged_decode_attention
    from pagedserve_b200.attention import clear_metadata_cache
    lens = [40, 61, 33]
    cache = PagedKVCache(num_blocks=32, num_layers=1, num_kv_heads=2, head_dim=64, block_size=16,
                         dtype=torch.bfloat16, device="cuda", free_order=np.random.default_rng(6).permutation(32))
    ids = [f"r{i}" for i in range(len(lens))]
    for rid, n in zip(ids, lens):
        cache.allocate(rid, n)
    g = torch.Generator(device="cuda").manual_seed(8)
    cache.kv_cache.k_cache.copy_(torch.randn(cache.kv_cache.k_cache.shape, generator=g, device="cuda"))
    cache.kv_cache.v_cache.copy_(torch.randn(cache.kv_cache.v_cache.shape, generator=g, device="cuda"))
    q = torch.randn(len(lens), 14, 1, 64, generator=g, device="cuda").to(torch.bfloat16)
    kept = [n - 1 for n in lens]
    first = paged_decode_attention(q, cache, ids, kept, 0)
    for k in range(1, 12):
        paged_decode_attention(q, cache, ids, [n - 1 - k for n in lens], 0)
        again = paged_decode_attention(q, cache, ids, list(kept), 0)
    clear_metadata_cache(cache)
    fresh = paged_decode_attention(q, cache, ids, kept, 0)
    torch.cuda.synchronize()
    assert torch.equal(again, first) and torch.equal(fresh, first)
