"""Decode parity on the GPU: the sm_100a kernels vs the CPU oracle and the
reference's own golden outputs.

Ports the reference's test_triton_paged_decode.py scenarios (fragmented
interleaved allocations, boundary lengths 1/15/16/17/31/32/33/65, layer
independence, fp32 2e-4 / bf16 2e-2 tolerances) and adds split-K lengths up
to 32768, the serving-scale batch of 256 lognormal contexts, strided queries,
poisoned pools and device-side error reporting.
"""

from __future__ import annotations

import math
import os

import numpy as np
import pytest
import torch

from oracle import paged_attention as ora
from tests.golden.cases import DECODE_CASES, decode_case, fifo_tables
from tests.helpers import TOL, err_stats, poison_unused, to_dev

pytestmark = pytest.mark.gpu

HERE = os.path.dirname(os.path.abspath(__file__))
GOLD = np.load(os.path.join(HERE, "golden", "reference_outputs.npz"))


@pytest.fixture(scope="module", autouse=True)
def _cuda():
    if not torch.cuda.is_available():
        pytest.fail("CUDA device required for -m gpu tests")
    import pagedserve_b200._native as native
    native.load()


def _run_tensor_api(c, poison=True, max_context=None):
    from pagedserve_b200 import ops
    kc, vc = (poison_unused(c["k_cache"], c["v_cache"], c["layer"], c["tables"], c["context_lens"])
              if poison else (c["k_cache"], c["v_cache"]))
    k = to_dev(kc, c["dtype"])
    v = to_dev(vc, c["dtype"])
    q = to_dev(c["q"], c["dtype"])
    table = torch.from_numpy(ora.padded_block_table(c["tables"])).cuda()
    lens = torch.tensor(c["context_lens"], dtype=torch.int32, device="cuda")
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    out = ops.paged_decode(q, k, v, table, lens, c["layer"], error_flag=err, max_context=max_context)
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    return out


@pytest.mark.parametrize("name", DECODE_CASES)
def test_decode_matches_oracle_and_reference(name):
    c = decode_case(name)
    out = _run_tensor_api(c)
    exact = ora.decode_attention(c["q"], c["k_cache"], c["v_cache"], c["tables"], c["context_lens"], c["layer"])
    mx, mean = err_stats(out, exact)
    max_tol, mean_tol = TOL[c["dtype"]]
    assert mx <= max_tol and mean <= mean_tol, (mx, mean)
    # the reference's own output, at the reference test's tolerance
    gold = torch.from_numpy(GOLD[f"decode/{name}"])
    tol = 2e-4 if c["dtype"] == "float32" else 2e-2
    torch.testing.assert_close(out.float().cpu(), gold, rtol=tol, atol=tol)


def _fill_like_reference_test(cache, request_ids, lengths, layers, dtype, seed):
    """Interleaved allocation then growth, every layer filled independently
    (test_triton_paged_decode.py:101-120), through the mirror's write_token."""
    torch.manual_seed(seed)
    for rid in request_ids:
        cache.allocate(rid, 1)
    for rid, n in zip(request_ids, lengths):
        if n > 1:
            cache.append_tokens(rid, n - 1)
    kvh, d = cache.kv_cache.num_kv_heads, cache.kv_cache.head_dim
    for rid, n in zip(request_ids, lengths):
        for layer in range(layers):
            for pos in range(n):
                key = torch.randn(kvh, d, device="cuda", dtype=dtype)
                cache.write_token(rid, layer, pos, key, torch.randn_like(key))


def _oracle_from_cache(cache, query, request_ids, positions, layer):
    kc = cache.kv_cache.k_cache.float().cpu().numpy()
    vc = cache.kv_cache.v_cache.float().cpu().numpy()
    tables = [cache.get_block_table(r).get_blocks() for r in request_ids]
    return ora.decode_attention(query.squeeze(2).float().cpu().numpy(), kc, vc, tables,
                                [p + 1 for p in positions], layer)


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_drop_in_fragmented_blocks(dtype):
    from pagedserve_b200 import PagedKVCache, paged_decode_attention
    lengths, ids = [17, 32, 65], ["a", "b", "c"]
    cache = PagedKVCache(num_blocks=32, num_layers=1, num_kv_heads=2, head_dim=64, block_size=16, dtype=dtype,
                         device="cuda")
    cache.kv_cache.k_cache.fill_(float("nan"))
    cache.kv_cache.v_cache.fill_(float("nan"))
    _fill_like_reference_test(cache, ids, lengths, 1, dtype, 7)
    assert [cache.get_block_table(r).get_blocks() for r in ids] == fifo_tables([1] * 3, lengths, 32, 16)
    query = torch.randn(3, 4, 1, 64, device="cuda", dtype=dtype)
    positions = [n - 1 for n in lengths]
    out = paged_decode_attention(query, cache, ids, positions, layer=0)
    torch.cuda.synchronize()
    assert out.shape == query.shape and out.dtype == dtype
    exact = _oracle_from_cache(cache, query, ids, positions, 0)
    tol = 2e-4 if dtype == torch.float32 else 2e-2
    torch.testing.assert_close(out.squeeze(2).float().cpu(), torch.from_numpy(exact).float(), rtol=tol, atol=tol)


@pytest.mark.parametrize("layer", [0, 1])
@pytest.mark.parametrize("batch_size", [1, 2, 4, 8])
def test_drop_in_layers_and_block_boundaries(layer, batch_size):
    from pagedserve_b200 import PagedKVCache, paged_decode_attention
    lengths = [1, 15, 16, 17, 31, 32, 33, 65][:batch_size]
    ids = [f"boundary-{i}" for i in range(batch_size)]
    cache = PagedKVCache(num_blocks=128, num_layers=2, num_kv_heads=2, head_dim=64, block_size=16,
                         dtype=torch.bfloat16, device="cuda")
    cache.kv_cache.k_cache.fill_(float("nan"))
    cache.kv_cache.v_cache.fill_(float("nan"))
    _fill_like_reference_test(cache, ids, lengths, 2, torch.bfloat16, 1000 + layer * 100 + batch_size)
    query = torch.randn(batch_size, 4, 1, 64, device="cuda", dtype=torch.bfloat16)
    positions = [n - 1 for n in lengths]
    out = paged_decode_attention(query, cache, ids, positions, layer=layer)
    torch.cuda.synchronize()
    exact = _oracle_from_cache(cache, query, ids, positions, layer)
    torch.testing.assert_close(out.squeeze(2).float().cpu(), torch.from_numpy(exact).float(), rtol=2e-2, atol=2e-2)


def _synthetic(seed, lens, dtype="bfloat16", hq=14, hkv=2, d=64, bs=16, slack=1.25, layers=1):
    rng = np.random.default_rng(seed)
    need = sum(-(-n // bs) for n in lens)
    nb = max(1, int(need * slack) + 1)
    perm = rng.permutation(nb)
    tables, at = [], 0
    for n in lens:
        k = -(-n // bs)
        tables.append([int(x) for x in perm[at:at + k]])
        at += k
    shape = (layers, nb, hkv, bs, d)
    mk = (lambda s: ora.bf16_round(rng.standard_normal(s, dtype=np.float32))) if dtype == "bfloat16" else \
         (lambda s: rng.standard_normal(s, dtype=np.float32))
    return dict(dtype=dtype, tables=tables, context_lens=list(lens), layer=layers - 1, k_cache=mk(shape),
                v_cache=mk(shape), q=mk((len(lens), hq, d)))


@pytest.mark.parametrize("lens", [[1, 255, 256, 257, 1000, 8192], [32768, 5], [512, 513, 4095, 4096, 4097]])
def test_split_k_long_contexts(lens):
    c = _synthetic(5, lens)
    out = _run_tensor_api(c)
    exact = ora.decode_attention(c["q"], c["k_cache"], c["v_cache"], c["tables"], c["context_lens"], c["layer"])
    mx, mean = err_stats(out, exact)
    assert mx <= 2e-2 and mean <= 2e-3, (mx, mean)


def test_serving_scale_batch_256():
    """256 sequences, lognormal(median 1024, sigma 0.8) clipped to [16, 8192],
    pool 1.25x the need, blocks shuffled: the serving-scale decode workload."""
    rng = np.random.default_rng(2)
    lens = np.clip(np.round(rng.lognormal(math.log(1024), 0.8, 256)), 16, 8192).astype(int).tolist()
    c = _synthetic(3, lens)
    out = _run_tensor_api(c, poison=True)
    exact = ora.decode_attention(c["q"], c["k_cache"], c["v_cache"], c["tables"], c["context_lens"], c["layer"])
    mx, mean = err_stats(out, exact)
    assert mx <= 2e-2 and mean <= 2e-3, (mx, mean)


@pytest.mark.parametrize("hq,hkv", [(16, 1), (8, 8), (6, 3)])
def test_other_gqa_ratios(hq, hkv):
    c = _synthetic(9, [3, 70, 300], hq=hq, hkv=hkv)
    out = _run_tensor_api(c)
    exact = ora.decode_attention(c["q"], c["k_cache"], c["v_cache"], c["tables"], c["context_lens"], c["layer"])
    mx, mean = err_stats(out, exact)
    assert mx <= 2e-2 and mean <= 2e-3, (mx, mean)


@pytest.mark.parametrize("d,bs", [(128, 16), (64, 8), (32, 32)])
def test_other_head_dims_and_block_sizes(d, bs):
    c = _synthetic(13, [1, 40, 333], d=d, bs=bs)
    out = _run_tensor_api(c)
    exact = ora.decode_attention(c["q"], c["k_cache"], c["v_cache"], c["tables"], c["context_lens"], c["layer"])
    mx, mean = err_stats(out, exact)
    assert mx <= 2e-2 and mean <= 2e-3, (mx, mean)


def test_strided_query_and_output_like_projection_layout():
    """q from ``proj(h).view(B, 1, Hq, D).transpose(1, 2)`` (batched_paged_attention.py:87-91)."""
    from pagedserve_b200 import ops
    c = _synthetic(17, [20, 300, 700])
    kc, vc = poison_unused(c["k_cache"], c["v_cache"], c["layer"], c["tables"], c["context_lens"])
    k, v = to_dev(kc, "bfloat16"), to_dev(vc, "bfloat16")
    # a fused QKV projection output: q is a strided view of [B, (14 + 2 + 2) * 64]
    qkv = torch.zeros(3, 18 * 64, device="cuda", dtype=torch.bfloat16)
    qkv[:, : 14 * 64] = to_dev(c["q"].reshape(3, 14 * 64), "bfloat16")
    q = qkv[:, : 14 * 64].view(3, 14, 1, 64)  # [B, Hq, 1, D], row stride 1152
    assert not q.is_contiguous()
    table = torch.from_numpy(ora.padded_block_table(c["tables"])).cuda()
    lens = torch.tensor(c["context_lens"], dtype=torch.int32, device="cuda")
    out = ops.paged_decode(q, k, v, table, lens, c["layer"])
    exact = ora.decode_attention(c["q"], c["k_cache"], c["v_cache"], c["tables"], c["context_lens"], c["layer"])
    mx, mean = err_stats(out.squeeze(2), exact)
    assert mx <= 2e-2 and mean <= 2e-3


def test_workspace_reuse_and_varying_batches():
    """Split-K counters must be left at zero: repeated and differently sized
    calls on the shared workspace give identical results."""
    c = _synthetic(21, [5000, 9, 2600, 300])
    first = _run_tensor_api(c)
    second = _run_tensor_api(c)
    assert torch.equal(first, second)
    small = _synthetic(22, [700])
    _run_tensor_api(small)
    third = _run_tensor_api(c)
    assert torch.equal(first, third)


def test_bad_block_id_is_reported_not_faulted():
    from pagedserve_b200 import ops
    c = _synthetic(23, [40, 40])
    k, v = to_dev(c["k_cache"], "bfloat16"), to_dev(c["v_cache"], "bfloat16")
    q = to_dev(c["q"], "bfloat16")
    table = torch.from_numpy(ora.padded_block_table(c["tables"])).cuda()
    table[1, 1] = 10_000_000  # outside the pool
    lens = torch.tensor(c["context_lens"], dtype=torch.int32, device="cuda")
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    out = ops.paged_decode(q, k, v, table, lens, c["layer"], error_flag=err)
    torch.cuda.synchronize()
    assert int(err.item()) & 1
    exact = ora.decode_attention(c["q"][:1], c["k_cache"], c["v_cache"], c["tables"][:1], [40], c["layer"])
    mx, _ = err_stats(out[:1], exact)
    assert mx <= 2e-2  # the untouched sequence is still right


def test_context_longer_than_table_is_clamped_and_reported():
    from pagedserve_b200 import ops
    c = _synthetic(29, [32, 16])
    k, v = to_dev(c["k_cache"], "bfloat16"), to_dev(c["v_cache"], "bfloat16")
    q = to_dev(c["q"], "bfloat16")
    table = torch.from_numpy(ora.padded_block_table(c["tables"])).cuda()
    lens = torch.tensor([32, 999], dtype=torch.int32, device="cuda")
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    ops.paged_decode(q, k, v, table, lens, c["layer"], error_flag=err)
    torch.cuda.synchronize()
    assert int(err.item()) & 4


def test_float16_cache():
    c = decode_case("qwen_f16")
    out = _run_tensor_api(c)
    exact = ora.decode_attention(c["q"], c["k_cache"], c["v_cache"], c["tables"], c["context_lens"], c["layer"])
    mx, mean = err_stats(out, exact)
    assert mx <= TOL["float16"][0] and mean <= TOL["float16"][1]
