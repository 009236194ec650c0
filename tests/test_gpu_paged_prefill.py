"""Prefix-aware (chunked) prefill over the paged pool (psb_paged_prefill):
the reference's paged_attention with query_start_position > 0, for packed
batches.  Checked against the reference's own golden output (the prefix
case), the oracle on pools poisoned with NaN outside every context, and
bit-for-bit against psb_varlen_prefill when no prefix exists."""

from __future__ import annotations

import os

import numpy as np
import pytest
import torch

from oracle import paged_attention as ora
from tests.golden.cases import prefill_case
from tests.helpers import TOL, TORCH_DTYPES, err_stats, to_dev

pytestmark = pytest.mark.gpu

HERE = os.path.dirname(os.path.abspath(__file__))
GOLD = np.load(os.path.join(HERE, "golden", "reference_outputs.npz"))


@pytest.fixture(scope="module", autouse=True)
def _cuda():
    if not torch.cuda.is_available():
        pytest.fail("CUDA device required for -m gpu tests")
    import pagedserve_b200._native as native
    native.load()


@pytest.mark.parametrize("name", ["prefix_bf16", "qwen_bf16", "qwen_fp32", "gqa_tiny"])
def test_paged_prefill_matches_reference_golden(name):
    """One request through the pool, as the reference's paged_attention runs
    it (the prefix case starts at position 20), at the reference test's
    tolerance."""
    from pagedserve_b200 import ops
    c = prefill_case(name)
    hq, s, d = c["q"].shape
    ctx = c["start"] + s
    table = torch.tensor([c["table"]], dtype=torch.int32, device="cuda")
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    out = ops.paged_prefill(to_dev(np.transpose(c["q"], (1, 0, 2)), c["dtype"]), to_dev(c["k_cache"], c["dtype"]),
                            to_dev(c["v_cache"], c["dtype"]), table,
                            torch.tensor([ctx], dtype=torch.int32, device="cuda"),
                            torch.tensor([0, s], dtype=torch.int32, device="cuda"), s, 0, error_flag=err)
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    gold = torch.from_numpy(GOLD[f"prefill/{name}"])
    tol = 1e-4 if c["dtype"] == "float32" else 2e-2
    torch.testing.assert_close(out.float().cpu().permute(1, 0, 2), gold, rtol=tol, atol=tol)


def _chunked_case(seed, qlens, ctxs, hq, hkv, d, bs, dtype, layers=2, layer=1):
    """Sequences with ctxs[i] tokens in a shuffled pool whose last qlens[i]
    are the new rows; every slot outside the contexts (and every other
    layer) holds NaN."""
    rng = np.random.default_rng(seed)
    need = [-(-c // bs) for c in ctxs]
    nb = sum(need) + 5
    perm = rng.permutation(nb)
    tables, at = [], 0
    for k in need:
        tables.append([int(x) for x in perm[at:at + k]])
        at += k
    kc = ora.round_to(rng.standard_normal((layers, nb, hkv, bs, d)).astype(np.float32), dtype)
    vc = ora.round_to(rng.standard_normal((layers, nb, hkv, bs, d)).astype(np.float32), dtype)
    kp, vp = np.full_like(kc, np.nan), np.full_like(vc, np.nan)
    for t, c in zip(tables, ctxs):
        for pos in range(c):
            kp[layer, t[pos // bs], :, pos % bs] = kc[layer, t[pos // bs], :, pos % bs]
            vp[layer, t[pos // bs], :, pos % bs] = vc[layer, t[pos // bs], :, pos % bs]
    total = int(sum(qlens))
    q = ora.round_to(rng.standard_normal((total, hq, d)).astype(np.float32), dtype)
    cu = np.zeros(len(qlens) + 1, dtype=np.int32)
    cu[1:] = np.cumsum(qlens)
    width = max(need) + 2
    table = np.zeros((len(qlens), width), dtype=np.int32)
    for i, t in enumerate(tables):
        table[i, :len(t)] = t
    return dict(q=q, kc=kc, vc=vc, kp=kp, vp=vp, tables=tables, table=table, cu=cu, ctxs=list(ctxs),
                qlens=list(qlens), layer=layer, bs=bs, width=width)


def _run(c, dtype, poison=True, err=None):
    from pagedserve_b200 import ops
    err = torch.zeros(1, dtype=torch.int32, device="cuda") if err is None else err
    out = ops.paged_prefill(to_dev(c["q"], dtype), to_dev(c["kp"] if poison else c["kc"], dtype),
                            to_dev(c["vp"] if poison else c["vc"], dtype), torch.from_numpy(c["table"]).cuda(),
                            torch.tensor(c["ctxs"], dtype=torch.int32, device="cuda"),
                            torch.from_numpy(c["cu"]).cuda(), max(c["qlens"]), c["layer"], error_flag=err)
    torch.cuda.synchronize()
    return out, int(err.item())


def _oracle(c):
    outs = []
    for i, (n, ctx) in enumerate(zip(c["qlens"], c["ctxs"])):
        qi = np.transpose(c["q"][c["cu"][i]:c["cu"][i + 1]], (1, 0, 2))  # [Hq, n, D]
        o = ora.paged_causal_attention(qi, c["kc"], c["vc"], c["tables"][i], c["layer"], ctx - n)
        outs.append(np.transpose(o, (1, 0, 2)))
    return np.concatenate(outs)


CHUNKED = [
    ([8], [28]),                                   # the reference test's shape: a short chunk after a prefix
    ([1, 17, 130, 64], [1, 40, 130, 1000]),        # decode-like row, prefixes, no prefix, long prefix
    ([300, 129, 5], [4096, 700, 5]),               # chunk of a long context; block-unaligned ends
    ([128, 256], [2048 + 7, 263]),
]


@pytest.mark.parametrize("dtype", ["bfloat16", "float16"])
@pytest.mark.parametrize("qlens,ctxs", CHUNKED)
def test_paged_prefill_tensor_cores_match_oracle(dtype, qlens, ctxs):
    c = _chunked_case(sum(ctxs) + len(qlens), qlens, ctxs, 14, 2, 64, 16, dtype)
    out, err = _run(c, dtype)
    assert err == 0
    mx, mean = err_stats(out, _oracle(c))
    max_tol, mean_tol = TOL[dtype]
    assert mx <= max_tol and mean <= mean_tol, (mx, mean)


@pytest.mark.parametrize("dtype,hq,hkv,d,bs", [("float32", 14, 2, 64, 16), ("bfloat16", 8, 2, 128, 16),
                                               ("float16", 4, 4, 64, 8), ("float32", 4, 2, 4, 2)])
def test_paged_prefill_generic_match_oracle(dtype, hq, hkv, d, bs):
    c = _chunked_case(7, [3, 40, 1], [20, 40, 33], hq, hkv, d, bs, dtype)
    out, err = _run(c, dtype)
    assert err == 0
    mx, mean = err_stats(out, _oracle(c))
    max_tol, mean_tol = TOL[dtype]
    assert mx <= max_tol and mean <= mean_tol, (mx, mean)


def test_no_prefix_equals_varlen_prefill_bit_for_bit():
    """Without a prefix the paged kernel reads the same keys from the pool
    that varlen_prefill reads packed: the outputs are identical."""
    from pagedserve_b200 import ops
    dtype = "bfloat16"
    qlens = [300, 1, 129, 64, 700]
    c = _chunked_case(3, qlens, qlens, 14, 2, 64, 16, dtype)
    out, err = _run(c, dtype)
    assert err == 0
    keys, vals = [], []
    for t, n in zip(c["tables"], qlens):
        keys.append(np.transpose(ora.gather_context(c["kc"], c["layer"], t, n), (1, 0, 2)))
        vals.append(np.transpose(ora.gather_context(c["vc"], c["layer"], t, n), (1, 0, 2)))
    ref = ops.varlen_prefill(to_dev(c["q"], dtype), to_dev(np.concatenate(keys), dtype),
                             to_dev(np.concatenate(vals), dtype), torch.from_numpy(c["cu"]).cuda(), max(qlens))
    torch.cuda.synchronize()
    assert torch.equal(out, ref)


def test_bad_context_and_block_flagged():
    c = _chunked_case(5, [16, 8], [40, 30], 14, 2, 64, 16, "bfloat16")
    c["ctxs"] = [10, 30]  # shorter than its 16 query rows: flagged, clamped
    _, err = _run(c, "bfloat16", poison=False)
    assert err & 4
    c = _chunked_case(5, [16, 8], [40, 30], 14, 2, 64, 16, "bfloat16")
    c["table"][1, 0] = 10 ** 6  # outside the pool: flagged, not read
    _, err = _run(c, "bfloat16", poison=False)
    assert err & 1
