"""The allocation-free decode entry point (psb_paged_decode_static) on the GPU.

Called straight through the C ABI and compared with the workspace entry point
(ops.paged_decode) and the exact oracle, twice in a row on the same stream so
the second call runs on scratch the first one used.  This file is collected
last so it also runs after every other GPU test has used the library; it
passes alone too.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import paged_attention as ora
from tests.helpers import TOL, TORCH_DTYPES, err_stats, to_dev

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module", autouse=True)
def _cuda():
    if not torch.cuda.is_available():
        pytest.fail("CUDA device required for -m gpu tests")


def _case(dtype, batch, max_len, hq, hkv, d, bs, seed, typical=None):
    rng = np.random.default_rng(seed)
    lens = [int(x) for x in rng.integers(1, (typical or max_len) + 1, size=batch)]
    lens[0] = max_len
    need = [-(-n // bs) for n in lens]
    nb = sum(need) + 5
    perm = rng.permutation(nb)
    tables, at = [], 0
    for k in need:
        tables.append(perm[at:at + k].tolist())
        at += k
    layers, layer = 2, 1
    k_cache = ora.round_to(rng.standard_normal((layers, nb, hkv, bs, d), dtype=np.float32), dtype)
    v_cache = ora.round_to(rng.standard_normal((layers, nb, hkv, bs, d), dtype=np.float32), dtype)
    q = ora.round_to(rng.standard_normal((batch, hq, d), dtype=np.float32), dtype)
    return dict(q=q, k=k_cache, v=v_cache, tables=tables, lens=lens, layer=layer, dtype=dtype,
                max_context=max(need) * bs)


def _call_static(lib, q, out, k, v, table, lens, layer, max_context, err):
    nl, nb, hkv, bs, d = k.shape
    from pagedserve_b200 import ops
    return lib.psb_paged_decode_static(
        q.data_ptr(), q.stride(0), q.stride(1), out.data_ptr(), out.stride(0), out.stride(1), k.data_ptr(),
        v.data_ptr(), table.data_ptr(), table.stride(0), lens.data_ptr(), q.shape[0], q.shape[1], layer, nl, nb, hkv,
        bs, d, ops.dtype_code(q.dtype), max_context, d ** -0.5, err.data_ptr(),
        torch.cuda.current_stream().cuda_stream)


@pytest.mark.parametrize("dtype,batch,max_len,hq,hkv,d,bs", [
    ("bfloat16", 48, 3000, 14, 2, 64, 16),   # fast path, split-K over up to 24 chunks
    ("float16", 9, 700, 14, 2, 64, 16),
    ("float32", 12, 900, 8, 2, 32, 8),       # generic path
])
def test_static_decode_matches_workspace_decode(dtype, batch, max_len, hq, hkv, d, bs):
    from pagedserve_b200 import _native, ops
    lib = _native.load()
    c = _case(dtype, batch, max_len, hq, hkv, d, bs, seed=batch * 31 + max_len)
    need = lib.psb_paged_decode_workspace_size(batch, hq, hkv, d, bs, c["max_context"],
                                               ops.dtype_code(TORCH_DTYPES[dtype]))
    assert 0 < need <= lib.psb_paged_decode_static_capacity()
    q = to_dev(c["q"], dtype)
    k, v = to_dev(c["k"], dtype), to_dev(c["v"], dtype)
    table = torch.from_numpy(ora.padded_block_table(c["tables"])).cuda()
    lens = torch.tensor(c["lens"], dtype=torch.int32, device="cuda")
    err = torch.zeros(1, dtype=torch.int32, device="cuda")

    want = ops.paged_decode(q, k, v, table, lens, c["layer"], max_context=c["max_context"])
    exact = ora.decode_attention(c["q"], c["k"], c["v"], c["tables"], c["lens"], c["layer"])
    max_tol, mean_tol = TOL[dtype]
    outs = []
    for _ in range(2):
        out = torch.full_like(q, float("nan"))
        status = _call_static(lib, q, out, k, v, table, lens, c["layer"], c["max_context"], err)
        _native.check(status, "paged_decode_static")
        outs.append(out)
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    for out in outs:
        assert not torch.isnan(out).any()
        torch.testing.assert_close(out.float(), want.float(), rtol=0, atol=max_tol)
        mx, mean = err_stats(out, exact)
        assert mx <= max_tol and mean <= mean_tol, (mx, mean)


def test_static_decode_shrinking_then_growing_batch():
    """A smaller call after a larger one (and back) finds its counters zero."""
    from pagedserve_b200 import _native, ops
    lib = _native.load()
    big = _case("bfloat16", 40, 2500, 14, 2, 64, 16, seed=1)
    small = _case("bfloat16", 5, 400, 14, 2, 64, 16, seed=2)
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    for c in (big, small, big):
        q = to_dev(c["q"], "bfloat16")
        k, v = to_dev(c["k"], "bfloat16"), to_dev(c["v"], "bfloat16")
        table = torch.from_numpy(ora.padded_block_table(c["tables"])).cuda()
        lens = torch.tensor(c["lens"], dtype=torch.int32, device="cuda")
        out = torch.empty_like(q)
        _native.check(_call_static(lib, q, out, k, v, table, lens, c["layer"], c["max_context"], err),
                      "paged_decode_static")
        torch.cuda.synchronize()
        exact = ora.decode_attention(c["q"], c["k"], c["v"], c["tables"], c["lens"], c["layer"])
        mx, mean = err_stats(out, exact)
        assert mx <= 2e-2 and mean <= 2e-3, (mx, mean)
    assert int(err.item()) == 0


def test_static_decode_serving_batch_fits():
    """The serving batch (256 bf16 sequences, contexts up to 8192 tokens)
    takes the fast path, whose scratch is a fixed ~10.8 MB: it fits the
    array, matches the workspace entry point and the oracle."""
    from pagedserve_b200 import _native, ops
    lib = _native.load()
    c = _case("bfloat16", 256, 8192, 14, 2, 64, 16, seed=8192, typical=1024)
    q = to_dev(c["q"], "bfloat16")
    k, v = to_dev(c["k"], "bfloat16"), to_dev(c["v"], "bfloat16")
    table = torch.from_numpy(ora.padded_block_table(c["tables"])).cuda()
    lens = torch.tensor(c["lens"], dtype=torch.int32, device="cuda")
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    want = ops.paged_decode(q, k, v, table, lens, c["layer"], max_context=c["max_context"])
    outs = []
    for _ in range(2):
        out = torch.full_like(q, float("nan"))
        _native.check(_call_static(lib, q, out, k, v, table, lens, c["layer"], c["max_context"], err),
                      "paged_decode_static")
        outs.append(out)
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    rows = [0, 1, 77, 255]  # the oracle on a few rows (one with the longest context)
    exact = ora.decode_attention(c["q"][rows], c["k"], c["v"], [c["tables"][r] for r in rows],
                                 [c["lens"][r] for r in rows], c["layer"])
    for out in outs:
        torch.testing.assert_close(out.float(), want.float(), rtol=0, atol=2e-2)
        mx, mean = err_stats(out[rows], exact)
        assert mx <= 2e-2 and mean <= 2e-3, (mx, mean)


def test_static_decode_rejects_oversized_geometry():
    """The CUDA-core path (fp32) needs per-chunk partials that grow with
    batch x context: 256 sequences of 8192 tokens exceed the array."""
    from pagedserve_b200 import _native
    lib = _native.load()
    q = torch.zeros(256, 14, 64, dtype=torch.float32, device="cuda")
    k = torch.zeros(1, 8, 2, 16, 64, dtype=torch.float32, device="cuda")
    table = torch.zeros(256, 512, dtype=torch.int32, device="cuda")
    lens = torch.ones(256, dtype=torch.int32, device="cuda")
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    out = torch.empty_like(q)
    status = _call_static(lib, q, out, k, k, table, lens, 0, 8192, err)
    assert status == _native.PSB_ERR_WORKSPACE
    with pytest.raises(_native.NativeError, match="workspace too small"):
        _native.check(status, "paged_decode_static")
