"""The decoder-layer glue kernels against the transformers Qwen2 modules they
replace: ``act_fn(gate_proj(x)) * up_proj(x)`` (Qwen2MLP, reference model
runner engine.py:595) and ``residual + x`` followed by Qwen2RMSNorm
(engine.py:577-598)."""

from __future__ import annotations

import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32])
@pytest.mark.parametrize("rows,inter", [(1, 4864), (256, 4864), (1000, 4864), (7, 40), (3, 6)])
def test_silu_and_mul_matches_torch_bit_exact(dtype, rows, inter):
    """Each product and the SiLU are rounded to the storage type as PyTorch
    rounds them (fp32 arithmetic, the accurate exponential), so the outputs
    are bit-identical; 16-byte path (inter a multiple of 8 or 4) and the
    element-wise path."""
    from pagedserve_b200 import ops
    g = torch.Generator(device="cuda").manual_seed(rows * 31 + inter)
    gu = (torch.randn(rows, 2 * inter, generator=g, device="cuda") * 3).to(dtype)
    out = ops.silu_and_mul(gu)
    want = torch.nn.functional.silu(gu[:, :inter]) * gu[:, inter:]
    torch.cuda.synchronize()
    assert out.shape == (rows, inter) and out.dtype == dtype
    assert torch.equal(out, want)


def test_silu_and_mul_strided_rows_and_output():
    """Rows of a wider buffer in and out; the columns past each row stay untouched."""
    from pagedserve_b200 import ops
    rows, inter = 33, 4864
    g = torch.Generator(device="cuda").manual_seed(5)
    big = torch.randn(rows, 2 * inter + 64, generator=g, device="cuda").to(torch.bfloat16)
    gu = big[:, :2 * inter]
    wide = torch.full((rows, inter + 32), 3.0, dtype=torch.bfloat16, device="cuda")
    out = ops.silu_and_mul(gu, out=wide[:, :inter])
    want = torch.nn.functional.silu(gu[:, :inter]) * gu[:, inter:]
    torch.cuda.synchronize()
    assert out.data_ptr() == wide.data_ptr() and torch.equal(out, want)
    assert bool((wide[:, inter:] == 3.0).all())


@pytest.mark.parametrize("dtype,tol", [(torch.bfloat16, 1e-2), (torch.float16, 2e-3), (torch.float32, 1e-5)])
@pytest.mark.parametrize("rows,hidden", [(1, 896), (256, 896), (1000, 896), (5, 4096), (3, 100)])
@pytest.mark.parametrize("with_residual", [True, False])
def test_add_rms_norm_matches_qwen2_rmsnorm(dtype, tol, rows, hidden, with_residual):
    """out = Qwen2RMSNorm(x + residual) (weight * normalised row in fp32,
    rounded to the storage type), and the residual updated in place to
    x + residual; the reduction order differs from torch's mean, so the
    normalised rows agree to the storage type's rounding."""
    from transformers.models.qwen2.modeling_qwen2 import Qwen2RMSNorm
    from pagedserve_b200 import ops
    g = torch.Generator(device="cuda").manual_seed(rows + hidden)
    x = torch.randn(rows, hidden, generator=g, device="cuda").to(dtype)
    res = torch.randn(rows, hidden, generator=g, device="cuda").to(dtype) if with_residual else None
    norm = Qwen2RMSNorm(hidden, eps=1e-6).to(device="cuda", dtype=dtype)
    with torch.no_grad():
        norm.weight.copy_(torch.rand(hidden, generator=g, device="cuda") + 0.5)
        summed = x + res if with_residual else x
        want = norm(summed)
    res_in = res.clone() if with_residual else None
    out = ops.add_rms_norm(x, norm.weight, 1e-6, residual=res_in)
    torch.cuda.synchronize()
    if with_residual:
        assert torch.equal(res_in, summed)  # the sum, rounded once, as torch rounds it
    err = (out.float() - want.float()).abs().max().item()
    assert err <= tol * max(1.0, want.float().abs().max().item()), err
