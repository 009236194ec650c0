"""The library's device-side waits are bounded: a wait that can never finish
ends with PSB_DEVERR_TIMEOUT on the host's error flag, not a hang, and the
device keeps running kernels afterwards (psb_bounded_wait_check)."""

from __future__ import annotations

import time

import pytest
import torch

from pagedserve_b200 import _native

pytestmark = pytest.mark.gpu


def test_wait_that_cannot_finish_reports_timeout():
    from pagedserve_b200 import ops
    lib = _native.load()
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    assert lib.psb_bounded_wait_check(err.data_ptr(), torch.cuda.current_stream().cuda_stream) == 0
    torch.cuda.synchronize()
    elapsed = time.perf_counter() - t0
    assert int(err.item()) == 16, _native.describe_device_error(int(err.item()))
    assert 1.5 < elapsed < 60.0, elapsed
    # the context is intact: the next kernel runs and is right
    g = torch.Generator(device="cuda").manual_seed(1)
    gu = torch.randn(64, 2 * 4864, generator=g, device="cuda").to(torch.bfloat16)
    out = ops.silu_and_mul(gu)
    assert torch.equal(out, torch.nn.functional.silu(gu[:, :4864]) * gu[:, 4864:])
