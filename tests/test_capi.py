"""The C-ABI library on the CPU: it loads, exports every symbol the header
declares, and its argument checks answer without touching a GPU."""

from __future__ import annotations

import ctypes
import os
import re
import subprocess

import pytest
import torch

from pagedserve_b200 import _native

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "pagedserve_b200.h")


def _declared():
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(psb_[a-z0-9_]+)\s*\(", text)))


def test_library_exports_every_declared_symbol():
    lib = _native.load()
    declared = _declared()
    assert len(declared) >= 10
    out = subprocess.run(["nm", "-D", "--defined-only", _native.LIB_PATH], capture_output=True, text=True,
                         check=True).stdout
    exported = set(re.findall(r"\bT (psb_[a-z0-9_]+)", out))
    missing = [s for s in declared if s not in exported]
    assert not missing, missing
    for s in declared:
        assert hasattr(lib, s)


def test_binding_covers_header():
    assert set(_declared()) <= set(_native.SIGNATURES)


def test_version_and_status_strings():
    lib = _native.load()
    assert lib.psb_version().decode().startswith("pagedserve_b200")
    assert lib.psb_status_string(0).decode() == "ok"
    assert lib.psb_status_string(-2).decode() == "workspace too small"


def test_workspace_size_grows_with_context_and_batch():
    lib = _native.load()
    a = lib.psb_paged_decode_workspace_size(256, 14, 2, 64, 16, 8192, _native.PSB_BF16)
    b = lib.psb_paged_decode_workspace_size(256, 14, 2, 64, 16, 16384, _native.PSB_BF16)
    c = lib.psb_paged_decode_workspace_size(512, 14, 2, 64, 16, 8192, _native.PSB_BF16)
    assert 0 < a < b and a < c
    # bad geometry -> 0
    assert lib.psb_paged_decode_workspace_size(4, 14, 3, 64, 16, 128, _native.PSB_BF16) == 0


def test_argument_checks_need_no_gpu():
    lib = _native.load()
    null = None
    # null pointers / bad geometry are rejected before any CUDA call
    assert lib.psb_paged_decode(null, 0, 0, null, 0, 0, null, null, null, 0, null, 1, 14, 0, 1, 8, 2, 16, 64,
                                _native.PSB_BF16, 16, 0.125, null, 0, null, null) == _native.PSB_ERR_INVALID
    assert lib.psb_reshape_and_cache(null, 0, 0, null, 0, 0, null, null, null, 1, 0, 1, 8, 2, 16, 64,
                                     _native.PSB_BF16, null, null) == _native.PSB_ERR_INVALID
    assert lib.psb_reshape_and_cache(null, 0, 0, null, 0, 0, null, null, null, 0, 0, 1, 8, 2, 16, 64,
                                     _native.PSB_BF16, null, null) == _native.PSB_OK  # zero tokens: no-op
    assert lib.psb_varlen_prefill(null, 0, 0, null, 0, 0, null, 0, 0, null, 0, 0, null, 1, 4, 4, 14, 3, 64,
                                  _native.PSB_BF16, 0.125, null, null) == _native.PSB_ERR_INVALID
    assert lib.psb_pack_step(null, 4, 1, null, null, null, 0, 0, 16, null, null, null, null, null, 4, null,
                             null) == _native.PSB_OK
    # select_tokens: null buffers, too many EOS ids, a cluster wider than 8,
    # overlapping rows and an empty vocabulary are rejected; an empty batch is a no-op
    bf16 = _native.PSB_BF16
    assert lib.psb_select_tokens(null, 8, 2, 8, bf16, null, 0, null, null, null, 0, null,
                                 null) == _native.PSB_ERR_INVALID
    assert lib.psb_select_tokens(null, 8, 0, 8, bf16, null, 0, null, null, null, 0, null, null) == _native.PSB_OK
    assert lib.psb_select_tokens(null, 8, 0, 8, bf16, null, 65, null, null, null, 0, null,
                                 null) == _native.PSB_ERR_INVALID
    assert lib.psb_select_tokens(null, 8, 0, 8, bf16, null, 0, null, null, null, 9, null,
                                 null) == _native.PSB_ERR_INVALID
    assert lib.psb_select_tokens(null, 8, 0, 0, bf16, null, 0, null, null, null, 0, null,
                                 null) == _native.PSB_ERR_INVALID
    fake = 1 << 20  # never dereferenced: the stride check fails first
    assert lib.psb_select_tokens(fake, 4, 2, 8, bf16, null, 0, fake, fake, fake, 0, null,
                                 null) == _native.PSB_ERR_INVALID


def test_ops_reject_cpu_tensors():
    from pagedserve_b200 import ops
    k = torch.zeros(1, 4, 2, 16, 64)
    with pytest.raises(ValueError, match="requires CUDA"):
        ops.paged_decode(torch.zeros(1, 4, 64), k, k, torch.zeros(1, 1, dtype=torch.int32),
                         torch.ones(1, dtype=torch.int32), 0)
    with pytest.raises(ValueError, match="requires CUDA"):
        ops.reshape_and_cache(torch.zeros(1, 2, 64), torch.zeros(1, 2, 64), k, k, torch.zeros(1, dtype=torch.int64), 0)


def test_drop_in_rejects_cpu_query():
    """test_triton_paged_decode.py:65-74: a CPU query raises 'requires CUDA'."""
    from pagedserve_b200 import PagedKVCache, paged_decode_attention
    cache = PagedKVCache(num_blocks=4, num_layers=1, num_kv_heads=1, head_dim=4, block_size=2, dtype=torch.float32,
                         device="cpu")
    cache.allocate("a", 1)
    with pytest.raises(ValueError, match="requires CUDA"):
        paged_decode_attention(torch.randn(1, 1, 1, 4), cache, ["a"], [0], 0)


def test_static_decode_checks_need_no_gpu():
    """The allocation-free decode rejects bad arguments and geometries whose
    scratch would exceed its fixed capacity before any CUDA call."""
    lib = _native.load()
    cap = lib.psb_paged_decode_static_capacity()
    assert cap == 32 << 20
    null, fake = None, 256  # never dereferenced: every call below is rejected first
    assert lib.psb_paged_decode_static(null, 0, 0, null, 0, 0, null, null, null, 0, null, 1, 14, 0, 1, 8, 2, 16, 64,
                                       _native.PSB_BF16, 16, 0.125, null, null) == _native.PSB_ERR_INVALID
    # on the CUDA-core path (fp32 here), 256 sequences of up to 8192 tokens
    # need ~115 MiB of per-chunk partials: rejected before any CUDA call
    assert lib.psb_paged_decode_workspace_size(256, 14, 2, 64, 16, 8192, _native.PSB_F32) > cap
    assert lib.psb_paged_decode_static(fake, 896, 64, fake, 896, 64, fake, fake, fake, 512, fake, 256, 14, 0, 1,
                                       40000, 2, 16, 64, _native.PSB_F32, 8192, 0.125, null,
                                       null) == _native.PSB_ERR_WORKSPACE
    # a misaligned bf16 query also takes that path, and is rejected the same way
    assert lib.psb_paged_decode_static(fake + 2, 896, 64, fake, 896, 64, fake, fake, fake, 512, fake, 256, 14, 0, 1,
                                       40000, 2, 16, 64, _native.PSB_BF16, 8192, 0.125, null,
                                       null) == _native.PSB_ERR_WORKSPACE
    # 64 sequences of up to 4096 tokens fit
    assert 0 < lib.psb_paged_decode_workspace_size(64, 14, 2, 64, 16, 4096, _native.PSB_BF16) <= cap
    # bad geometry (q heads not a multiple of kv heads)
    assert lib.psb_paged_decode_static(fake, 0, 0, fake, 0, 0, fake, fake, fake, 8, fake, 4, 14, 0, 1, 8, 3, 16, 64,
                                       _native.PSB_BF16, 128, 0.125, null, null) == _native.PSB_ERR_INVALID


def test_decode_args_struct_and_checks():
    """psb_decode_args has the binding's layout, and psb_paged_decode_args
    rejects a null struct, one null new row pointer, and the null pointers
    psb_paged_decode rejects, before any CUDA call."""
    lib = _native.load()
    assert lib.psb_decode_args_size() == ctypes.sizeof(_native.DecodeArgs)
    offsets = {name: getattr(_native.DecodeArgs, name).offset for name, _ in _native.DecodeArgs._fields_}
    assert offsets["k_cache"] == 0 and offsets["batch"] == 72 and offsets["scale"] == 104
    null = None
    assert lib.psb_paged_decode_args(null, null, 0, 0, null, 0, 0, null, 0, 0, null, 0, 0, 0,
                                     null) == _native.PSB_ERR_INVALID
    a = _native.DecodeArgs(batch=1, q_heads=14, num_layers=1, num_blocks=8, num_kv_heads=2, block_size=16,
                           head_dim=64, dtype=_native.PSB_BF16, max_context=16, table_stride=1, scale=0.125)
    ap = ctypes.addressof(a)
    assert lib.psb_paged_decode_args(ap, null, 0, 0, null, 0, 0, null, 0, 0, null, 0, 0, 0,
                                     null) == _native.PSB_ERR_INVALID  # null query / pools / table
    assert lib.psb_paged_decode_args(ap, 16, 64, 64, 16, 64, 64, 16, 0, 0, null, 0, 0, 0,
                                     null) == _native.PSB_ERR_INVALID  # new_key without new_value


def test_bounded_wait_check_rejects_null_flag():
    lib = _native.load()
    assert lib.psb_bounded_wait_check(None, None) == _native.PSB_ERR_INVALID
