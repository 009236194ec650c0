"""ctypes binding of libpagedserve_b200.so (the C ABI in include/pagedserve_b200.h).

The library is built in-tree by ``python -m pagedserve_b200.build``.  There is
no fallback: if the library is missing or fails to load, every entry point
raises.
"""

from __future__ import annotations

import ctypes
import os
import threading

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libpagedserve_b200.so")

PSB_F32, PSB_F16, PSB_BF16 = 0, 1, 2
PSB_OK, PSB_ERR_INVALID, PSB_ERR_WORKSPACE, PSB_ERR_UNSUPPORTED, PSB_ERR_CUDA = 0, -1, -2, -3, -4

DEVERR_BITS = {
    1: "block id outside the pool",
    2: "slot outside the pool",
    4: "context length outside the block table",
    8: "split-K work exceeded the workspace",
    16: "async wait exceeded its bound",
    32: "cu_seqlens malformed",
    64: "a row had no tokens left to generate",
}

_c_void_p, _i32, _i64, _f32, _sz = ctypes.c_void_p, ctypes.c_int32, ctypes.c_int64, ctypes.c_float, ctypes.c_size_t


class DecodeArgs(ctypes.Structure):
    """``psb_decode_args``: the fixed arguments of psb_paged_decode_args
    (same fields, order and types as the header; ``load`` checks the size
    against ``psb_decode_args_size``)."""

    _fields_ = [("k_cache", _c_void_p), ("v_cache", _c_void_p), ("block_tables", _c_void_p),
                ("table_stride", _i64), ("context_lens", _c_void_p), ("num_blocks", _i64),
                ("workspace", _c_void_p), ("workspace_bytes", _sz), ("error_flag", _c_void_p),
                ("batch", _i32), ("q_heads", _i32), ("num_layers", _i32), ("num_kv_heads", _i32),
                ("block_size", _i32), ("head_dim", _i32), ("dtype", _i32), ("max_context", _i32),
                ("scale", _f32), ("reserved", _i32)]


# name -> (restype, argtypes); mirrors include/pagedserve_b200.h
SIGNATURES = {
    "psb_version": (ctypes.c_char_p, []),
    "psb_status_string": (ctypes.c_char_p, [ctypes.c_int]),
    "psb_last_cuda_error": (ctypes.c_int, []),
    "psb_device_sm_count": (ctypes.c_int, []),
    "psb_bounded_wait_check": (ctypes.c_int, [_c_void_p, _c_void_p]),
    "psb_reshape_and_cache": (ctypes.c_int, [
        _c_void_p, _i64, _i64, _c_void_p, _i64, _i64, _c_void_p, _c_void_p, _c_void_p, _i32, _i32, _i32, _i64,
        _i32, _i32, _i32, _i32, _c_void_p, _c_void_p]),
    "psb_paged_decode_workspace_size": (_sz, [_i32, _i32, _i32, _i32, _i32, _i32, _i32]),
    "psb_paged_decode_workspace_init": (ctypes.c_int, [_c_void_p, _sz, _i32, _i32, _c_void_p]),
    "psb_paged_decode": (ctypes.c_int, [
        _c_void_p, _i64, _i64, _c_void_p, _i64, _i64, _c_void_p, _c_void_p, _c_void_p, _i64, _c_void_p, _i32,
        _i32, _i32, _i32, _i64, _i32, _i32, _i32, _i32, _i32, _f32, _c_void_p, _sz, _c_void_p, _c_void_p]),
    "psb_rope_reshape_and_cache": (ctypes.c_int, [
        _c_void_p, _i64, _i64, _c_void_p, _i64, _i64, _c_void_p, _i64, _i64, _c_void_p, _i64, _i64, _c_void_p, _i64,
        _i64, _c_void_p, _c_void_p, _i64, _c_void_p, _c_void_p, _c_void_p, _i32, _i32, _i32, _i32, _i64, _i32, _i32,
        _i32, _i32, _c_void_p, _c_void_p]),
    "psb_paged_prefill": (ctypes.c_int, [
        _c_void_p, _i64, _i64, _c_void_p, _c_void_p, _c_void_p, _i64, _c_void_p, _c_void_p, _i64, _i64, _c_void_p,
        _i32, _i32, _i32, _i32, _i32, _i32, _i32, _i64, _i32, _i32, _i32, _i32, _f32, _c_void_p, _c_void_p]),
    "psb_paged_decode_append": (ctypes.c_int, [
        _c_void_p, _i64, _i64, _c_void_p, _i64, _i64, _c_void_p, _c_void_p, _c_void_p, _i64, _i64, _c_void_p, _i64,
        _i64, _c_void_p, _i64, _c_void_p, _i32, _i32, _i32, _i32, _i64, _i32, _i32, _i32, _i32, _i32, _f32,
        _c_void_p, _sz, _c_void_p, _c_void_p]),
    "psb_decode_args_size": (_sz, []),
    "psb_paged_decode_args": (ctypes.c_int, [
        _c_void_p, _c_void_p, _i64, _i64, _c_void_p, _i64, _i64, _c_void_p, _i64, _i64, _c_void_p, _i64, _i64,
        _i32, _c_void_p]),
    "psb_paged_decode_static": (ctypes.c_int, [
        _c_void_p, _i64, _i64, _c_void_p, _i64, _i64, _c_void_p, _c_void_p, _c_void_p, _i64, _c_void_p, _i32,
        _i32, _i32, _i32, _i64, _i32, _i32, _i32, _i32, _i32, _f32, _c_void_p, _c_void_p]),
    "psb_paged_decode_static_capacity": (_sz, []),
    "psb_varlen_prefill": (ctypes.c_int, [
        _c_void_p, _i64, _i64, _c_void_p, _i64, _i64, _c_void_p, _i64, _i64, _c_void_p, _i64, _i64, _c_void_p,
        _i32, _i32, _i32, _i32, _i32, _i32, _i32, _f32, _c_void_p, _c_void_p]),
    "psb_select_tokens": (ctypes.c_int, [
        _c_void_p, _i64, _i32, _i32, _i32, _c_void_p, _i32, _c_void_p, _c_void_p, _c_void_p, _i32, _c_void_p,
        _c_void_p]),
    "psb_add_rms_norm": (ctypes.c_int, [
        _c_void_p, _i64, _c_void_p, _i64, _c_void_p, _c_void_p, _i64, _i32, _i32, _f32, _i32, _c_void_p]),
    "psb_silu_and_mul": (ctypes.c_int, [_c_void_p, _i64, _c_void_p, _i64, _i32, _i32, _i32, _c_void_p]),
    "psb_pack_step": (ctypes.c_int, [
        _c_void_p, _i64, _i32, _c_void_p, _c_void_p, _c_void_p, _i32, _i32, _i32, _c_void_p, _c_void_p,
        _c_void_p, _c_void_p, _c_void_p, _i32, _c_void_p, _c_void_p]),
}

_lock = threading.Lock()
_lib = None


class NativeError(RuntimeError):
    """A C-ABI call returned a non-zero status."""


def load() -> ctypes.CDLL:
    """Load the library once and declare every entry point's signature."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is not None:
            return _lib
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(
                f"{LIB_PATH} is missing; build it with `python -m pagedserve_b200.build` (nvcc, sm_100a)")
        lib = ctypes.CDLL(LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        if lib.psb_decode_args_size() != ctypes.sizeof(DecodeArgs):
            raise RuntimeError(f"psb_decode_args is {lib.psb_decode_args_size()} bytes in {LIB_PATH}, "
                               f"{ctypes.sizeof(DecodeArgs)} in the binding")
        _lib = lib
    return _lib


def check(status: int, what: str) -> None:
    if status == PSB_OK:
        return
    lib = load()
    msg = lib.psb_status_string(status).decode()
    if status == PSB_ERR_CUDA:
        msg += f" (cuda error {lib.psb_last_cuda_error()})"
    raise NativeError(f"{what} failed: {msg} [{status}]")


def describe_device_error(bits: int) -> str:
    return ", ".join(text for bit, text in DEVERR_BITS.items() if bits & bit) or "none"
