"""Loads libtbf16_sm100.so (the C-ABI library of the sm_100a kernels) through ctypes.

Replaces the reference's JIT torch-extension loader (tbf16/_ext.py:1-107 of the reference). There
is no fallback: if the library cannot be built or loaded, or the GPU is not sm_100, every op raises.
The library is built ahead of time (turing-bf16_b200/build.py, also run by __graft_entry__.build());
when it is missing or older than its sources, the first call builds it with nvcc.
"""
import ctypes
import importlib.util
import os
import pathlib
import threading

import torch

_HERE = pathlib.Path(__file__).resolve().parent
LIB_PATH = _HERE / "lib" / "libtbf16_sm100.so"
_lib = None
_lock = threading.Lock()
_failed = None

_vp, _i64, _i32, _u32 = ctypes.c_void_p, ctypes.c_int64, ctypes.c_int, ctypes.c_uint

# name -> argtypes; every entry point returns an int status. Mirrors include/tbf16_sm100.h.
SIGNATURES = {
    "tbf16_row_scale": [_vp, _i64, _i64, _i64, _i32, _i32, _vp, _vp, _vp, _i64, _vp],
    "tbf16_quantize_rows": [_vp, _i64, _i64, _i64, _i32, _i32, _vp, _i64, _vp, _vp],
    "tbf16_quantize_cols": [_vp, _i64, _i64, _i64, _i32, _vp, _vp, _i64, _vp, _vp, _vp],
    "tbf16_quantize_cols_noalloc": [_vp, _i64, _i64, _i64, _i32, _vp, _vp, _i64, _vp, _vp],
    "tbf16_head_amax": [_vp, _i32, _i64, _i64, _i64, _i64, _i64, _i64, _i64, _vp, _vp],
    "tbf16_head_exp": [_vp, _i32, _i64, _i64, _i64, _i64, _i64, _i64, _i64, _vp, _vp, _vp],
    "tbf16_head_scale_cast": [_vp, _i32, _i64, _i64, _i64, _i64, _i64, _i64, _i64, _vp, _i64, _i64, _vp, _i32, _vp],
    "tbf16_prepare_qkv": [_vp, _i64, _i64, _i64, _vp, _i64, _i64, _i64, _vp, _i64, _i64, _i64, _i64, _i64, _i64, _i64,
                          _i64, _i64, _i32, _vp, _vp, _vp, _vp, _vp, _vp, _vp],
    "tbf16_qkv_local_exponents": [_vp, _i64, _i64, _i64, _vp, _i64, _i64, _i64, _vp, _i64, _i64, _i64, _i64, _i64,
                                  _i64, _i64, _i64, _i64, _vp, _vp, _vp],
    "tbf16_prepare_qkv_global": [_vp, _i64, _i64, _i64, _vp, _i64, _i64, _i64, _vp, _i64, _i64, _i64, _i64, _i64, _i64,
                                 _i64, _i64, _i64, _i32, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp],
    "tbf16_linear": [_vp, _i64, _i64, _i64, _vp, _i64, _i64, _vp, _vp, _vp, _i64, _vp, _vp, _i32, _i32, _vp],
    "tbf16_linear_scaled": [_vp, _i64, _i64, _i64, _vp, _i64, _i64, _vp, _vp, _vp, _i64, _vp, _vp],
    "tbf16_gemm_f16": [_vp, _i32, _i64, _vp, _i32, _i64, _i64, _i64, _i64, _vp, _vp, _vp, _vp, _i64, _vp],
    "tbf16_gemv": [_vp, _i64, _i64, _i64, _vp, _i64, _i64, _vp, _vp, _vp, _i64, _vp],
    "tbf16_glu_rows": [_vp, _i64, _vp, _i64, _i64, _i64, _i32, _i32, _vp, _i64, _vp, _vp, _i64, _vp],
    "tbf16_add_rmsnorm_rows": [_vp, _i64, _vp, _i64, _vp, _vp, _i64, _i64, ctypes.c_float, _i32, ctypes.c_float, _i32,
                               _vp, _i64, _vp, _i64, _vp, _vp, _i64, _vp],
    "tbf16_glu_bwd": [_vp, _i64, _vp, _i64, _vp, _i64, _i64, _i64, _i32, _vp, _i64, _vp, _i64, _vp],
    "tbf16_rmsnorm_rope": [_vp, _i64, _vp, _i64, _i64, ctypes.c_float, _i32, ctypes.c_float, _vp, _vp, _i64, _i64,
                           _i64, _vp, _i64, _vp],
    "tbf16_rmsnorm_rows": [_vp, _i64, _vp, _i64, _i64, ctypes.c_float, _i32, ctypes.c_float, _i32, _vp, _i64, _vp, _vp,
                           _i64, _vp],
    "tbf16_conv_sample_scale": [_vp, _i64, _i64, _i64, _i32, _vp, _vp, _vp, _vp],
    "tbf16_conv_im2col": [_vp, _vp, _i64, _i64, _vp, _vp, _vp, _vp, _vp],
    "tbf16_conv_im2col_cl": [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp],
    "tbf16_conv_grouped": [_vp, _vp, _i64, _i64, _vp, _vp, _vp, _vp, _vp, _vp, _vp],
    "tbf16_conv_implicit_supported": [_vp, _i64],
    "tbf16_conv_implicit": [_vp, _vp, _i32, _vp, _vp, _vp, _vp, _vp, _i64, _vp, _vp, _vp, _vp],
    "tbf16_attn_fwd": [_vp, _vp, _vp, _i64, _i64, _i64, _i64, _i64, _i64, ctypes.c_float, _i32, _vp, _vp, _i64, _i64,
                       _i64, _vp, _vp, _i64, _vp, _vp],
    "tbf16_attn_fwd_out": [_vp, _vp, _vp, _i64, _i64, _i64, _i64, _i64, _i64, ctypes.c_float, _i32, _vp, _vp, _i64,
                           _i64, _i64, _vp, _i64, _i64, _i64, _vp, _i64, _vp, _vp],
    "tbf16_attn_bwd": [_vp, _vp, _vp, _vp, _vp, _i64, _vp, _i64, _i64, _i64, _i64, _vp, _vp, _i64, _i64, _i64, _i64, _i64,
                       _i64,
                       ctypes.c_float, _i32, _vp, _i64, _i64, _i64, _i32, _vp, _vp, _vp, _vp, _vp, _vp, _i64, _vp],
    "tbf16_attn_fwd_dropout": [_vp, _vp, _vp, _i64, _i64, _i64, _i64, _i64, _i64, ctypes.c_float, _i32, _vp, _vp, _i64,
                               _i64, _i64, _vp, _i64, _i64, _i64, _vp, _i64, _vp, ctypes.c_float, ctypes.c_uint64, _vp],
    "tbf16_attn_bwd_dropout": [_vp, _vp, _vp, _vp, _vp, _i64, _vp, _i64, _i64, _i64, _i64, _vp, _vp, _i64, _i64, _i64,
                               _i64, _i64, _i64, ctypes.c_float, _i32, _vp, _i64, _i64, _i64, _i32, _vp, _vp, _vp, _vp,
                               _vp, _vp, _i64, ctypes.c_float, ctypes.c_uint64, _vp],
    "tbf16_attn_dropout_keep": [_vp, _i64, _i64, _i64, ctypes.c_float, ctypes.c_uint64, _vp],
    "tbf16_attn_fwd_ws": [_vp, _vp, _vp, _i64, _i64, _i64, _i64, _i64, _i64, ctypes.c_float, _i32, _vp, _vp, _i64,
                          _i64, _i64, _vp, _i64, _i64, _i64, _vp, _i64, _vp, ctypes.c_float, ctypes.c_uint64, _vp,
                          _i64, _vp],
    "tbf16_attn_bwd_sharded": [_vp, _vp, _vp, _vp, _vp, _i64, _vp, _i64, _i64, _i64, _i64, _vp, _vp, _i64, _i64, _i64,
                               _i64, _i64, _i64, ctypes.c_float, _i32, _vp, _i64, _i64, _i64, _i32, _vp, _vp, _vp, _vp,
                               _vp, _vp, _i64, ctypes.c_float, ctypes.c_uint64, _vp, _vp],
    "tbf16_device_check": [_i32],
    "tbf16_device_status": [_vp, _i32],
    "tbf16_selftest_bounded_wait": [ctypes.c_uint64, _vp],
}

# entry points returning a size (int64) rather than a status
SIGNATURES_I64 = {
    "tbf16_attn_bwd_workspace_size": [_i64, _i64, _i64, _i64, _i64, _i64],
    "tbf16_attn_fwd_ws_size": [_i64, _i64, _i64, _i64, _i64, _i64, _i32],
}

BF16, F16 = 0, 1
STATUS = {1: "invalid argument", 2: "misaligned pointer or leading dimension", 3: "unsupported dtype",
          4: "CUDA launch error", 5: "not an sm_100 (B200) GPU", 6: "unsupported by this build",
          7: "kernel timed out on a bounded wait"}


def _build_module():
    spec = importlib.util.spec_from_file_location("_tbf16_build", _HERE.parent / "build.py")
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def build(force=False):
    """Compile the library (nvcc, sm_100a) if it is missing or stale."""
    return _build_module().build(force=force)


def lib():
    """The loaded library; builds it first if needed. Raises RuntimeError if that fails."""
    global _lib, _failed
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is not None:
            return _lib
        if not os.environ.get("TBF16_NO_BUILD"):
            try:
                if _build_module().stale():
                    build()
            except Exception as e:  # a missing toolkit is fine if the library is already there
                if not LIB_PATH.exists():
                    _failed = e
                    raise RuntimeError(f"tbf16: cannot build {LIB_PATH.name}: {e}") from e
        if not LIB_PATH.exists():
            raise RuntimeError(f"tbf16: {LIB_PATH} is missing; run turing-bf16_b200/build.py")
        L = ctypes.CDLL(str(LIB_PATH))
        for name, args in SIGNATURES.items():
            fn = getattr(L, name)
            fn.argtypes = args
            fn.restype = ctypes.c_int
        for name, args in SIGNATURES_I64.items():
            fn = getattr(L, name)
            fn.argtypes = args
            fn.restype = ctypes.c_int64
        L.tbf16_status_string.argtypes = [_i32]
        L.tbf16_status_string.restype = ctypes.c_char_p
        L.tbf16_abi_version.argtypes = []
        L.tbf16_abi_version.restype = ctypes.c_int
        _lib = L
    return _lib


def available() -> bool:
    """True if the library loads (it is always required: there is no fallback path)."""
    try:
        lib()
        return True
    except Exception:
        return False


def check(status: int, what: str):
    if status != 0:
        text = lib().tbf16_status_string(status).decode()
        raise RuntimeError(f"tbf16: {what} failed: {text} (status {status})")


def call(name: str, *args):
    check(getattr(lib(), name)(*args), name)


def stream_ptr(device=None):
    return ctypes.c_void_p(torch.cuda.current_stream(device).cuda_stream)


def ptr(t):
    return ctypes.c_void_p(0 if t is None else t.data_ptr())


def require_cuda(*ts):
    for t in ts:
        if t is not None and not t.is_cuda:
            raise RuntimeError("tbf16: expected CUDA tensors (there is no CPU path)")


def device_status(reset: bool = True) -> int:
    """Error bits the kernels recorded on the current device (synchronises)."""
    bits = ctypes.c_uint(0)
    check(lib().tbf16_device_status(ctypes.byref(bits), int(reset)), "tbf16_device_status")
    return bits.value


# kept for callers of the reference's loader (tbf16/_ext.py:61-107 there)
def ext():
    return lib()


def gemm_ext():
    return lib()


def gemm_available() -> bool:
    return available()
