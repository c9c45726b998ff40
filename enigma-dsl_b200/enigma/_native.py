"""ctypes binding of libenigma_cuda.so (include/enigma_cuda.h).

This is the analogue of the reference's ctypes binding of its Swift runtime
(enigma/runtime_dispatch/runtime.py:242-316): one shared library, prototypes
declared once, every call's int32 status turned into a Python exception.
There is no fallback: if the library is missing or cannot load, every
operator raises.
"""
from __future__ import annotations

import ctypes
import os
from pathlib import Path
from typing import Optional

_LIB_PATH = Path(__file__).resolve().parent / "_lib" / "libenigma_cuda.so"

OK, ERR_LAUNCH, ERR_EXEC, ERR_TIMEOUT, ERR_BADARG, ERR_DEVICE = 0, -1, -2, -3, -4, -5
DTYPE_F32, DTYPE_BF16 = 0, 1
KERNEL_RMSNORM, KERNEL_GEMM, KERNEL_SDPA = 1, 2, 3

_STATUS_NAMES = {
    ERR_LAUNCH: "launch failed",
    ERR_EXEC: "GPU execution error",
    ERR_TIMEOUT: "device-side wait timed out",
    ERR_BADARG: "bad argument",
    ERR_DEVICE: "no usable sm_100 device",
}

# Every exported symbol with its (restype, argtypes).  Kept in the order of
# include/enigma_cuda.h; tests check the two lists agree.
_c = ctypes
_vp, _i32, _i64, _sz, _f32 = _c.c_void_p, _c.c_int32, _c.c_int64, _c.c_size_t, _c.c_float
_u32p = _c.POINTER(_c.c_uint32)
PROTOTYPES = {
    "enigma_init": [_i32],
    "enigma_device_count": [_c.POINTER(_i32)],
    "enigma_stream_create": [_c.POINTER(_vp)],
    "enigma_stream_destroy": [_vp],
    "enigma_synchronize": [_vp],
    "enigma_last_error": [_c.c_char_p, _sz],
    "enigma_last_kernel": [_c.c_char_p, _sz],
    "enigma_device_name": [_i32, _c.c_char_p, _sz],
    "enigma_device_attrs": [_i32, _c.POINTER(_i64), _c.POINTER(_i64), _c.POINTER(_i64),
                            _c.POINTER(_i64), _c.POINTER(_i32), _c.POINTER(_i32)],
    "enigma_alloc": [_c.POINTER(_vp), _sz],
    "enigma_free": [_vp],
    "enigma_host_alloc": [_c.POINTER(_vp), _sz],
    "enigma_host_free": [_vp],
    "enigma_upload": [_vp, _vp, _sz, _vp],
    "enigma_download": [_vp, _vp, _sz, _vp],
    "enigma_memset": [_vp, _i32, _sz, _vp],
    "enigma_rmsnorm": [_i32, _vp, _vp, _vp, _i64, _i64, _f32, _vp],
    "enigma_gemm_bf16": [_vp, _vp, _vp, _i64, _i64, _i64, _vp],
    "enigma_sdpa_bf16": [_vp, _vp, _vp, _vp, _i64, _i64, _i64, _i64, _i64, _i64, _f32, _i32, _vp],
    "enigma_elementwise": [_i32, _i32, _vp, _vp, _vp, _i64, _vp],
    "enigma_gemm_f32": [_vp, _vp, _vp, _i64, _i64, _i64, _i32, _vp],
    "enigma_gemm_f32_trans": [_vp, _vp, _vp, _i64, _i64, _i64, _i32, _i32, _i32, _vp],
    "enigma_sdpa_f32": [_vp, _vp, _vp, _vp, _i64, _i64, _i64, _i64, _i64, _i64, _f32, _i32, _vp],
    "enigma_sdpa_strided": [_i32, _vp, _vp, _vp, _vp, _i64, _i64, _i64, _i64, _i64, _i64,
                            _c.POINTER(_i64), _f32, _i32, _vp],
    "enigma_sdpa_strided_sinks": [_i32, _vp, _vp, _vp, _vp, _i64, _i64, _i64, _i64, _i64,
                                  _i64, _c.POINTER(_i64), _f32, _i32, _vp, _vp],
    "enigma_rmsnorm_host_workspace_bytes": [_i32, _i64, _i64, _c.POINTER(_sz)],
    "enigma_rmsnorm_host": [_i32, _vp, _vp, _vp, _i64, _i64, _f32, _vp, _sz, _i64, _vp],
    "enigma_decode_workspace_bytes": [_vp, _c.POINTER(_sz)],
    "enigma_decode_layer_bf16": [_vp, _vp, _vp, _vp, _sz, _vp],
    "enigma_qwen_decode_f32": [_vp, _vp],
    "enigma_decode_layer_bf16_noalloc": [_vp, _vp, _vp, _vp],
    "enigma_decode_noalloc_check_timeout_path": [_i64, _vp],
    "enigma_dispatch": [_i32, _c.POINTER(_vp), _i32, _c.POINTER(_i64), _i32, _c.POINTER(_f32),
                        _i32, _u32p, _u32p, _vp],
    "enigma_dispatch_timed": [_i32, _c.POINTER(_vp), _i32, _c.POINTER(_i64), _i32,
                              _c.POINTER(_f32), _i32, _u32p, _u32p, _vp,
                              _c.POINTER(_c.c_double)],
    "enigma_event_create": [_c.POINTER(_vp)],
    "enigma_event_destroy": [_vp],
    "enigma_event_record": [_vp, _vp],
    "enigma_event_elapsed_ms": [_vp, _vp, _c.POINTER(_f32)],
    "enigma_take_device_status": [_c.POINTER(_i32)],
    "enigma_check_timeout_path": [_i64, _vp],
}


class EnigmaCudaError(RuntimeError):
    """A libenigma_cuda call returned a non-zero status."""

    def __init__(self, status: int, func: str, message: str):
        self.status = status
        self.func = func
        super().__init__(f"enigma GPU error: {func} -> {status} "
                         f"({_STATUS_NAMES.get(status, 'unknown')}): {message}")


_lib: Optional[ctypes.CDLL] = None


def library_path() -> Path:
    return Path(os.environ.get("ENIGMA_CUDA_LIB", str(_LIB_PATH)))


def lib() -> ctypes.CDLL:
    """Load (once) and return the native library; raises if it is not built."""
    global _lib
    if _lib is None:
        path = library_path()
        if not path.exists():
            raise RuntimeError(
                f"libenigma_cuda.so not found at {path}; build it with "
                f"`python enigma-dsl_b200/build.py` (there is no CPU fallback)")
        handle = ctypes.CDLL(str(path))
        for name, argtypes in PROTOTYPES.items():
            fn = getattr(handle, name)
            fn.argtypes = argtypes
            fn.restype = _i32
        _lib = handle
    return _lib


def last_error() -> str:
    buf = ctypes.create_string_buffer(512)
    lib().enigma_last_error(buf, 512)
    return buf.value.decode(errors="replace")


def last_kernel() -> str:
    """The device kernel the last operator call on this thread launched."""
    buf = ctypes.create_string_buffer(128)
    lib().enigma_last_kernel(buf, 128)
    return buf.value.decode()


def check(status: int, func: str) -> None:
    if status != OK:
        raise EnigmaCudaError(status, func, last_error())


def call(name: str, *args) -> None:
    check(getattr(lib(), name)(*args), name)
