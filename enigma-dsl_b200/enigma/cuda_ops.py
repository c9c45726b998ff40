"""torch-tensor front end of the sm_100a operators.

PyTorch only provides device memory and the current stream here; all compute
is in libenigma_cuda.so.  Every function launches asynchronously on the
current torch stream of the tensors' device and returns the output tensor.
Inputs must be contiguous CUDA tensors; there is no CPU path.
"""
from __future__ import annotations

import ctypes
import math
from typing import Optional

from . import _native

_initialised: set = set()


def _torch():
    import torch  # local: the package imports without torch for host-only use

    return torch


def ensure_device(device_index: int) -> None:
    if device_index not in _initialised:
        _native.call("enigma_init", device_index)
        _initialised.add(device_index)


def _stream_ptr(t) -> int:
    torch = _torch()
    return torch.cuda.current_stream(t.device).cuda_stream


def _check_cuda(*ts):
    dev = None
    for t in ts:
        if not t.is_cuda:
            raise ValueError("enigma CUDA operators take CUDA tensors (no CPU fallback)")
        if not t.is_contiguous():
            raise ValueError("enigma CUDA operators take contiguous tensors")
        if dev is None:
            dev = t.device
        elif t.device != dev:
            raise ValueError("all tensors must be on the same device")
    ensure_device(dev.index if dev.index is not None else 0)


def _dtype_code(t) -> int:
    torch = _torch()
    if t.dtype == torch.float32:
        return _native.DTYPE_F32
    if t.dtype == torch.bfloat16:
        return _native.DTYPE_BF16
    raise TypeError(f"unsupported dtype {t.dtype}: expected float32 or bfloat16")


def rmsnorm(x, w, eps: float = 1e-6, out=None):
    """y = x * rsqrt(mean(x^2, -1) + eps) * w over the last axis (fp32 accumulate)."""
    torch = _torch()
    if out is None:
        out = torch.empty_like(x)
    _check_cuda(x, w, out)
    hidden = x.shape[-1]
    if w.numel() != hidden or w.dtype != x.dtype or out.dtype != x.dtype:
        raise ValueError("rmsnorm: w must have hidden elements and x's dtype")
    rows = x.numel() // hidden if hidden else 0
    _native.call("enigma_rmsnorm", _dtype_code(x), x.data_ptr(), w.data_ptr(), out.data_ptr(),
                 rows, hidden, ctypes.c_float(eps), _stream_ptr(x))
    return out


def gemm(a, b, out=None, accumulate: bool = False):
    """C = A @ B for row-major A [M,K], B [K,N]; bf16 (tensor cores) or fp32 (CUDA cores).

    accumulate=True computes C += A @ B and is fp32-only (the reference's gemm_k4).
    """
    torch = _torch()
    if a.dim() != 2 or b.dim() != 2 or a.shape[1] != b.shape[0]:
        raise ValueError(f"gemm: shapes {tuple(a.shape)} x {tuple(b.shape)} do not chain")
    if a.dtype != b.dtype:
        raise TypeError("gemm: A and B must share a dtype")
    m, k = a.shape
    n = b.shape[1]
    if out is None:
        if accumulate:
            raise ValueError("gemm: accumulate=True needs out")
        out = torch.empty((m, n), dtype=a.dtype, device=a.device)
    _check_cuda(a, b, out)
    if a.dtype == torch.bfloat16:
        if accumulate:
            raise TypeError("gemm: accumulate is fp32-only")
        _native.call("enigma_gemm_bf16", a.data_ptr(), b.data_ptr(), out.data_ptr(), m, n, k,
                     _stream_ptr(a))
    elif a.dtype == torch.float32:
        _native.call("enigma_gemm_f32", a.data_ptr(), b.data_ptr(), out.data_ptr(), m, n, k,
                     int(accumulate), _stream_ptr(a))
    else:
        raise TypeError(f"gemm: unsupported dtype {a.dtype}")
    return out


def sdpa(q, k, v, scale: Optional[float] = None, causal: bool = False, out=None):
    """O = softmax(scale * Q K^T [causal]) V for [B, H, S, D] tensors (GQA when Hk < Hq).

    scale defaults to 1/sqrt(D).  causal keeps key j <= i + (Sk - Sq).
    """
    torch = _torch()
    if q.dim() != 4 or k.dim() != 4 or v.dim() != 4:
        raise ValueError("sdpa: expected [B, H, S, D] tensors")
    b, hq, sq, d = q.shape
    bk, hk, sk, dk = k.shape
    if bk != b or dk != d or tuple(v.shape) != tuple(k.shape):
        raise ValueError("sdpa: K/V shapes do not match Q")
    if scale is None:
        scale = 1.0 / math.sqrt(d)
    if out is None:
        out = torch.empty_like(q)
    _check_cuda(q, k, v, out)
    fn = "enigma_sdpa_bf16" if q.dtype == torch.bfloat16 else "enigma_sdpa_f32"
    if q.dtype not in (torch.bfloat16, torch.float32) or k.dtype != q.dtype or v.dtype != q.dtype:
        raise TypeError("sdpa: Q/K/V must all be bf16 or all fp32")
    _native.call(fn, q.data_ptr(), k.data_ptr(), v.data_ptr(), out.data_ptr(), b, hq, hk, sq, sk,
                 d, ctypes.c_float(scale), int(causal), _stream_ptr(q))
    return out


def synchronize(device_index: int = 0) -> None:
    """Synchronize the device and raise if a kernel reported a device-side timeout."""
    ensure_device(device_index)
    _native.call("enigma_synchronize", None)
