"""The generic C-ABI entry (enigma_dispatch / enigma_dispatch_timed, the counterparts of
the Swift runtime's enigma_dispatch / enigma_dispatch_timed, libenigma_runtime.swift:132-214)
called through ctypes with exactly the prototypes INTEGRATION.md gives a reference
maintainer, for RMSNorm, GEMM and SDPA, checked against the oracle."""
import ctypes

import numpy as np
import pytest

from oracle import numerics as orc

pytestmark = pytest.mark.gpu

KERNEL_RMSNORM, KERNEL_GEMM, KERNEL_SDPA = 1, 2, 3
DTYPE_F32, DTYPE_BF16 = 0, 1


@pytest.fixture(scope="module")
def lib(cuda):
    from enigma import _native
    lib = ctypes.CDLL(str(_native.library_path()))
    lib.enigma_init.argtypes = [ctypes.c_int32]
    lib.enigma_dispatch.argtypes = [ctypes.c_int32, ctypes.POINTER(ctypes.c_void_p),
                                    ctypes.c_int32, ctypes.POINTER(ctypes.c_int64), ctypes.c_int32,
                                    ctypes.POINTER(ctypes.c_float), ctypes.c_int32,
                                    ctypes.POINTER(ctypes.c_uint32),
                                    ctypes.POINTER(ctypes.c_uint32), ctypes.c_void_p]
    lib.enigma_dispatch_timed.argtypes = lib.enigma_dispatch.argtypes + [
        ctypes.POINTER(ctypes.c_double)]
    lib.enigma_synchronize.argtypes = [ctypes.c_void_p]
    for f in (lib.enigma_init, lib.enigma_dispatch, lib.enigma_dispatch_timed,
              lib.enigma_synchronize):
        f.restype = ctypes.c_int32
    assert lib.enigma_init(0) == 0
    return lib


def _call(lib, kid, tensors, ip, fp, grid=(1, 1, 1), threads=(1, 1, 1), timed=False):
    import torch
    bufs = (ctypes.c_void_p * len(tensors))(*[t.data_ptr() for t in tensors])
    ipa = (ctypes.c_int64 * len(ip))(*ip)
    fpa = (ctypes.c_float * max(1, len(fp)))(*fp)
    g = (ctypes.c_uint32 * 3)(*grid)
    th = (ctypes.c_uint32 * 3)(*threads)
    s = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    if timed:
        us = ctypes.c_double()
        rc = lib.enigma_dispatch_timed(kid, bufs, len(tensors), ipa, len(ip), fpa, len(fp), g, th,
                                       s, ctypes.byref(us))
        return rc, us.value
    rc = lib.enigma_dispatch(kid, bufs, len(tensors), ipa, len(ip), fpa, len(fp), g, th, s)
    return rc, lib.enigma_synchronize(s)


@pytest.mark.parametrize("timed", [False, True])
def test_dispatch_rmsnorm(lib, timed):
    import torch
    rng = np.random.default_rng(0)
    x = rng.standard_normal((512, 4096), dtype=np.float32)
    w = (1 + 0.1 * rng.standard_normal(4096)).astype(np.float32)
    tx, tw = torch.from_numpy(x).cuda(), torch.from_numpy(w).cuda()
    ty = torch.empty_like(tx)
    rc, extra = _call(lib, KERNEL_RMSNORM, [tx, tw, ty], [512, 4096, DTYPE_F32], [1e-6],
                      grid=(512 * 256, 1, 1), threads=(256, 1, 1), timed=timed)
    assert rc == 0 and (extra > 0 if timed else extra == 0)
    np.testing.assert_allclose(ty.cpu().numpy(), orc.rmsnorm(x, w, 1e-6), rtol=1e-5, atol=1e-6)


@pytest.mark.parametrize("timed", [False, True])
def test_dispatch_gemm_bf16(lib, timed):
    import torch
    rng = np.random.default_rng(1)
    m = n = k = 1024
    a = orc.bf16_round(rng.standard_normal((m, k), dtype=np.float32) / np.sqrt(k))
    b = orc.bf16_round(rng.standard_normal((k, n), dtype=np.float32))
    ta, tb = torch.from_numpy(a).cuda().bfloat16(), torch.from_numpy(b).cuda().bfloat16()
    tc = torch.empty(m, n, device="cuda", dtype=torch.bfloat16)
    rc, extra = _call(lib, KERNEL_GEMM, [ta, tb, tc], [m, n, k, DTYPE_BF16, 0], [], timed=timed)
    assert rc == 0
    got, ref = tc.float().cpu().numpy(), orc.gemm(a, b)
    assert orc.max_abs(got, ref) <= 2e-2 and orc.rel_fro(got, ref) <= 5e-3


@pytest.mark.parametrize("timed", [False, True])
@pytest.mark.parametrize("causal", [0, 1])
def test_dispatch_sdpa_bf16(lib, timed, causal):
    import torch
    rng = np.random.default_rng(2)
    B, H, S, D = 1, 4, 512, 128
    q, k, v = (orc.bf16_round(rng.standard_normal((B, H, S, D), dtype=np.float32))
               for _ in range(3))
    tq, tk, tv = (torch.from_numpy(a).cuda().bfloat16() for a in (q, k, v))
    to = torch.empty_like(tq)
    rc, extra = _call(lib, KERNEL_SDPA, [tq, tk, tv, to], [B, H, H, S, S, D, causal, DTYPE_BF16],
                      [D ** -0.5], timed=timed)
    assert rc == 0
    got, ref = to.float().cpu().numpy(), orc.sdpa(q, k, v, D ** -0.5, bool(causal))
    assert orc.max_abs(got, ref) <= 2e-2 and orc.rel_fro(got, ref) <= 5e-3


def test_dispatch_rejects_bad_launch_shape(lib):
    import torch
    t = torch.zeros(16, device="cuda")
    rc, _ = _call(lib, KERNEL_RMSNORM, [t, t, t], [1, 16, DTYPE_F32], [1e-6], grid=(0, 1, 1))
    assert rc == -4
    rc, _ = _call(lib, KERNEL_RMSNORM, [t, t, t], [1, 16, DTYPE_F32], [1e-6],
                  threads=(64, 32, 1))
    assert rc == -4
    rc, _ = _call(lib, 99, [t], [], [])
    assert rc == -4
