"""GPU parity: the sm_100a kernels (through the C ABI) against the CPU oracle.

Tolerances are the ones the build is held to:
  * fp32 RMSNorm: rtol 1e-5 (plus a tiny atol for values near zero)
  * bf16 RMSNorm: within one bf16 ulp of the oracle rounded to bf16
  * bf16 GEMM / SDPA: max-abs <= 2e-2 and ||d||_F / ||ref||_F <= 5e-3 against an
    fp32/fp64 computation on the same bf16-rounded inputs
"""
import numpy as np
import pytest

from oracle import numerics as orc

pytestmark = pytest.mark.gpu


def _t(a, dtype, dev):
    import torch
    return torch.from_numpy(np.ascontiguousarray(a)).to(dev).to(dtype)


def _np(t):
    import torch
    return t.float().cpu().numpy()


# ------------------------------------------------------------------ RMSNorm
@pytest.mark.parametrize("rows,hidden", [(4096, 4096), (3, 4096), (1, 8), (7, 1000), (33, 8192),
                                         (5, 2048), (2, 1024), (9, 256), (4, 16384)])
def test_rmsnorm_f32(cuda, rows, hidden):
    import torch
    from enigma import cuda_ops
    rng = np.random.default_rng(0)
    x = rng.standard_normal((rows, hidden), dtype=np.float32)
    w = (1 + 0.1 * rng.standard_normal(hidden)).astype(np.float32)
    y = cuda_ops.rmsnorm(_t(x, torch.float32, cuda), _t(w, torch.float32, cuda), 1e-6)
    torch.cuda.synchronize()
    ref = orc.rmsnorm(x, w, 1e-6)
    np.testing.assert_allclose(_np(y), ref, rtol=1e-5, atol=1e-6)


@pytest.mark.parametrize("rows,hidden", [(64, 2048), (64, 4096), (64, 8192), (3, 24), (5, 1000)])
def test_rmsnorm_bf16(cuda, rows, hidden):
    import torch
    from enigma import cuda_ops
    rng = np.random.default_rng(1)
    x = orc.bf16_round(rng.standard_normal((rows, hidden), dtype=np.float32))
    w = orc.bf16_round((1 + 0.1 * rng.standard_normal(hidden)).astype(np.float32))
    y = cuda_ops.rmsnorm(_t(x, torch.bfloat16, cuda), _t(w, torch.bfloat16, cuda), 1e-6)
    torch.cuda.synchronize()
    ref = orc.rmsnorm(x, w, 1e-6)
    got = _np(y)
    # one bf16 ulp of the reference value (2^-7 relative at worst) + fp32 slack
    tol = np.abs(ref) * 2.0 ** -7 + 1e-6
    assert np.all(np.abs(got - ref) <= tol), orc.max_abs(got, ref)


def test_rmsnorm_empty(cuda):
    import torch
    from enigma import cuda_ops
    x = torch.empty((0, 64), device=cuda)
    w = torch.ones(64, device=cuda)
    y = cuda_ops.rmsnorm(x, w)
    assert y.shape == (0, 64)


# ------------------------------------------------------------------ GEMM
def _check_bf16(got, ref):
    assert orc.max_abs(got, ref) <= 2e-2, orc.max_abs(got, ref)
    assert orc.rel_fro(got, ref) <= 5e-3, orc.rel_fro(got, ref)


@pytest.mark.parametrize("m,n,k", [(128, 256, 64), (256, 512, 256), (1024, 1024, 1024),
                                   (200, 136, 72), (1, 8, 8), (300, 264, 1000), (128, 256, 8),
                                   (64, 64, 4), (33, 17, 5),
                                   (2560, 2304, 256)])   # 90 tiles on 74 pairs: split tail
def test_gemm_bf16(cuda, m, n, k):
    import torch
    from enigma import cuda_ops
    rng = np.random.default_rng(2)
    a = orc.bf16_round(rng.standard_normal((m, k), dtype=np.float32) / np.sqrt(k))
    b = orc.bf16_round(rng.standard_normal((k, n), dtype=np.float32))
    c = cuda_ops.gemm(_t(a, torch.bfloat16, cuda), _t(b, torch.bfloat16, cuda))
    torch.cuda.synchronize()
    _check_bf16(_np(c), orc.gemm(a, b))


def test_gemm_bf16_4096(cuda):
    import torch
    from enigma import cuda_ops
    n = 4096
    g = torch.Generator(device=cuda).manual_seed(0)
    a = (torch.randn(n, n, device=cuda, generator=g) / n ** 0.5).bfloat16()
    b = torch.randn(n, n, device=cuda, generator=g).bfloat16()
    c = cuda_ops.gemm(a, b)
    rows = torch.arange(0, n, 61, device=cuda)[:64]
    ref = (a[rows].double() @ b.double()).float().cpu().numpy()
    _check_bf16(_np(c[rows]), ref)


@pytest.mark.parametrize("m", [4, 32, 128])
def test_gemm_f32_k4(cuda, m):
    """matmul_k4 / gemm_k4 shapes (tests/metal/test_gemm_matmul_runtime.py:119-175)."""
    import torch
    from enigma import cuda_ops
    rng = np.random.default_rng(3)
    a = rng.standard_normal((m, 4), dtype=np.float32)
    b = rng.standard_normal((4, 64), dtype=np.float32)
    c0 = rng.standard_normal((m, 64), dtype=np.float32)
    c = cuda_ops.gemm(_t(a, torch.float32, cuda), _t(b, torch.float32, cuda))
    np.testing.assert_allclose(_np(c), orc.gemm(a, b), rtol=1e-4, atol=1e-4)
    cc = _t(c0, torch.float32, cuda)
    cuda_ops.gemm(_t(a, torch.float32, cuda), _t(b, torch.float32, cuda), out=cc, accumulate=True)
    np.testing.assert_allclose(_np(cc), orc.gemm(a, b, c0), rtol=1e-4, atol=1e-4)


# ------------------------------------------------------------------ SDPA
@pytest.mark.parametrize("b,hq,hk,sq,sk,d,causal", [
    (1, 2, 2, 128, 128, 128, False), (1, 2, 2, 128, 128, 128, True),
    (2, 4, 2, 256, 256, 64, True), (1, 1, 1, 100, 77, 128, False), (1, 1, 1, 77, 100, 128, True),
    (1, 8, 1, 1, 300, 64, False), (1, 2, 1, 300, 200, 64, True), (1, 2, 2, 2048, 2048, 128, True),
    (1, 2, 2, 2048, 2048, 128, False), (2, 2, 1, 129, 1000, 64, False), (1, 1, 1, 1, 1, 128, True),
    (1, 1, 1, 5, 3, 16, False),
    # more items than SMs (the persistent loop walks several per CTA), including items
    # whose second query tile lies entirely past Sq (Sq = 800), GQA, and Sq < Sk causal
    (2, 64, 8, 800, 800, 128, True), (2, 64, 64, 800, 800, 64, False),
    (1, 160, 160, 300, 1000, 128, True), (4, 48, 16, 1024, 1024, 128, True),
    # causal: items taken from the device-wide work counter (32-head order up to 2048)
    (1, 40, 8, 4096, 4096, 128, True), (1, 64, 64, 4352, 4352, 64, True),
    (3, 40, 8, 2048, 2048, 128, True)])
def test_sdpa_bf16(cuda, b, hq, hk, sq, sk, d, causal):
    import torch
    from enigma import cuda_ops
    rng = np.random.default_rng(4)
    q = orc.bf16_round(rng.standard_normal((b, hq, sq, d), dtype=np.float32))
    k = orc.bf16_round(rng.standard_normal((b, hk, sk, d), dtype=np.float32))
    v = orc.bf16_round(rng.standard_normal((b, hk, sk, d), dtype=np.float32))
    scale = 1.0 / np.sqrt(d)
    o = cuda_ops.sdpa(_t(q, torch.bfloat16, cuda), _t(k, torch.bfloat16, cuda),
                      _t(v, torch.bfloat16, cuda), scale=scale, causal=causal)
    torch.cuda.synchronize()
    _check_bf16(_np(o), orc.sdpa(q, k, v, scale, causal))


@pytest.mark.parametrize("q_scale", [4.0, 8.0])
@pytest.mark.parametrize("causal", [False, True])
def test_sdpa_bf16_peaked(cuda, q_scale, causal):
    """A peaked softmax: Q scaled x4 / x8 puts scores at tens of units, so a few keys
    carry each row and the exponent arguments span a wide range (the kernel's exponent
    path is exercised far from the unit-variance case)."""
    import torch
    from enigma import cuda_ops, _native
    rng = np.random.default_rng(11)
    b, h, s, d = 2, 4, 1024, 128
    q = orc.bf16_round(q_scale * rng.standard_normal((b, h, s, d), dtype=np.float32))
    k = orc.bf16_round(rng.standard_normal((b, h, s, d), dtype=np.float32))
    v = orc.bf16_round(rng.standard_normal((b, h, s, d), dtype=np.float32))
    scale = 1.0 / np.sqrt(d)
    o = cuda_ops.sdpa(_t(q, torch.bfloat16, cuda), _t(k, torch.bfloat16, cuda),
                      _t(v, torch.bfloat16, cuda), scale=scale, causal=causal)
    torch.cuda.synchronize()
    assert _native.last_kernel() == "sdpa_fwd_tc_kernel"
    _check_bf16(_np(o), orc.sdpa(q, k, v, scale, causal))


def test_sdpa_f32_fa_d4(cuda):
    """FlashAttention showcase shape: M = N = 1024, D = 4, scale 1/sqrt(D)
    (examples/showcase_attention.py:22-26, check at :150-153)."""
    import torch
    from enigma import cuda_ops
    rng = np.random.default_rng(1234)
    q = rng.standard_normal((1, 1, 1024, 4), dtype=np.float32)
    k = rng.standard_normal((1, 1, 1024, 4), dtype=np.float32)
    v = rng.standard_normal((1, 1, 1024, 4), dtype=np.float32)
    o = cuda_ops.sdpa(_t(q, torch.float32, cuda), _t(k, torch.float32, cuda),
                      _t(v, torch.float32, cuda), scale=0.5)
    np.testing.assert_allclose(_np(o), orc.sdpa(q, k, v, 0.5), rtol=1e-4, atol=1e-5)


@pytest.mark.parametrize("rows,hidden,chunk,pinned,dtype", [
    (1000, 512, 300, True, "bf16"), (1000, 512, 300, False, "bf16"), (7, 4096, 2, True, "f32"),
    (4096, 4096, 4096, True, "f32"), (65536, 2048, 16384, True, "bf16")])
def test_rmsnorm_host(cuda, rows, hidden, chunk, pinned, dtype):
    """enigma_rmsnorm_host: host x / w in, host y out, chunked with overlapped copies."""
    import ctypes
    import torch
    from enigma import _native
    rng = np.random.default_rng(8)
    x = rng.standard_normal((rows, hidden), dtype=np.float32)
    w = (1 + 0.1 * rng.standard_normal(hidden)).astype(np.float32)
    if dtype == "bf16":
        x, w = orc.bf16_round(x), orc.bf16_round(w)
        tdt, code = torch.bfloat16, _native.DTYPE_BF16
    else:
        tdt, code = torch.float32, _native.DTYPE_F32
    hx = torch.from_numpy(x).to(tdt)
    hw = torch.from_numpy(w).to(tdt)
    hy = torch.empty_like(hx)
    if pinned:
        hx, hw, hy = hx.pin_memory(), hw.pin_memory(), hy.pin_memory()
    lib = _native.lib()
    wsb = ctypes.c_size_t()
    _native.check(lib.enigma_rmsnorm_host_workspace_bytes(code, hidden, chunk, ctypes.byref(wsb)),
                  "ws")
    ws = torch.empty(wsb.value, dtype=torch.uint8, device=cuda)
    _native.check(lib.enigma_rmsnorm_host(code, hx.data_ptr(), hw.data_ptr(), hy.data_ptr(), rows,
                                          hidden, 1e-6, ws.data_ptr(), wsb.value, chunk, None),
                  "rmsnorm_host")
    ref = orc.rmsnorm(x, w, 1e-6)
    got = hy.float().numpy()
    if dtype == "bf16":
        assert np.all(np.abs(got - ref) <= np.abs(ref) * 2.0 ** -8 + 1e-6)
    else:
        np.testing.assert_allclose(got, ref, rtol=1e-5, atol=1e-6)
    with pytest.raises(_native.EnigmaCudaError, match="workspace"):
        _native.check(lib.enigma_rmsnorm_host(code, hx.data_ptr(), hw.data_ptr(), hy.data_ptr(),
                                              rows, hidden, 1e-6, ws.data_ptr(), 16, chunk, None),
                      "rmsnorm_host")
