"""End to end through the reference-facing API on the GPU:
enigma.compile -> MetalRuntime.execute / prepare -> sm_100a kernel, checked
against the CPU oracle with the same tolerances as the example scripts
(benchmark_rmsnorm.py:127-136, benchmark_sdpa.py:220-232,
showcase_attention.py:159-170, test_gemm_matmul_runtime.py:136,166) or tighter."""
import numpy as np
import pytest

import enigma
import dsl_kernels as K
from oracle import numerics as orc

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def rt(cuda):
    return enigma.MetalRuntime()


def test_rmsnorm_config1(rt):
    rows = n = 4096
    jit, args = K.make_rmsnorm(rows, n, 256, 4, 1e-6)
    ck = enigma.compile(jit, *args)
    rng = np.random.default_rng(0)
    x = rng.standard_normal((rows, n), dtype=np.float32)
    w = (1 + 0.1 * rng.standard_normal(n)).astype(np.float32)
    raw = rt.execute(ck, [x.ravel(), w], rows * n * 4, grid=ck.grid, threads=ck.block)
    y = np.frombuffer(raw, np.float32).reshape(rows, n)
    np.testing.assert_allclose(y, orc.rmsnorm(x, w, 1e-6), rtol=1e-5, atol=1e-6)


def test_rmsnorm_prepare_timed(rt):
    jit, args = K.make_rmsnorm(512, 4096, 256, 16, 1e-5)
    ck = enigma.compile(jit, *args)
    rng = np.random.default_rng(42)
    x = rng.standard_normal((512, 4096), dtype=np.float32)
    w = rng.standard_normal(4096).astype(np.float32)
    prep = rt.prepare(ck, [x.ravel(), w], 512 * 4096 * 4)
    try:
        for _ in range(3):
            prep.dispatch(ck.grid, ck.block)
        us = prep.dispatch_timed(ck.grid, ck.block)
        assert 0 < us < 1e5
        r = enigma.benchmark.bench_gpu(prep, ck.grid, ck.block, repeat=5, warmup=1)
        assert r.median_us > 0
        y = np.frombuffer(prep.read_output(), np.float32).reshape(512, 4096)
        np.testing.assert_allclose(y, orc.rmsnorm(x, w, 1e-5), rtol=1e-5, atol=1e-6)
    finally:
        prep.release()


def test_sdpa_gqa_reference_shape(rt):
    """benchmark_sdpa.py shape: 128 tokens, 64 q heads / 8 kv heads, d 64, 512 kv tokens,
    interleaved KV, no scale, running max buffer = -1e30."""
    T, H, G, D, S = 128, 64, 8, 64, 512
    jit, args, thr = K.make_sdpa_gqa(T, H, G, D, S)
    ck = enigma.compile(jit, *args)
    rng = np.random.default_rng(42)
    q = (rng.standard_normal((T, H, D)) * 0.1).astype(np.float32)
    k = (rng.standard_normal((G, S, D)) * 0.1).astype(np.float32)
    v = (rng.standard_normal((G, S, D)) * 0.1).astype(np.float32)
    kv = np.concatenate([k, v], axis=2)
    m0 = np.full(H, -1e30, np.float32)
    raw = rt.execute(ck, [q.ravel(), kv.ravel(), m0], T * H * D * 4, grid=ck.grid,
                     threads=ck.block)
    o = np.frombuffer(raw, np.float32).reshape(T, H, D)
    ref = orc.sdpa(q.transpose(1, 0, 2)[None], k[None], v[None], 1.0)[0].transpose(1, 0, 2)
    np.testing.assert_allclose(o, ref, rtol=1e-4, atol=1e-5)


def test_fa_d4(rt):
    ck = enigma.compile(K.make_fa(1024))
    rng = np.random.default_rng(1234)
    q, k, v = (rng.standard_normal((1024, 4)).astype(np.float32) for _ in range(3))
    raw = rt.execute(ck, [q.ravel(), k.ravel(), v.ravel()], 1024 * 4 * 4, grid=(1024, 1, 1),
                     threads=(32, 1, 1))
    o = np.frombuffer(raw, np.float32).reshape(1024, 4)
    np.testing.assert_allclose(o, orc.sdpa(q[None, None], k[None, None], v[None, None], 0.5)[0, 0],
                               rtol=1e-4, atol=1e-5)


@pytest.mark.parametrize("acc", [False, True])
@pytest.mark.parametrize("m", [4, 32, 128])
def test_k4(rt, m, acc):
    ck = enigma.compile(K.make_k4(64, acc))
    rng = np.random.default_rng(m)
    a = rng.standard_normal((m, 4)).astype(np.float32)
    b = rng.standard_normal((4, 64)).astype(np.float32)
    raw = rt.execute(ck, [a.ravel(), b.ravel()], m * 64 * 4, grid=(64, m, 1),
                     threads=(16, min(m, 16), 1))
    np.testing.assert_allclose(np.frombuffer(raw, np.float32).reshape(m, 64), a @ b,
                               rtol=1e-4, atol=1e-4)


def test_async_gemm(rt):
    ck = enigma.compile(K.make_async_gemm(64, 64, 64))
    rng = np.random.default_rng(0)
    a = (rng.standard_normal((64, 64)) * 0.1).astype(np.float32)
    b = (rng.standard_normal((64, 64)) * 0.1).astype(np.float32)
    raw = rt.execute(ck, [a.ravel(), b.ravel()], 64 * 64 * 4, grid=(4, 1, 1), threads=(128, 1, 1))
    np.testing.assert_allclose(np.frombuffer(raw, np.float32).reshape(64, 64), a @ b,
                               rtol=1e-4, atol=1e-5)


def test_torch_zero_copy_and_torch_outputs(rt):
    import torch
    jit, args = K.make_rmsnorm(64, 2048, 256, 8, 1e-6, dtype="bfloat")
    ck = enigma.compile(jit, *args)
    x = torch.randn(64, 2048, device="cuda").bfloat16()
    w = torch.ones(2048, device="cuda").bfloat16()
    y = rt.execute(ck, [x, w], None, grid=ck.grid, threads=ck.block,
                   output_shapes=[(64, 2048)], output_dtypes=[torch.bfloat16])
    ref = orc.rmsnorm(x.float().cpu().numpy(), w.float().cpu().numpy(), 1e-6)
    got = y.float().cpu().numpy()
    assert np.all(np.abs(got - ref) <= np.abs(ref) * 2.0 ** -7 + 1e-6)


def test_bind_count_error(rt):
    ck = enigma.compile(K.make_k4(64, False))
    with pytest.raises(RuntimeError, match="Outputs are appended AFTER inputs"):
        rt.execute(ck, [np.zeros(16, np.float32)], 64, grid=(1, 1, 1), threads=(1, 1, 1))


def test_device_capabilities(rt):
    caps = rt.device_capabilities()
    assert caps.gpu_family == "sm_100" and caps.sm_count >= 100 and caps.simdgroup_size == 32


@pytest.mark.parametrize("H,INTER,QH,KVH,CT", [(1024, 3072, 16, 8, 33), (256, 512, 4, 2, 9)])
def test_qwen_fused_reference_shape(rt, H, INTER, QH, KVH, CT):
    """examples/qwen_megakernel.py: fp32, one token, caches pre-filled; its bar is 1e-3."""
    HD = H // QH
    ck = enigma.compile(K.make_qwen(H, INTER, QH, KVH, CT))
    rng = np.random.default_rng(0)
    f32 = lambda a: np.asarray(a, np.float32)  # noqa: E731
    x = f32(rng.standard_normal(H) * 0.1)
    w_in, w_post = f32(rng.standard_normal(H) * 0.1 + 1), f32(rng.standard_normal(H) * 0.1 + 1)
    wqn, wkn = f32(rng.standard_normal(HD) * 0.1 + 1), f32(rng.standard_normal(HD) * 0.1 + 1)
    Wq = f32(rng.standard_normal((QH * HD, H)) / np.sqrt(H))
    Wk = f32(rng.standard_normal((KVH * HD, H)) / np.sqrt(H))
    Wv = f32(rng.standard_normal((KVH * HD, H)) / np.sqrt(H))
    Wo = f32(rng.standard_normal((H, QH * HD)) / np.sqrt(QH * HD))
    Wg = f32(rng.standard_normal((INTER, H)) / np.sqrt(H))
    Wu = f32(rng.standard_normal((INTER, H)) / np.sqrt(H))
    Wd = f32(rng.standard_normal((H, INTER)) / np.sqrt(INTER))
    ang = np.arange(HD, dtype=np.float32) / HD * (np.pi / 2)
    cs, sn = f32(np.cos(ang)), f32(np.sin(ang))
    kc = f32(rng.standard_normal((KVH, CT, HD)) * 0.1)
    vc = f32(rng.standard_normal((KVH, CT, HD)) * 0.1)
    z = lambda n: np.zeros(n, np.float32)  # noqa: E731
    ins = [x, w_in, Wq.ravel(), Wk.ravel(), Wv.ravel(), wqn, wkn, cs, sn, kc.ravel(), vc.ravel(),
           Wo.ravel(), w_post, Wg.ravel(), Wu.ravel(), Wd.ravel(), z(H), z(QH * HD), z(KVH * HD),
           z(KVH * HD), z(QH * HD), z(INTER), z(H), z(QH * HD), z(KVH * HD)]
    raw = rt.execute(ck, ins, H * 4, grid=(256, 1, 1), threads=(256, 1, 1))
    out = np.frombuffer(raw, np.float32)
    ref = orc.qwen_decode_f32(x, w_in, Wq, Wk, Wv, wqn, wkn, cs, sn, kc, vc, Wo, w_post, Wg, Wu,
                              Wd, QH, KVH, 1e-6)
    assert np.max(np.abs(out - ref)) < 1e-4, np.max(np.abs(out - ref))


def test_tv_add_reference_shape(rt):
    """examples/vector_add_tv.py: 256 x 512 fp32, rtol 1e-5."""
    jit, args = K.make_tv_add(256, 512)
    ck = enigma.compile(jit, *args)
    rng = np.random.default_rng(0)
    a, b = (rng.standard_normal((256, 512)).astype(np.float32) for _ in range(2))
    raw = rt.execute(ck, [a.ravel(), b.ravel()], a.nbytes, grid=ck.grid, threads=ck.block)
    np.testing.assert_allclose(np.frombuffer(raw, np.float32).reshape(256, 512), a + b,
                               rtol=1e-5, atol=1e-7)


@pytest.mark.parametrize("n", [4, 256, 1024, 65536, 1001])
def test_naive_add(rt, n):
    """tests/metal/test_vector_add_runtime.py sizes, rtol 1e-5 (1001: ragged tail)."""
    ck = enigma.compile(K.make_naive_binary(lambda a, b: a + b))
    rng = np.random.default_rng(n)
    a, b = (rng.standard_normal(n).astype(np.float32) for _ in range(2))
    raw = rt.execute(ck, [a, b], a.nbytes, grid=(n, 1, 1), threads=(min(n, 256), 1, 1))
    np.testing.assert_allclose(np.frombuffer(raw, np.float32), a + b, rtol=1e-5)


@pytest.mark.parametrize("mode", ["scalar", "constant"])
def test_rmsnorm_runtime_eps(rt, mode):
    """eps as a Scalar parameter (runtime.py:125-175) or a function constant (:358-364)."""
    ck = enigma.compile(K.make_rmsnorm_runtime_eps(1024, mode))
    rng = np.random.default_rng(5)
    x = rng.standard_normal((64, 1024)).astype(np.float32)
    w = (1 + 0.1 * rng.standard_normal(1024)).astype(np.float32)
    kw = {"scalars": [1e-2]} if mode == "scalar" else {"constants": {0: ("float", 1e-2)}}
    raw = rt.execute(ck, [x.ravel(), w], x.nbytes, grid=(64 * 256, 1, 1), threads=(256, 1, 1),
                     **kw)
    np.testing.assert_allclose(np.frombuffer(raw, np.float32).reshape(64, 1024),
                               orc.rmsnorm(x, w, 1e-2), rtol=1e-5, atol=1e-6)


@pytest.mark.parametrize("sink", ["none", "finite"])
def test_sdpa_gqa_sinks(rt, sink):
    """The DSL gpt-oss kernel's buffer 2 is an attention sink (benchmark_sdpa.py:64-72): with
    finite values it joins the softmax denominator."""
    T, H, G, D, S = 16, 64, 8, 64, 100
    jit, args, thr = K.make_sdpa_gqa(T, H, G, D, S)
    ck = enigma.compile(jit, *args)
    rng = np.random.default_rng(7)
    q = rng.standard_normal((T, H, D)).astype(np.float32) * 0.3
    k = rng.standard_normal((G, S, D)).astype(np.float32) * 0.3
    v = rng.standard_normal((G, S, D)).astype(np.float32)
    kv = np.concatenate([k, v], axis=2)
    s0 = (np.full(H, -1e30) if sink == "none" else rng.standard_normal(H) * 2).astype(np.float32)
    raw = rt.execute(ck, [q.ravel(), kv.ravel(), s0], T * H * D * 4, grid=ck.grid,
                     threads=ck.block)
    o = np.frombuffer(raw, np.float32).reshape(T, H, D)
    ref = orc.sdpa(q.transpose(1, 0, 2)[None], k[None], v[None], 1.0,
                   sinks=None if sink == "none" else s0)[0].transpose(1, 0, 2)
    np.testing.assert_allclose(o, ref, rtol=1e-4, atol=1e-5)


# ------------------------------------------------------------------ DSL -> tensor-core kernels
# The reference's FA and async-copy GEMM kernels written at BASELINE's bf16 shapes
# (config 3 GEMM, config 4 SDPA), compiled by enigma.compile and run by
# MetalRuntime.execute on torch device buffers; enigma_last_kernel names the sm_100a
# kernel the dispatch reached.  Bars: max-abs 2e-2, relative Frobenius 5e-3.
def _check_bf16(got, ref):
    assert orc.max_abs(got, ref) <= 2e-2, orc.max_abs(got, ref)
    assert orc.rel_fro(got, ref) <= 5e-3, orc.rel_fro(got, ref)


@pytest.mark.parametrize("n", [4096, 8192])
def test_dsl_async_gemm_bf16_reaches_tcgen05(rt, n):
    """examples/async_copy_gemm.py:32-79 at config 3 (bf16, M = N = K = n)."""
    import torch
    from enigma import _native
    ck = enigma.compile(K.make_async_gemm(n, n, n, dtype="bfloat"))
    assert (ck.cuda_kernel.op, ck.cuda_kernel.dtype) == ("gemm", "bfloat")
    g = torch.Generator(device="cuda").manual_seed(3)
    a = (torch.randn(n, n, device="cuda", generator=g) / n ** 0.5).bfloat16()
    b = torch.randn(n, n, device="cuda", generator=g).bfloat16()
    c = rt.execute(ck, [a, b], None, grid=((n // 32) ** 2, 1, 1), threads=(128, 1, 1),
                   output_shapes=[(n, n)], output_dtypes=[torch.bfloat16])
    assert _native.last_kernel() == "gemm_bf16_pair_kernel"
    idx = torch.linspace(0, n - 1, 48, device="cuda").long()
    _check_bf16(c[idx].float().cpu().numpy(),
                orc.gemm(a[idx].float().cpu().numpy(), b.float().cpu().numpy()))


def _fa_inputs(B, H, S, D, seed):
    import torch
    g = torch.Generator(device="cuda").manual_seed(seed)
    return [torch.randn(B, H, S, D, device="cuda", generator=g).bfloat16() for _ in range(3)]


def _check_fa_sample(o, q, k, v, causal, seed=0):
    B, H, S, D = q.shape
    rng = np.random.default_rng(seed)
    pairs = [(int(rng.integers(B)), int(rng.integers(H))) for _ in range(4)]
    rows = np.sort(np.concatenate([[0, S - 1], rng.integers(0, S, 30)]))
    got, ref = [], []
    for bb, hh in pairs:
        got.append(o[bb, hh, rows].float().cpu().numpy())
        ref.append(orc.sdpa_query_rows(q[bb, hh, rows].float().cpu().numpy(),
                                       k[bb, hh].float().cpu().numpy(),
                                       v[bb, hh].float().cpu().numpy(), 1.0 / D ** 0.5, causal,
                                       rows))
    _check_bf16(np.stack(got), np.stack(ref))


@pytest.mark.parametrize("S", [1024, 4096])
@pytest.mark.parametrize("causal", [False, True])
def test_dsl_fa_bf16_config4_reaches_tcgen05(rt, S, causal):
    """The showcase FA body (showcase_attention.py:31-91) at D = 128 over [8, 32, S, 128],
    (batch, head) slices along the grid's y extent; causal from the traced key > row mask."""
    import torch
    from enigma import _native
    B, H, D = 8, 32, 128
    ck = enigma.compile(K.make_fa_heads(S, D, causal))
    bnd = ck.cuda_kernel
    assert (bnd.op, bnd.layout, bnd.params["head_dim"], bnd.params["causal"]) == \
        ("sdpa", "rows", 128, causal)
    q, k, v = _fa_inputs(B, H, S, D, seed=S + causal)
    o = rt.execute(ck, [q, k, v], None, grid=(S, B * H, 1), threads=(32, 1, 1),
                   output_shapes=[(B, H, S, D)], output_dtypes=[torch.bfloat16])
    assert _native.last_kernel() == "sdpa_fwd_tc_kernel"
    _check_fa_sample(o, q, k, v, causal)


def test_dsl_fa_tv_reference_shape(rt):
    """fa_tv (showcase_attention.py:94-131): the TV-layout launcher at the example's own
    M = N = 1024, D = 4, fp32; the example's bar is 1e-3, checked here at 1e-4."""
    jit, args = K.make_fa_tv(1024, 1024, 4)
    ck = enigma.compile(jit, *args)
    assert ck.grid == (1024, 1, 1) and ck.block == (32, 1, 1)
    rng = np.random.default_rng(1234)
    q, k, v = (rng.standard_normal((1024, 4)).astype(np.float32) for _ in range(3))
    raw = rt.execute(ck, [q.ravel(), k.ravel(), v.ravel()], 1024 * 4 * 4, grid=ck.grid,
                     threads=ck.block)
    o = np.frombuffer(raw, np.float32).reshape(1024, 4)
    np.testing.assert_allclose(o, orc.sdpa(q[None, None], k[None, None], v[None, None], 0.5)[0, 0],
                               rtol=1e-4, atol=1e-5)


def test_dsl_fa_tv_bf16_heads_causal(rt):
    """fa_tv's launcher with a (batch x head) y extent at D = 128, bf16, causal: the
    tensor-core kernel behind the TV-layout form."""
    import torch
    from enigma import _native
    B, H, S, D = 2, 16, 2048, 128
    jit, args = K.make_fa_tv(S, S, D, heads=B * H, causal=True, dtype="bfloat")
    ck = enigma.compile(jit, *args)
    assert ck.grid == (S, B * H, 1) and ck.cuda_kernel.params["causal"] is True
    q, k, v = _fa_inputs(B, H, S, D, seed=9)
    o = rt.execute(ck, [q, k, v], None, grid=ck.grid, threads=ck.block,
                   output_shapes=[(B, H, S, D)], output_dtypes=[torch.bfloat16])
    assert _native.last_kernel() == "sdpa_fwd_tc_kernel"
    _check_fa_sample(o, q, k, v, True)


def test_dsl_fa_prepare_dispatch_timed(rt):
    """prepare / dispatch_timed / read_output on the tensor-core FA (runtime.py:529-656)."""
    import torch
    B, H, S, D = 1, 8, 1024, 128
    ck = enigma.compile(K.make_fa_heads(S, D, True))
    q, k, v = _fa_inputs(B, H, S, D, seed=2)
    prep = rt.prepare(ck, [q, k, v], B * H * S * D * 2)
    try:
        prep.dispatch((S, B * H, 1), (32, 1, 1))
        us = prep.dispatch_timed((S, B * H, 1), (32, 1, 1))
        assert 0 < us < 1e5
        raw = prep.read_output()
        o = torch.frombuffer(bytearray(raw), dtype=torch.bfloat16).reshape(B, H, S, D)
        _check_fa_sample(o, q.cpu(), k.cpu(), v.cpu(), True)
    finally:
        prep.release()


@pytest.mark.parametrize("M,N,Kd,ta,tb", [(3, 4, 2, False, False), (3, 4, 2, True, False),
                                         (5, 7, 6, False, True), (8, 8, 6, False, False)])
def test_tile_gemm(rt, M, N, Kd, ta, tb):
    """The reference's enigma.gemm runtime test (test_new_features_runtime.py:25-56: 3x4x2,
    grid (1,1,1), rtol 1e-5) and transposed / 8x8x8 tiles."""
    from enigma import _native
    ck = enigma.compile(K.make_tile_gemm(M, N, Kd, ta, tb))
    if (M, N, Kd) == (3, 4, 2) and not (ta or tb):
        a = np.array([[1, 2], [3, 4], [5, 6]], dtype=np.float32)
        b = np.array([[7, 8, 9, 10], [11, 12, 13, 14]], dtype=np.float32)
    else:
        rng = np.random.default_rng(M * N * Kd)
        a = rng.standard_normal((M, Kd)).astype(np.float32)
        b = rng.standard_normal((Kd, N)).astype(np.float32)
    a_buf = a.T.copy() if ta else a
    b_buf = b.T.copy() if tb else b
    raw = rt.execute(ck, [a_buf.ravel(), b_buf.ravel()], M * N * 4, grid=(1, 1, 1),
                     threads=(1, 1, 1))
    assert _native.last_kernel() == "gemm_simt_kernel"
    out = np.frombuffer(raw, np.float32).reshape(M, N)
    np.testing.assert_allclose(out, a @ b, rtol=1e-5, atol=1e-5)
