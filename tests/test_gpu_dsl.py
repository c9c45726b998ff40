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
