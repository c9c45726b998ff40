"""compile() -> recognizer bindings for the hot-path kernels (CPU only)."""
import pytest

import enigma
import dsl_kernels as K


def test_rmsnorm_binding_config1():
    jit, args = K.make_rmsnorm(4096, 4096, 256, 4, 1e-6)
    ck = enigma.compile(jit, *args)
    b = ck.cuda_kernel
    assert b.op == "rmsnorm" and b.dtype == "float"
    assert b.params["eps"] == pytest.approx(1e-6) and b.params["hidden"] == 4096
    assert b.params["rows"] == 4096 and b.params["vector_run"] == 4
    assert ck.grid == (4096 * 256, 1, 1) and ck.block == (256, 1, 1)
    assert ck.num_params == 3 and ck.param_names == ["X", "W", "Out"]


def test_rmsnorm_binding_bf16_vec8():
    jit, args = K.make_rmsnorm(64, 8192, 256, 8, 1e-5, dtype="bfloat")
    b = enigma.compile(jit, *args).cuda_kernel
    assert (b.op, b.dtype, b.params["vector_run"]) == ("rmsnorm", "bfloat", 8)
    assert b.params["eps"] == pytest.approx(1e-5)


def test_sdpa_gqa_binding():
    jit, args, thr = K.make_sdpa_gqa(16, 16, 2, 64, 64)
    ck = enigma.compile(jit, *args)
    assert ck.cuda_kernel.op == "sdpa" and ck.cuda_kernel.layout == "gqa_interleaved"
    assert ck.grid == (16 * thr, 2, 1)


def test_fa_binding():
    ck = enigma.compile(K.make_fa(1024))
    b = ck.cuda_kernel
    assert (b.op, b.layout, b.params["head_dim"]) == ("sdpa", "rows", 4)
    assert b.params["scale"] == pytest.approx(0.5)


@pytest.mark.parametrize("acc", [False, True])
def test_k4_binding(acc):
    b = enigma.compile(K.make_k4(64, acc)).cuda_kernel
    assert (b.op, b.params["K"], b.params["N"], b.params["accumulate"]) == ("gemm", 4, 64, acc)


def test_async_gemm_binding():
    b = enigma.compile(K.make_async_gemm(64, 64, 64)).cuda_kernel
    assert (b.op, b.layout, b.params["K"], b.params["N"]) == ("gemm", "async_tiles", 64, 64)


def test_unrecognised_kernel_raises():
    @enigma.kernel
    def wave(A: enigma.f32, B: enigma.f32, C: enigma.f32):
        i = enigma.thread_position_in_grid
        C[i] = enigma.sin(A[i]) * B[i]

    with pytest.raises(enigma.EnigmaError, match="no sm_100a implementation"):
        enigma.compile(wave)


def test_launch_outside_compile_raises():
    jit, args = K.make_rmsnorm(8, 1024, 256, 4, 1e-6)
    with pytest.raises(RuntimeError, match="outside enigma.compile"):
        jit.fn(*args)


def test_tracing_records_loops_and_carries():
    ck = enigma.compile(K.make_fa(64))
    assert "scf_for" in ck.metal_source and "exp" in ck.metal_source


def test_qwen_fused_binding():
    ck = enigma.compile(K.make_qwen(256, 512, 4, 2, 9))
    b = ck.cuda_kernel
    assert (b.op, b.layout) == ("decode", "qwen_fused_f32") and b.params["eps"] == pytest.approx(1e-6)
    assert ck.num_params == 26


def test_tv_add_binding():
    jit, args = K.make_tv_add(256, 512)
    b = enigma.compile(jit, *args).cuda_kernel
    assert (b.op, b.layout, b.params["op"]) == ("elementwise", "tv", 0)


@pytest.mark.parametrize("fn,code", [(lambda a, b: a + b, 0), (lambda a, b: a * b, 2),
                                     (lambda a, b: enigma.fmax(a, b), 3)])
def test_naive_binary_binding(fn, code):
    b = enigma.compile(K.make_naive_binary(fn)).cuda_kernel
    assert (b.op, b.layout, b.params["op"]) == ("elementwise", "naive", code)


def test_runtime_eps_bindings():
    b = enigma.compile(K.make_rmsnorm_runtime_eps(1024, "scalar")).cuda_kernel
    assert b.op == "rmsnorm" and b.params["eps"] == {"scalar": 2} and b.params["hidden"] == 1024
    b = enigma.compile(K.make_rmsnorm_runtime_eps(1024, "constant")).cuda_kernel
    assert b.params["eps"] == {"constant": 0}


def test_runtime_eps_resolution():
    from enigma.runtime_dispatch import launch
    b = enigma.compile(K.make_rmsnorm_runtime_eps(1024, "scalar")).cuda_kernel
    p = launch.plan(b, [8 * 1024 * 4, 1024 * 4, 8 * 1024 * 4], (8 * 256, 1, 1), (256, 1, 1),
                    {"scalars": {2: 1e-3}, "constants": {}})
    assert "eps=0.001" in p.describe
    with pytest.raises(RuntimeError, match="Scalar parameter 2 has no value"):
        launch.plan(b, [8 * 1024 * 4, 1024 * 4, 8 * 1024 * 4], (1, 1, 1), (1, 1, 1),
                    {"scalars": {}, "constants": {}})
    with pytest.raises(RuntimeError, match="execute"):
        launch.plan(b, [8 * 1024 * 4, 1024 * 4, 8 * 1024 * 4], (1, 1, 1), (1, 1, 1))


@pytest.mark.parametrize("causal", [False, True])
def test_fa_heads_binding_d128(causal):
    b = enigma.compile(K.make_fa_heads(1024, 128, causal)).cuda_kernel
    assert (b.op, b.dtype, b.layout, b.params["head_dim"], b.params["causal"]) == \
        ("sdpa", "bfloat", "rows", 128, causal)
    assert b.params["scale"] == pytest.approx(128 ** -0.5)


def test_fa_tv_binding_reference_shape():
    """fa_tv (showcase_attention.py:104-131): grid from zipped_divide(Q, (32, 4))."""
    jit, args = K.make_fa_tv(1024, 1024, 4)
    ck = enigma.compile(jit, *args)
    b = ck.cuda_kernel
    assert (b.op, b.layout, b.params["head_dim"], b.params["seq_q"], b.params["causal"]) == \
        ("sdpa", "rows", 4, 1024, False)
    assert ck.grid == (1024, 1, 1) and ck.block == (32, 1, 1)


def test_async_gemm_bf16_binding():
    b = enigma.compile(K.make_async_gemm(4096, 4096, 4096, dtype="bfloat")).cuda_kernel
    assert (b.op, b.dtype, b.params["K"], b.params["N"]) == ("gemm", "bfloat", 4096, 4096)


def test_unsupported_mask_raises():
    """A mask that keeps key > query (anti-causal) has no sm_100a kernel."""
    @enigma.kernel
    def fa_anti(Q: enigma.f32, K_: enigma.f32, V: enigma.f32, O: enigma.f32):
        row = enigma.thread_position_in_grid
        neg = enigma.metal_cast(-1e30, "float")
        z = enigma.metal_cast(0, "float")
        with enigma.for_range(0, 16, init=[neg, z, z]) as (t, c):
            s = Q[row] * K_[t]
            s = enigma.where(s, neg, enigma.cmp_ult(enigma.metal_cast(t, "uint"), row))
            qv = enigma.make_float4(Q[row], Q[row], Q[row], Q[row])
            s = s + enigma.dot(qv, qv)
            mn = enigma.fmax(c[0], s)
            p = enigma.exp(s - mn)
            c[1] = c[1] * enigma.exp(c[0] - mn) + p
            c[2] = c[2] + p * V[t]
            c[0] = mn
        O[row] = c[2] / c[1]

    with pytest.raises(enigma.EnigmaError, match="key > query"):
        enigma.compile(fa_anti)


@pytest.mark.parametrize("ta,tb", [(False, False), (True, False), (False, True)])
def test_tile_gemm_binding(ta, tb):
    """enigma.gemm tile op (enigma/ops/gemm.py:51-167) at the reference test's 3x4x2."""
    b = enigma.compile(K.make_tile_gemm(3, 4, 2, ta, tb)).cuda_kernel
    assert (b.op, b.layout, b.params["M"], b.params["N"], b.params["K"]) == ("gemm", "tile", 3, 4, 2)
    assert (b.params["transpose_A"], b.params["transpose_B"]) == (ta, tb)
