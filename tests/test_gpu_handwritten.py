"""The reference's hand-written Metal kernels, dispatched the way its benchmarks do: a bare
CompiledKernel(kernel_name, metallib_path, metallib_bytes, metal_source) through
MetalRuntime.execute / prepare (examples/benchmark_rmsnorm.py:95-151,
examples/benchmark_sdpa.py:171-260), bound by kernel name to the sm_100a kernels and
checked against the oracle with the examples' tolerances or tighter."""
import struct

import numpy as np
import pytest

import enigma
from enigma.compiler.compiler import CompiledKernel
from oracle import numerics as orc

pytestmark = pytest.mark.gpu

# The compile-time constants as the shipped sources declare them.
RMSNORM_SRC = "kernel void rmsnorm(...) {\n    const uint N = 4096;\n    const float eps = 1e-5f;\n}\n"


@pytest.fixture(scope="module")
def rt(cuda):
    return enigma.MetalRuntime()


def test_handwritten_rmsnorm(rt):
    rows, n = 512, 4096
    ck = CompiledKernel(kernel_name="rmsnorm", metallib_path=None, metallib_bytes=None,
                        metal_source=RMSNORM_SRC)
    rng = np.random.default_rng(42)
    x = rng.standard_normal((rows, n)).astype(np.float32)
    w = rng.standard_normal(n).astype(np.float32)
    raw = rt.execute(ck, [x.ravel(), w], rows * n * 4, grid=(rows * 256, 1, 1),
                     threads=(256, 1, 1))
    y = np.frombuffer(raw, np.float32).reshape(rows, n)
    np.testing.assert_allclose(y, orc.rmsnorm(x, w, 1e-5), rtol=1e-5, atol=1e-6)
    prep = rt.prepare(ck, [x.ravel(), w], rows * n * 4)
    try:
        assert prep.dispatch_timed((rows * 256, 1, 1), (256, 1, 1)) > 0
    finally:
        prep.release()


@pytest.mark.parametrize("sink", ["none", "finite"])
def test_handwritten_sdpa_gptoss(rt, sink):
    """benchmark_sdpa.py:182-232: 128 tokens, 64 q / 8 kv heads, d 64, 512 kv tokens, args
    struct first, no metal_source (the example passes "")."""
    T, H, G, D, S, THR = 128, 64, 8, 64, 512, 128
    rng = np.random.default_rng(42)
    q = (rng.standard_normal((T, H, D)) * 0.1).astype(np.float32)
    k = (rng.standard_normal((G, S, D)) * 0.1).astype(np.float32)
    v = (rng.standard_normal((G, S, D)) * 0.1).astype(np.float32)
    kv = np.zeros((G, S, 2 * D), np.float32)
    kv[:, :, :D], kv[:, :, D:] = k, v
    s = (np.full(H, -1e30) if sink == "none" else rng.standard_normal(H)).astype(np.float32)
    args = np.frombuffer(struct.pack("<IIII", H * D, S, S * 2 * D, S), dtype=np.float32)
    ck = CompiledKernel("sdpa_gptoss", None, None, "")
    raw = rt.execute(ck, [args, q.ravel(), kv.ravel(), s], T * H * D * 4,
                     grid=(T * THR, G, 1), threads=(THR, 1, 1))
    o = np.frombuffer(raw, np.float32).reshape(T, H, D)
    ref = orc.sdpa(q.transpose(1, 0, 2)[None], k[None], v[None], 1.0,
                   sinks=None if sink == "none" else s)[0].transpose(1, 0, 2)
    np.testing.assert_allclose(o, ref, rtol=1e-4, atol=1e-5)
    assert orc.max_abs(o, ref) < 0.05          # the example's own bar


def test_unknown_bare_kernel_raises(rt):
    ck = CompiledKernel("not_a_reference_kernel", None, None, "")
    with pytest.raises(RuntimeError, match="no sm_100a binding"):
        rt.execute(ck, [np.zeros(4, np.float32)], 16, grid=(1, 1, 1), threads=(1, 1, 1))
