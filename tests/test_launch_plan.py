"""Launch planning: sizes resolved from buffer bytes / grid, errors before launch (CPU)."""
import numpy as np
import pytest

import enigma
import dsl_kernels as K
from enigma.runtime_dispatch import launch


def test_rmsnorm_plan_sizes():
    jit, args = K.make_rmsnorm(4096, 4096, 256, 4, 1e-6)
    b = enigma.compile(jit, *args).cuda_kernel
    p = launch.plan(b, [4096 * 4096 * 4, 4096 * 4, 4096 * 4096 * 4], (4096 * 256, 1, 1), (256, 1, 1))
    assert "rows=4096 hidden=4096" in p.describe and p.outputs == (2,)


def test_rmsnorm_plan_rejects_ragged_x():
    jit, args = K.make_rmsnorm(8, 1024, 256, 4, 1e-6)
    b = enigma.compile(jit, *args).cuda_kernel
    with pytest.raises(RuntimeError, match="whole number"):
        launch.plan(b, [1024 * 4 + 4, 1024 * 4, 1024 * 4], (256, 1, 1), (256, 1, 1))


def test_sdpa_gqa_plan_sizes():
    jit, args, thr = K.make_sdpa_gqa(128, 64, 8, 64, 512)
    b = enigma.compile(jit, *args).cuda_kernel
    p = launch.plan(b, [128 * 64 * 64 * 4, 8 * 512 * 128 * 4, 64 * 4, 128 * 64 * 64 * 4],
                    (128 * thr, 8, 1), (thr, 1, 1))
    assert "tokens=128 Hq=64 Hkv=8 D=64 kv_tokens=512" in p.describe


def test_gemm_k4_plan_sizes():
    b = enigma.compile(K.make_k4(64, True)).cuda_kernel
    p = launch.plan(b, [32 * 4 * 4, 4 * 64 * 4, 32 * 64 * 4], (64, 32, 1), (16, 16, 1))
    assert p.describe == "gemm M=32 N=64 K=4 accumulate=True"


def test_gemm_plan_rejects_small_c():
    b = enigma.compile(K.make_k4(64, False)).cuda_kernel
    with pytest.raises(RuntimeError, match="C holds"):
        launch.plan(b, [32 * 16, 4 * 64 * 4, 16], (64, 32, 1), (16, 16, 1))


def test_bind_count_message():
    from enigma.runtime_dispatch.runtime import MetalRuntime
    ck = enigma.compile(K.make_k4(64, False))
    with pytest.raises(RuntimeError, match="has 3 parameter"):
        MetalRuntime._check_bind_count("execute", ck, 1, 0, 1)


def test_merge_scalars():
    import numpy as np
    from enigma.runtime_dispatch.runtime import _merge_scalar_buffers
    a, b = np.zeros(2), np.ones(2)
    out = _merge_scalar_buffers([a, b], [7], [("n", 1, "uint")], num_outputs=1)
    assert out[0] is a and out[2] is b and out[1].dtype == np.uint32 and out[1][0] == 7
    with pytest.raises(RuntimeError, match="output region"):
        _merge_scalar_buffers([a], [7], [("n", 2, "uint")], num_outputs=1)


def test_handwritten_bindings_parse_constants():
    """Hand-written kernels bind by name; sizes come from the source when present."""
    import struct
    from enigma.runtime_dispatch import handwritten as hw
    b = hw.bind("rmsnorm", "const uint N = 2048;\n const float eps = 1e-6f;", [])
    assert (b.op, b.dtype, b.params["hidden"], b.params["eps"]) == ("rmsnorm", "float", 2048, 1e-6)
    assert hw.bind("rmsnorm", "", []).params == {"hidden": 4096, "eps": 1e-5}
    args = np.frombuffer(struct.pack("<IIII", 4096, 512, 65536, 512), dtype=np.float32)
    g = hw.bind("sdpa_gptoss", "", [args])
    assert g.layout == "gptoss_args" and g.params["kv_tokens"] == 512 and g.params["qkv_dim"] == 4096
    assert g.params["head_dim"] == 64 and g.params["num_q_heads"] == 64 and g.params["qmul"] == 8
    assert hw.bind("unknown", "", []) is None
    with pytest.raises(RuntimeError, match="16"):
        hw.bind("sdpa_gptoss", "", [np.zeros(2, np.float32)])


def test_handwritten_gptoss_plan_checks_sizes():
    import struct
    from enigma.runtime_dispatch import handwritten as hw
    args = np.frombuffer(struct.pack("<IIII", 64 * 64, 512, 512 * 128, 512), dtype=np.float32)
    b = hw.bind("sdpa_gptoss", "", [args])
    T, H, D, G, S = 128, 64, 64, 8, 512
    nbytes = [16, T * H * D * 4, G * S * 2 * D * 4, H * 4, T * H * D * 4]
    p = launch.plan(b, nbytes, (T * 128, G, 1), (128, 1, 1), {})
    assert "sdpa_gptoss" in p.describe and p.outputs == (4,)
    with pytest.raises(RuntimeError, match="kv buffer too small"):
        launch.plan(b, [16, nbytes[1], 1024, nbytes[3], nbytes[4]], (T * 128, G, 1), (128, 1, 1), {})
