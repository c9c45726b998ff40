"""Parity at the BASELINE configurations' full sizes, on deterministic samples (a full CPU
result would take minutes): RMSNorm bf16 262144 x 8192 (64 rows), GEMM bf16 8192^3 (64 full
rows of C), SDPA bf16 [8, 32, 8192, 128] causal and non-causal (8 (b, h) pairs x 16 query
rows).  Inputs are generated on the GPU from a seeded generator; only the sampled slices
come back to the host.  SDPA runs at S = 1024 and 4096 as well (config 4's other lengths).  Tolerances: BASELINE's max-abs <= 2e-2 and relative Frobenius
<= 5e-3 for bf16 GEMM / SDPA, one bf16 ulp of the fp64 result for RMSNorm."""
import numpy as np
import pytest

from oracle import numerics as orc

pytestmark = pytest.mark.gpu


def _np(t):
    return t.float().cpu().numpy()


def test_rmsnorm_bf16_262144x8192(cuda):
    import torch
    from enigma import cuda_ops
    rows, hidden, eps = 262144, 8192, 1e-6
    g = torch.Generator(device=cuda).manual_seed(0)
    x = torch.randn(rows, hidden, device=cuda, generator=g).bfloat16()
    w = (1 + 0.1 * torch.randn(hidden, device=cuda, generator=g)).bfloat16()
    y = cuda_ops.rmsnorm(x, w, eps)
    idx = torch.linspace(0, rows - 1, 64, device=cuda).long()
    ref = orc.rmsnorm(_np(x[idx]), _np(w), eps)
    got = _np(y[idx])
    # within one bf16 ulp (2^-8 relative) of the fp64 result, plus a tiny absolute floor
    assert np.all(np.abs(got - ref) <= np.abs(ref) * 2.0 ** -8 + 1e-6)
    del x, y


def test_gemm_bf16_8192(cuda):
    import torch
    from enigma import cuda_ops
    n = 8192
    g = torch.Generator(device=cuda).manual_seed(0)
    a = (torch.randn(n, n, device=cuda, generator=g) / n ** 0.5).bfloat16()
    b = torch.randn(n, n, device=cuda, generator=g).bfloat16()
    c = cuda_ops.gemm(a, b)
    idx = torch.linspace(0, n - 1, 64, device=cuda).long()
    ref = orc.gemm(_np(a[idx]), _np(b))
    got = _np(c[idx])
    assert orc.max_abs(got, ref) <= 2e-2, orc.max_abs(got, ref)
    assert orc.rel_fro(got, ref) <= 5e-3, orc.rel_fro(got, ref)
    del a, b, c


@pytest.mark.parametrize("S", [1024, 4096, 8192])
@pytest.mark.parametrize("causal", [True, False])
def test_sdpa_bf16_8x32xSx128(cuda, causal, S):
    """Config 4 at every listed sequence length, causal and non-causal."""
    import torch
    from enigma import cuda_ops, _native
    B, H, D = 8, 32, 128
    g = torch.Generator(device=cuda).manual_seed(1)
    q, k, v = (torch.randn(B, H, S, D, device=cuda, generator=g).bfloat16() for _ in range(3))
    o = cuda_ops.sdpa(q, k, v, scale=1.0 / D ** 0.5, causal=causal)
    assert _native.last_kernel() == "sdpa_fwd_tc_kernel"
    rng = np.random.default_rng(5)
    pairs = [(int(rng.integers(B)), int(rng.integers(H))) for _ in range(8)]
    rows = np.sort(np.concatenate([[0, S - 1], rng.integers(0, S, 14)]))
    got, ref = [], []
    for bb, hh in pairs:
        got.append(_np(o[bb, hh, rows]))
        ref.append(orc.sdpa_query_rows(_np(q[bb, hh, rows]), _np(k[bb, hh]), _np(v[bb, hh]),
                                       1.0 / D ** 0.5, causal, rows))
    got, ref = np.stack(got), np.stack(ref)
    assert orc.max_abs(got, ref) <= 2e-2, orc.max_abs(got, ref)
    assert orc.rel_fro(got, ref) <= 5e-3, orc.rel_fro(got, ref)
    del q, k, v, o
