"""The CPU oracle's helpers agree with each other (CPU only)."""
import numpy as np
import pytest

from oracle import numerics as orc


@pytest.mark.parametrize("causal,sq,sk", [(False, 40, 40), (True, 40, 40), (True, 17, 40)])
def test_sdpa_query_rows_matches_sdpa(causal, sq, sk):
    rng = np.random.default_rng(0)
    q = rng.standard_normal((1, 1, sq, 16)).astype(np.float32)
    k = rng.standard_normal((1, 1, sk, 16)).astype(np.float32)
    v = rng.standard_normal((1, 1, sk, 16)).astype(np.float32)
    full = orc.sdpa(q, k, v, 0.25, causal)[0, 0]
    rows = np.array([0, 3, sq - 1])
    part = orc.sdpa_query_rows(q[0, 0, rows], k[0, 0], v[0, 0], 0.25, causal, rows, sk - sq)
    np.testing.assert_allclose(part, full[rows], rtol=1e-6, atol=1e-6)


def test_sdpa_sinks_reduce_weight():
    """A sink logit only adds to the denominator: with s = -inf it is plain softmax, with a
    large s every output shrinks toward 0."""
    rng = np.random.default_rng(1)
    q = rng.standard_normal((1, 2, 4, 8)).astype(np.float32)
    k = rng.standard_normal((1, 1, 6, 8)).astype(np.float32)
    v = rng.standard_normal((1, 1, 6, 8)).astype(np.float32)
    plain = orc.sdpa(q, k, v, 1.0)
    np.testing.assert_allclose(orc.sdpa(q, k, v, 1.0, sinks=np.array([-1e30, -1e30])), plain,
                               rtol=1e-6)
    big = orc.sdpa(q, k, v, 1.0, sinks=np.array([50.0, 50.0]))
    assert np.abs(big).max() < 1e-6
