"""Failure reporting without a GPU fault: a bounded device-side wait that runs out (on a
barrier nothing arrives on) flags the device status word; the host learns it at the next
synchronize (ENIGMA_ERR_TIMEOUT, -3), the word is cleared, and the context stays usable."""
import numpy as np
import pytest

from oracle import numerics as orc

pytestmark = pytest.mark.gpu


def test_timeout_reported_then_context_usable(cuda):
    import torch
    from enigma import _native, cuda_ops
    lib = _native.lib()
    _native.check(lib.enigma_check_timeout_path(1000, None), "timeout probe")
    assert lib.enigma_synchronize(None) == -3
    assert "exceeded its limit" in _native.last_error()
    assert lib.enigma_synchronize(None) == 0          # reported once, then cleared
    # The Python wrapper raises the same status.
    _native.check(lib.enigma_check_timeout_path(10, None), "timeout probe")
    with pytest.raises(_native.EnigmaCudaError) as ei:
        cuda_ops.synchronize(torch.cuda.current_device())
    assert ei.value.status == -3
    # Kernels still run correctly afterwards.
    x = torch.randn(64, 4096, device=cuda)
    w = torch.randn(4096, device=cuda)
    y = cuda_ops.rmsnorm(x, w, 1e-6)
    np.testing.assert_allclose(y.cpu().numpy(), orc.rmsnorm(x.cpu().numpy(), w.cpu().numpy(), 1e-6),
                               rtol=1e-5, atol=1e-6)


def test_timeout_probe_rejects_bad_polls(cuda):
    from enigma import _native
    assert _native.lib().enigma_check_timeout_path(-1, None) == -4
