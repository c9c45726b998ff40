"""The no-allocation decode step (enigma_decode_layer_bf16_noalloc).

It exists for callers that cannot allocate device memory while a step runs (a
serving loop kept out of the allocator, a plugin whose host runtime owns all device
memory): the step's scratch is a fixed array inside the library.  These tests call it
through the C ABI twice in a row and compare each result with the workspace entry
point (enigma_decode_layer_bf16) on the same inputs.  Both run the same kernels with
the same reduction order (cluster partials summed in rank order), so the outputs must
be bit-identical.  The file sorts last so a stop-at-first-failure run has already run
every other test.
"""
import ctypes

import numpy as np
import pytest

from oracle import numerics as orc

pytestmark = pytest.mark.gpu


def _layer(cfg_kwargs, seed):
    from enigma.decode_layer import DecodeConfig, DecodeLayer
    return DecodeLayer.random(DecodeConfig(**cfg_kwargs), seed=seed)


@pytest.mark.parametrize("cfg_kwargs", [
    dict(batch=4, hidden=256, heads_q=4, heads_kv=2, intermediate=512, cache_len=100,
         cache_capacity=128),
    dict()])  # batch 64, hidden 896, 14/2 heads, 4864, 2048 cached tokens
def test_noalloc_matches_workspace_entry(cuda, cfg_kwargs):
    import torch
    from enigma import _native
    layer = _layer(cfg_kwargs, seed=7)
    lib = _native.lib()
    stream = torch.cuda.current_stream().cuda_stream
    x = torch.randn(layer.cfg.batch, layer.cfg.hidden, device="cuda").bfloat16()
    ref = torch.empty_like(x)
    _native.check(lib.enigma_decode_layer_bf16(ctypes.byref(layer.desc), x.data_ptr(),
                                               ref.data_ptr(), layer.workspace.data_ptr(),
                                               layer.workspace.numel(), stream),
                  "enigma_decode_layer_bf16")
    torch.cuda.synchronize()
    want = ref.float().cpu().numpy()
    for _ in range(2):  # two calls in a row share (and reuse) the fixed scratch array
        out = torch.full_like(x, float("nan"))
        _native.check(lib.enigma_decode_layer_bf16_noalloc(ctypes.byref(layer.desc),
                                                           x.data_ptr(), out.data_ptr(), stream),
                      "enigma_decode_layer_bf16_noalloc")
        _native.check(lib.enigma_synchronize(stream), "enigma_synchronize")
        got = out.float().cpu().numpy()
        assert np.isfinite(got).all()
        assert orc.max_abs(got, want) <= 2e-2, orc.max_abs(got, want)
        assert orc.rel_fro(got, want) <= 5e-3, orc.rel_fro(got, want)
        assert torch.equal(out, ref), "the fixed-scratch entry must match bit for bit"


def test_noalloc_rejects_oversized_step(cuda):
    import torch
    from enigma import _native
    layer = _layer(dict(batch=4, hidden=256, heads_q=4, heads_kv=2, intermediate=512,
                        cache_len=10, cache_capacity=16), seed=1)
    layer.desc.intermediate = 1 << 22   # the SwiGLU activations alone (4 x 2^22 bf16) exceed 16 MiB
    x = torch.zeros(4, 256, device="cuda").bfloat16()
    rc = _native.lib().enigma_decode_layer_bf16_noalloc(ctypes.byref(layer.desc), x.data_ptr(),
                                                        x.data_ptr(), None)
    assert rc == _native.ERR_BADARG
    assert "fixed" in _native.last_error() and "scratch" in _native.last_error()


def test_noalloc_timeout_reported_once(cuda):
    """A bounded wait that runs out on the no-allocation path flags that entry's own status
    word; the host sees ENIGMA_ERR_TIMEOUT (-3) at the next synchronize, once, and the next
    no-allocation step still matches the workspace entry bit for bit."""
    import torch
    from enigma import _native
    lib = _native.lib()
    layer = _layer(dict(batch=4, hidden=256, heads_q=4, heads_kv=2, intermediate=512,
                        cache_len=60, cache_capacity=64), seed=3)
    _native.check(lib.enigma_decode_noalloc_check_timeout_path(1000, None), "probe")
    assert lib.enigma_synchronize(None) == -3
    assert "exceeded its limit" in _native.last_error()
    assert lib.enigma_synchronize(None) == 0
    _native.check(lib.enigma_decode_noalloc_check_timeout_path(10, None), "probe")
    lib.enigma_synchronize(None)  # waits for the probe; reports and clears its flag
    n = ctypes.c_int32(-1)
    _native.check(lib.enigma_take_device_status(ctypes.byref(n)), "take status")
    assert n.value == 0
    _native.check(lib.enigma_decode_noalloc_check_timeout_path(10, None), "probe")
    torch.cuda.synchronize()
    _native.check(lib.enigma_take_device_status(ctypes.byref(n)), "take status")
    assert n.value == 1
    stream = torch.cuda.current_stream().cuda_stream
    x = torch.randn(4, 256, device="cuda").bfloat16()
    ref, out = torch.empty_like(x), torch.empty_like(x)
    _native.check(lib.enigma_decode_layer_bf16(ctypes.byref(layer.desc), x.data_ptr(),
                                               ref.data_ptr(), layer.workspace.data_ptr(),
                                               layer.workspace.numel(), stream), "workspace")
    _native.check(lib.enigma_decode_layer_bf16_noalloc(ctypes.byref(layer.desc), x.data_ptr(),
                                                       out.data_ptr(), stream), "noalloc")
    _native.check(lib.enigma_synchronize(stream), "enigma_synchronize")
    assert torch.equal(out, ref)
