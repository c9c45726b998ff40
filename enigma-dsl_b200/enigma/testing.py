"""Platform gates for tests (the reference's enigma/testing.py, for CUDA/sm_100).

ENIGMA_FORCE_NO_CUDA=1 makes every check report "unavailable" (the analogue
of ENIGMA_FORCE_NO_METAL).
"""
from __future__ import annotations

import os


def is_cuda_available() -> bool:
    if os.environ.get("ENIGMA_FORCE_NO_CUDA"):
        return False
    try:
        import torch
        return torch.cuda.is_available()
    except Exception:
        return False


def is_sm100() -> bool:
    if not is_cuda_available():
        return False
    import torch
    return torch.cuda.get_device_capability(0)[0] == 10


def _skip(reason):
    import pytest
    return pytest.mark.skipif(True, reason=reason)


def requires_cuda(fn):
    if is_cuda_available():
        return fn
    return _skip("CUDA device not available")(fn)


def requires_sm100(fn):
    if is_sm100():
        return fn
    return _skip("sm_100 (B200) device not available")(fn)


# Names kept for callers written against the reference.
is_metal_available = is_sm100
requires_metal = requires_sm100
