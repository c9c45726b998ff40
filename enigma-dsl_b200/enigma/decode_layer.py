"""Qwen-style decoder-layer decode step (examples/qwen_megakernel.py:228-269)."""
from __future__ import annotations

from ._tracing import EnigmaError


def bind_from_trace(t):
    raise EnigmaError("the decode-layer binding is built in enigma.decode_layer (pending)")


def plan_decode(binding, nbytes):
    raise EnigmaError("the decode-layer binding is built in enigma.decode_layer (pending)")
