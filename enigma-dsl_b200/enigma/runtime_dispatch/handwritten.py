"""Bindings for the reference's hand-written Metal kernels.

The reference's benchmarks build two kernels outside the DSL and wrap the compiled
metallib in a bare ``CompiledKernel(kernel_name, metallib_path, metallib_bytes,
metal_source)`` (examples/benchmark_rmsnorm.py:95-112, examples/benchmark_sdpa.py:171-181),
then dispatch them through the same ``MetalRuntime.execute`` / ``prepare``.  Such a kernel
has no trace to recognise, so it is bound here by its kernel name, with the sizes its
source compiles in read from ``metal_source`` when the caller passes it:

* ``rmsnorm`` (examples/metal/rmsnorm_handwritten.metal:4-46): buffers x, w, y (fp32,
  float4-vectorised rows), one threadgroup per row; N (4096) and eps (1e-5) are constants
  of the source.  Runs on the fp32 RMSNorm kernel.
* ``sdpa_gptoss`` (examples/metal/sdpa_handwritten.metal:16-158): buffers args
  {qkv_dim, num_kv_tokens, kv_stride, window} (uint32), q, kv (per kv head
  [token, K|V]), s (per query head: the sink logit the running max starts from, l starting
  at 1), output; grid.x = tokens * threads.x, grid.y = kv heads; num_q_heads (64),
  head_dim (64) and qmul (8) are constants of the source; no score scale.  Runs on the
  strided CUDA-core attention with the sink term (enigma_sdpa_strided_sinks).
"""
from __future__ import annotations

import re
from typing import Any, Callable, Dict, List, Optional

import numpy as np

from ..compiler.recognize import Binding


def _const(src: str, name: str, default, cast=int):
    m = re.search(r"const\s+(?:uint|int|float)\s+" + name + r"\s*=\s*([0-9.eE+-]+)f?\s*;",
                  src or "")
    return cast(m.group(1)) if m else default


def _host_bytes(x: Any) -> bytes:
    """Bytes of a host array / bytes object / torch tensor (copied back if on a GPU)."""
    if isinstance(x, (bytes, bytearray, memoryview)):
        return bytes(x)
    try:
        import torch
        if isinstance(x, torch.Tensor):
            t = x.detach().contiguous()
            if t.is_cuda:
                t = t.cpu()
            return t.view(torch.uint8).numpy().tobytes()
    except ImportError:
        pass
    return np.ascontiguousarray(x).tobytes()


def _rmsnorm(src: str, inputs: List[Any]) -> Binding:
    n = _const(src, "N", 4096)
    eps = _const(src, "eps", 1e-5, float)
    return Binding("rmsnorm", "float", {"hidden": n, "eps": eps}, layout="dense")


def _sdpa_gptoss(src: str, inputs: List[Any]) -> Binding:
    if not inputs:
        raise RuntimeError("enigma GPU error: sdpa_gptoss binds args, q, kv, s before the "
                           "output; got no inputs")
    raw = _host_bytes(inputs[0])
    if len(raw) < 16:
        raise RuntimeError(f"enigma GPU error: sdpa_gptoss args buffer holds {len(raw)} bytes, "
                           "needs 16 (qkv_dim, num_kv_tokens, kv_stride, window)")
    qkv_dim, kv_tokens, kv_stride, window = (int(v) for v in np.frombuffer(raw[:16], "<u4"))
    params = {"scale": 1.0, "causal": False, "head_dim": _const(src, "head_dim", 64),
              "num_q_heads": _const(src, "num_q_heads", 64), "qmul": _const(src, "qmul", 8),
              "qkv_dim": qkv_dim, "kv_tokens": kv_tokens, "kv_stride": kv_stride,
              "window": window}
    return Binding("sdpa", "float", params, layout="gptoss_args")


KNOWN: Dict[str, Callable[[str, List[Any]], Binding]] = {
    "rmsnorm": _rmsnorm,
    "sdpa_gptoss": _sdpa_gptoss,
}


def bind(kernel_name: str, metal_source: Optional[str], inputs: List[Any]) -> Optional[Binding]:
    """The binding of a known hand-written kernel, or None."""
    f = KNOWN.get(kernel_name)
    return f(metal_source or "", list(inputs)) if f else None
