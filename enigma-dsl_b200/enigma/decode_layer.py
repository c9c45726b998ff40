"""Decoder-layer decode step on B200 (the reference's
qwen_fused megakernel, examples/qwen_megakernel.py:228-269).

`DecodeLayer` owns bf16 weights and the KV cache as torch CUDA tensors and
calls enigma_decode_layer_bf16: RMSNorm -> QKV (cluster split-K tcgen05, RoPE +
KV append in its epilogue) -> split-KV attention -> O-proj (+ residual, norm weight
and row sums of squares) -> gate|up (RMSNorm factor, SwiGLU) -> down (+ residual).  `qwen_fused`-style DSL kernels are recognised by
enigma.compile and bound here too (bind_from_trace).
"""
from __future__ import annotations

import ctypes
import math
from dataclasses import dataclass
from typing import Optional

from . import _native
from ._tracing import EnigmaError


# Buffer order of the reference's qwen_fused kernel (examples/qwen_megakernel.py:229-240).
QWEN_BUFFERS = ("x", "w_norm", "Wq", "Wk", "Wv", "w_q_norm", "w_k_norm", "cos_pos", "sin_pos",
                "k_cache", "v_cache", "Wo", "w_post", "Wg", "Wu", "Wd", "norm_buf", "q_buf",
                "k_buf", "v_buf", "attn_buf", "mlp_buf", "post_buf", "q_rope_buf", "k_rope_buf",
                "out")


class DecodeDesc(ctypes.Structure):
    """Mirror of enigma_decode_layer_desc (include/enigma_cuda.h)."""

    _fields_ = [(n, ctypes.c_int64) for n in ("batch", "hidden", "heads_q", "heads_kv",
                                              "head_dim", "intermediate", "cache_capacity",
                                              "position")] + \
               [("eps", ctypes.c_float), ("attn_scale", ctypes.c_float)] + \
               [(n, ctypes.c_void_p) for n in ("w_in_norm", "w_qkv", "w_o", "w_post_norm",
                                               "w_gate_up", "w_down", "rope_cos", "rope_sin",
                                               "k_cache", "v_cache")]


@dataclass
class DecodeConfig:
    batch: int = 64
    hidden: int = 896
    heads_q: int = 14
    heads_kv: int = 2
    head_dim: int = 64
    intermediate: int = 4864
    cache_len: int = 2048          # tokens already in the cache
    cache_capacity: int = 2112     # room for cache_len + new tokens
    eps: float = 1e-6
    rope_theta: float = 1e6


def rope_tables(cfg: DecodeConfig, position: int):
    """Full-length rotate-half cos/sin tables (fp64 angles, returned fp32 numpy)."""
    import numpy as np
    half = cfg.head_dim // 2
    inv = cfg.rope_theta ** (-np.arange(half, dtype=np.float64) * 2.0 / cfg.head_dim)
    ang = position * np.concatenate([inv, inv])
    return np.cos(ang).astype(np.float32), np.sin(ang).astype(np.float32)


class DecodeLayer:
    """One layer's weights + KV cache on a CUDA device; step(x) runs one decode step."""

    def __init__(self, cfg: DecodeConfig, weights: dict, k_cache, v_cache):
        import torch
        from . import cuda_ops
        self.cfg = cfg
        self.w = weights
        self.k_cache, self.v_cache = k_cache, v_cache
        dev = k_cache.device
        cuda_ops.ensure_device(dev.index or 0)
        self.position = cfg.cache_len
        self._cos = torch.empty(cfg.head_dim, dtype=torch.float32, device=dev)
        self._sin = torch.empty(cfg.head_dim, dtype=torch.float32, device=dev)
        self._set_rope()
        self.desc = self._desc()
        n = ctypes.c_size_t()
        _native.call("enigma_decode_workspace_bytes", ctypes.byref(self.desc), ctypes.byref(n))
        self.workspace = torch.empty(n.value, dtype=torch.uint8, device=dev)

    @classmethod
    def random(cls, cfg: DecodeConfig, device="cuda", seed: int = 0):
        """Random-init bf16 weights ~ N(0, 0.02), norm weights 1 + 0.1 N(0,1), KV ~ N(0,1)."""
        import torch
        g = torch.Generator(device=device).manual_seed(seed)
        H, D, I = cfg.hidden, cfg.head_dim, cfg.intermediate
        nqkv = (cfg.heads_q + 2 * cfg.heads_kv) * D

        def rn(*shape, std=1.0, mean=0.0):
            return (torch.randn(*shape, device=device, generator=g) * std + mean).bfloat16()

        w = {"w_in_norm": rn(H, std=0.1, mean=1.0), "w_qkv": rn(H, nqkv, std=0.02),
             "w_o": rn(cfg.heads_q * D, H, std=0.02), "w_post_norm": rn(H, std=0.1, mean=1.0),
             "w_gate_up": rn(H, 2 * I, std=0.02), "w_down": rn(I, H, std=0.02)}
        kc = torch.zeros(cfg.batch, cfg.heads_kv, cfg.cache_capacity, D, dtype=torch.bfloat16,
                         device=device)
        vc = torch.zeros_like(kc)
        kc[:, :, :cfg.cache_len] = rn(cfg.batch, cfg.heads_kv, cfg.cache_len, D)
        vc[:, :, :cfg.cache_len] = rn(cfg.batch, cfg.heads_kv, cfg.cache_len, D)
        return cls(cfg, w, kc, vc)

    def _set_rope(self):
        import torch
        c, s = rope_tables(self.cfg, self.position)
        self._cos.copy_(torch.from_numpy(c))
        self._sin.copy_(torch.from_numpy(s))

    def _desc(self) -> DecodeDesc:
        c = self.cfg
        d = DecodeDesc(batch=c.batch, hidden=c.hidden, heads_q=c.heads_q, heads_kv=c.heads_kv,
                       head_dim=c.head_dim, intermediate=c.intermediate,
                       cache_capacity=c.cache_capacity, position=self.position, eps=c.eps,
                       attn_scale=1.0 / math.sqrt(c.head_dim))
        for k, t in self.w.items():
            setattr(d, k, t.data_ptr())
        d.rope_cos, d.rope_sin = self._cos.data_ptr(), self._sin.data_ptr()
        d.k_cache, d.v_cache = self.k_cache.data_ptr(), self.v_cache.data_ptr()
        return d

    def step(self, x, out=None, advance: bool = False):
        """out = layer(x) for x [batch, hidden] bf16; the new k/v land at `position`.

        advance=True moves `position` forward (and the RoPE tables) for the next token;
        the default re-runs the same position (what a benchmark repeats).
        """
        import torch
        if out is None:
            out = torch.empty_like(x)
        s = torch.cuda.current_stream(x.device).cuda_stream
        _native.call("enigma_decode_layer_bf16", ctypes.byref(self.desc), x.data_ptr(),
                     out.data_ptr(), self.workspace.data_ptr(), self.workspace.numel(), s)
        if advance:
            if self.position + 1 >= self.cfg.cache_capacity:
                raise EnigmaError("KV cache full")
            self.position += 1
            self._set_rope()
            self.desc.position = self.position
        return out

    def capture(self, x, out):
        """Record one step (fixed x / out buffers, current position) as a CUDA graph and
        return a function that replays it: the step's 6 launches become one submission."""
        import torch
        side = torch.cuda.Stream(device=x.device)
        side.wait_stream(torch.cuda.current_stream(x.device))
        with torch.cuda.stream(side):
            self.step(x, out=out)            # first launches happen outside capture
        torch.cuda.current_stream(x.device).wait_stream(side)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            self.step(x, out=out)
        self._graph = graph                  # keep alive
        return graph.replay

    def weight_bytes(self) -> int:
        return sum(t.numel() * t.element_size() for t in self.w.values())


class QwenF32Desc(ctypes.Structure):
    """Mirror of enigma_qwen_decode_f32_desc (include/enigma_cuda.h)."""

    _fields_ = [(n, ctypes.c_int64) for n in ("hidden", "heads_q", "heads_kv", "head_dim",
                                              "intermediate", "cache_total")] + \
               [("eps", ctypes.c_float), ("attn_scale", ctypes.c_float)] + \
               [(n, ctypes.c_void_p) for n in QWEN_BUFFERS]


def bind_from_trace(t):
    """Bind a qwen_fused-style trace (26 fp32 buffers in the reference's order,
    examples/qwen_megakernel.py:228-240): eps from the first rsqrt(sum / N + eps)."""
    from .compiler.recognize import Binding, _rmsnorm_eps
    if len(t.b.args) != len(QWEN_BUFFERS) or any(a[2] != "float" for a in t.b.args):
        return None
    eps, _ = _rmsnorm_eps(t)
    if eps is None:
        return None
    return Binding("decode", "float", {"eps": float(eps)}, layout="qwen_fused_f32")


def plan_decode(binding, nbytes):
    """Sizes from the buffers (fp32 elements): x [H], w_q_norm [D], Wq [Hq*D, H],
    Wk [Hkv*D, H], K cache [Hkv, T, D], Wg [I, H]; attention scale 1/sqrt(D) as in the
    reference (ATTN_SCALE, qwen_megakernel.py:32)."""
    from .runtime_dispatch.launch import LaunchPlan
    n = {name: b // 4 for name, b in zip(QWEN_BUFFERS, nbytes)}
    H, D = n["x"], n["w_q_norm"]
    if H <= 0 or D <= 0 or n["Wq"] % (H * D) or n["Wk"] % (H * D):
        raise RuntimeError("enigma GPU error: qwen decode buffers do not give consistent sizes")
    hq, hkv = n["Wq"] // (H * D), n["Wk"] // (H * D)
    total = n["k_cache"] // (hkv * D)
    inter = n["Wg"] // H
    eps = float(binding.params["eps"])

    def fn(ptrs, stream):
        d = QwenF32Desc(hidden=H, heads_q=hq, heads_kv=hkv, head_dim=D, intermediate=inter,
                        cache_total=total, eps=eps, attn_scale=1.0 / math.sqrt(D))
        for name, ptr in zip(QWEN_BUFFERS, ptrs):
            setattr(d, name, ptr)
        _native.call("enigma_qwen_decode_f32", ctypes.byref(d), stream)
    return LaunchPlan(f"qwen decode f32 H={H} Hq={hq} Hkv={hkv} D={D} I={inter} T={total}", fn,
                      (len(QWEN_BUFFERS) - 1,))
