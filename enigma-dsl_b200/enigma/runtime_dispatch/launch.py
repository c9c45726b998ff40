"""Turn a recognizer Binding plus the bound buffers into one C-ABI call.

The Metal kernels read their extents from the buffers they are bound to and
from compile-time constants; the same information resolves the sizes here:
buffer byte counts (in bind order), the Metal-style grid (total threads per
axis) and the trace's constants.  Every plan is validated before anything is
launched and raises RuntimeError with the kernel's context otherwise.
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass
from typing import Callable, List, Sequence, Tuple

from .. import _native

_ES = {"float": 4, "bfloat": 2}
_DT = {"float": _native.DTYPE_F32, "bfloat": _native.DTYPE_BF16}


@dataclass
class LaunchPlan:
    """A ready C-ABI call: fn(pointers, stream) enqueues the kernel."""

    describe: str
    fn: Callable[[Sequence[int], int], None]
    outputs: Tuple[int, ...]          # bind slots written by the kernel


def _need(cond: bool, msg: str):
    if not cond:
        raise RuntimeError(f"enigma GPU error: {msg}")


def _div(nbytes: int, per: int, what: str) -> int:
    _need(per > 0 and nbytes % per == 0,
          f"{what}: buffer of {nbytes} bytes is not a whole number of {per}-byte units")
    return nbytes // per


def resolve(v, values):
    """A bound parameter: a number, or {"scalar": slot} / {"constant": index} looked up in
    this dispatch's scalar values and function constants."""
    if isinstance(v, dict):
        if "scalar" in v:
            table, key, what = (values or {}).get("scalars", {}), v["scalar"], "Scalar parameter"
        else:
            table, key, what = (values or {}).get("constants", {}), v["constant"], \
                "function constant"
        _need(key in table, f"{what} {key} has no value: pass it with scalars= / constants=")
        return float(table[key])
    return float(v)


def plan(binding, nbytes: List[int], grid: Tuple[int, ...], threads: Tuple[int, ...],
         values=None) -> LaunchPlan:
    """`nbytes` lists the device buffers in bind order without Scalar slots; `values`
    holds {"scalars": {slot: value}, "constants": {index: value}} of this dispatch."""
    if values is None and any(isinstance(v, dict) for v in binding.params.values()):
        _need(False, "this kernel takes Scalar parameters / function constants: dispatch it with "
                     "execute(..., scalars=..., constants=...)")
    if values:
        binding = type(binding)(binding.op, binding.dtype,
                                {k: (resolve(v, values) if isinstance(v, dict) else v)
                                 for k, v in binding.params.items()}, binding.layout)
    op = binding.op
    if op == "rmsnorm":
        return _plan_rmsnorm(binding, nbytes)
    if op == "gemm":
        return _plan_gemm(binding, nbytes)
    if op == "sdpa":
        return _plan_sdpa(binding, nbytes, grid, threads)
    if op == "elementwise":
        return _plan_elementwise(binding, nbytes)
    if op == "decode":
        from ..decode_layer import plan_decode
        return plan_decode(binding, nbytes)
    raise RuntimeError(f"enigma GPU error: no launch plan for operator {op!r}")


def _plan_rmsnorm(b, nbytes):
    _need(len(nbytes) == 3, f"rmsnorm binds 3 buffers (x, w, y), got {len(nbytes)}")
    es = _ES[b.dtype]
    hidden = int(b.params.get("hidden") or _div(nbytes[1], es, "rmsnorm w"))
    rows = _div(nbytes[0], es * hidden, "rmsnorm x")
    _need(nbytes[2] >= rows * hidden * es, "rmsnorm: output buffer smaller than x")
    _need(nbytes[1] >= hidden * es, "rmsnorm: weight buffer smaller than hidden")
    eps, dt = float(b.params["eps"]), _DT[b.dtype]

    def fn(p, stream):
        _native.call("enigma_rmsnorm", dt, p[0], p[1], p[2], rows, hidden, ctypes.c_float(eps),
                     stream)
    return LaunchPlan(f"rmsnorm rows={rows} hidden={hidden} eps={eps}", fn, (2,))


def _plan_gemm(b, nbytes):
    _need(len(nbytes) == 3, f"gemm binds 3 buffers (A, B, C), got {len(nbytes)}")
    es = _ES[b.dtype]
    if b.layout == "tile":
        m, n, k = (int(b.params[x]) for x in "MNK")
        ta, tb = int(bool(b.params["transpose_A"])), int(bool(b.params["transpose_B"]))
        _need(nbytes[0] >= m * k * es and nbytes[1] >= k * n * es and nbytes[2] >= m * n * es,
              f"gemm tile {m}x{n}x{k}: a buffer is smaller than its tile")

        def fn(p, stream):
            _native.call("enigma_gemm_f32_trans", p[0], p[1], p[2], m, n, k, ta, tb, 0, stream)
        return LaunchPlan(f"gemm tile M={m} N={n} K={k} transA={ta} transB={tb}", fn, (2,))
    k = int(b.params["K"])
    m = _div(nbytes[0], es * k, "gemm A")
    n = int(b.params.get("N") or _div(nbytes[1], es * k, "gemm B"))
    _need(nbytes[1] >= k * n * es, f"gemm: B holds {nbytes[1]} bytes, needs K*N = {k}x{n}")
    _need(nbytes[2] >= m * n * es, f"gemm: C holds {nbytes[2]} bytes, needs M*N = {m}x{n}")
    acc = bool(b.params.get("accumulate", False))
    if b.dtype == "bfloat":
        _need(not acc, "gemm: C += A B is fp32-only")

        def fn(p, stream):
            _native.call("enigma_gemm_bf16", p[0], p[1], p[2], m, n, k, stream)
    else:
        def fn(p, stream):
            _native.call("enigma_gemm_f32", p[0], p[1], p[2], m, n, k, int(acc), stream)
    return LaunchPlan(f"gemm M={m} N={n} K={k} accumulate={acc}", fn, (2,))


def _plan_sdpa(b, nbytes, grid, threads):
    es, dt = _ES[b.dtype], _DT[b.dtype]
    scale = float(b.params.get("scale", 1.0))
    causal = int(bool(b.params.get("causal", False)))
    if b.layout == "gptoss_args":
        # The hand-written gpt-oss kernel: buffers args, q [tokens, qkv_dim], kv per kv head
        # (kv_stride elements: [token, K|V]), s (Hq sink logits), o [tokens, Hq * D].
        _need(len(nbytes) == 5, f"sdpa_gptoss binds 5 buffers (args, q, kv, s, o), got {len(nbytes)}")
        d, hq, qmul = (int(b.params[k]) for k in ("head_dim", "num_q_heads", "qmul"))
        hkv = int(grid[1])
        tokens = int(grid[0]) // max(1, int(threads[0]))
        _need(hkv * qmul == hq, f"grid.y = {hkv} kv heads x qmul {qmul} != {hq} query heads")
        qkv_dim, kv_tokens, kv_stride = (int(b.params[k]) for k in ("qkv_dim", "kv_tokens",
                                                                     "kv_stride"))
        _need(nbytes[1] >= ((tokens - 1) * qkv_dim + hq * d) * 4, "sdpa_gptoss: q buffer too small")
        _need(nbytes[2] >= ((hkv - 1) * kv_stride + kv_tokens * 2 * d) * 4,
              "sdpa_gptoss: kv buffer too small for args.kv_stride / num_kv_tokens")
        _need(nbytes[3] >= hq * 4 and nbytes[4] >= tokens * hq * d * 4,
              "sdpa_gptoss: s / output buffer too small")
        strides = (ctypes.c_int64 * 12)(0, d, qkv_dim, 0, kv_stride, 2 * d, 0, kv_stride, 2 * d,
                                        0, d, hq * d)

        def fn(p, stream):
            _native.call("enigma_sdpa_strided_sinks", dt, p[1], p[2], p[2] + d * es, p[4], 1, hq,
                         hkv, tokens, kv_tokens, d, strides, ctypes.c_float(scale), causal, p[3],
                         stream)
        return LaunchPlan(f"sdpa_gptoss tokens={tokens} Hq={hq} Hkv={hkv} D={d} "
                          f"kv_tokens={kv_tokens}", fn, (4,))
    _need(len(nbytes) == 4, f"attention binds 4 buffers, got {len(nbytes)}")
    if b.layout == "gqa_interleaved":
        # Q, O: [tokens, Hq, D]; KV: [Hkv, kv_tokens, 2D] (K then V); buffer 2: Hq floats,
        # the sink logit each head's running max starts from (with l = 1 on the first
        # simdgroup, benchmark_sdpa.py:64-72); -1e30 in the example, where it adds nothing.
        hq = _div(nbytes[2], 4, "running-max buffer")
        hkv = int(grid[1])
        tokens = int(grid[0]) // int(threads[0])
        _need(tokens > 0 and hkv > 0 and hq % hkv == 0,
              f"grid {grid} / threads {threads} do not give tokens and kv heads")
        d = _div(nbytes[0], es * tokens * hq, "attention Q")
        kv_tokens = _div(nbytes[1], es * hkv * 2 * d, "attention KV")
        strides = (ctypes.c_int64 * 12)(0, d, hq * d, 0, kv_tokens * 2 * d, 2 * d,
                                        0, kv_tokens * 2 * d, 2 * d, 0, d, hq * d)

        def fn(p, stream):
            _native.call("enigma_sdpa_strided_sinks", dt, p[0], p[1], p[1] + d * es, p[3], 1, hq,
                         hkv, tokens, kv_tokens, d, strides, ctypes.c_float(scale), causal, p[2],
                         stream)
        return LaunchPlan(f"sdpa gqa tokens={tokens} Hq={hq} Hkv={hkv} D={d} "
                          f"kv_tokens={kv_tokens}", fn, (3,))
    # One query row per thread along x; the grid's y * z extent counts the (batch, head)
    # slices of dense [B*H, S, D] buffers (1 for the single-head showcase kernel).
    d = int(b.params["head_dim"])
    bh = max(1, int(grid[1]) if len(grid) > 1 else 1) * max(1, int(grid[2]) if len(grid) > 2
                                                            else 1)
    sq = _div(nbytes[0], es * d * bh, "attention Q")
    sk = _div(nbytes[1], es * d * bh, "attention K")
    _need(nbytes[2] >= bh * sk * d * es and nbytes[3] >= bh * sq * d * es,
          "attention V / O too small")
    _need(int(grid[0]) <= sq or bh == 1,
          f"grid.x = {grid[0]} query rows exceeds the {sq} rows of each (batch, head) slice")
    name = "enigma_sdpa_bf16" if b.dtype == "bfloat" else "enigma_sdpa_f32"

    def fn(p, stream):
        _native.call(name, p[0], p[1], p[2], p[3], 1, bh, bh, sq, sk, d, ctypes.c_float(scale),
                     causal, stream)
    return LaunchPlan(f"sdpa rows heads={bh} Sq={sq} Sk={sk} D={d} scale={scale} "
                      f"causal={bool(causal)}", fn, (3,))


def _plan_elementwise(b, nbytes):
    _need(len(nbytes) == 3, f"elementwise binds 3 buffers (A, B, C), got {len(nbytes)}")
    es, dt = _ES[b.dtype], _DT[b.dtype]
    n = _div(nbytes[0], es, "elementwise A")
    _need(nbytes[1] >= n * es and nbytes[2] >= n * es, "elementwise: B / C smaller than A")
    opc = int(b.params["op"])

    def fn(p, stream):
        _native.call("enigma_elementwise", opc, dt, p[0], p[1], p[2], n, stream)
    return LaunchPlan(f"elementwise op={opc} n={n}", fn, (2,))
