"""Recognizer: the B200 build's "lowering" step.

The reference lowers a traced kernel to MSL through its MLIR dialect
(enigma/compiler/compiler.py:133-211).  Here a traced kernel is instead
identified as one of the hot-path operators the sm_100a library implements
and bound to that kernel with its parameters.  There is no code generation
and no fallback: an unrecognised kernel raises EnigmaError.

A Binding holds what the trace fixes (operator, dtype, eps, scale, shapes
that are compile-time constants, buffer layout variant) and resolves the
rest at dispatch time from the buffer sizes and launch grid, the way the
Metal kernels took their extents from the buffers they were bound to.

Fingerprints (op kinds present in the trace, buffer signature):
  rmsnorm    simd_sum + rsqrt + per-thread vector loads/stores, or the
             loop form used inside the Qwen layer; 3 buffers (x, w, y)
             -- examples/benchmark_rmsnorm.py:31-84
  sdpa_gqa   exp + fmax + simd_sum(dot) with an interleaved KV buffer and a
             running-max buffer; 4 buffers (Q, KV, M0, O)
             -- examples/benchmark_sdpa.py:48-158
  sdpa_rows  exp + fmax + dot inside a carried loop (one query row per
             thread); 4 buffers (Q, K, V, O); head_dim = the number of Q
             elements a thread loads; (batch, head) slices along the grid's
             y / z extent; causal when a score is replaced by a large negative
             constant where the key index (loop-dependent) exceeds the query
             row -- examples/showcase_attention.py:31-125
  gemm       one enigma.gemm tile op (fp32; shape and transposes from its marker)
             -- enigma/ops/gemm.py:51-167; or dot of two 4-vectors into C (C = A B, or C += A B when C is
             also read) -- tests/metal/test_gemm_matmul_runtime.py:20-60;
             or async 2-D tile copies of A and B into threadgroup memory
             -- examples/async_copy_gemm.py:32-79 (bound to the GEMM it
             stages tiles for: the shipped example never multiplies)
  decode     the Qwen single-layer decode megakernel (26 buffers)
             -- examples/qwen_megakernel.py:228-269
  elementwise  C = A op B with exactly one value op on two loads, per TV value or per
             thread -- examples/vector_add_tv.py:13-55, examples/vector_add.py
"""
from __future__ import annotations

import math
from collections import Counter
from dataclasses import dataclass, field
from typing import Dict, List, Optional, Tuple

from .._tracing import EnigmaError, IRValue, KernelBuilder
from ..tensor import Tensor
from ..tuple import product


@dataclass
class Binding:
    """Which sm_100a operator a compiled kernel runs, and with what."""

    op: str                                   # rmsnorm | sdpa | gemm | decode
    dtype: str                                # "float" | "bfloat"
    params: Dict[str, object] = field(default_factory=dict)
    layout: str = "dense"                     # buffer layout variant (sdpa: dense|gqa_interleaved)

    def describe(self) -> str:
        ps = ", ".join(f"{k}={v}" for k, v in sorted(self.params.items()))
        return f"{self.op}[{self.dtype}, {self.layout}]({ps})"


class _Trace:
    """Queries over a KernelBuilder: op counts, constants, producers."""

    def __init__(self, b: KernelBuilder):
        self.b = b
        self.ops = list(b.walk())
        self.kinds = Counter(op.op for op in self.ops)
        self.producer = {id(op.result): op for op in self.ops if op.result is not None}

    def has(self, *kinds) -> bool:
        return all(self.kinds[k] > 0 for k in kinds)

    def const_of(self, v) -> Optional[float]:
        if not isinstance(v, IRValue):
            return None
        op = self.producer.get(id(v))
        if op is None:
            return None
        if op.op == "const":
            return op.attrs.get("value")
        if op.op == "cast":
            return self.const_of(op.operands[0])
        return None

    def source_of(self, v):
        """Where a scalar operand comes from: a literal (float), a Scalar kernel
        parameter ({"scalar": buffer_index}) or a function constant ({"constant": index});
        None otherwise.  Lets eps / scale be runtime values (runtime.py:125-175, :358-364)."""
        c = self.const_of(v)
        if c is not None:
            return float(c)
        op = self.def_of(v)
        while op is not None and op.op == "cast":
            op = self.def_of(op.operands[0])
        if op is None:
            return None
        if op.op == "function_constant":
            return {"constant": int(op.attrs["index"])}
        if op.op == "load" and any(sp[1] == op.attrs.get("buffer_index") for sp in
                                   self.b.scalar_params):
            return {"scalar": int(op.attrs["buffer_index"])}
        return None

    def n_buffers(self) -> int:
        return len(self.b.args) - len(self.b.scalar_params)

    def buffer_dtypes(self):
        scal = {sp[1] for sp in self.b.scalar_params}
        return [a[2] for a in self.b.args if a[1] not in scal]

    def def_of(self, v):
        return self.producer.get(id(v)) if isinstance(v, IRValue) else None

    def consts(self, dtype_prefix: str = "") -> List:
        return [op.attrs.get("value") for op in self.ops
                if op.op == "const" and op.result.dtype.startswith(dtype_prefix)]

    def depends_on_loop(self, v, _memo=None) -> bool:
        """True when `v` is computed from the induction variable of a traced loop."""
        if _memo is None:
            _memo = {}
            ivs = {id(op.attrs["iv"]) for op in self.ops if op.op == "scf_for" and "iv" in op.attrs}
            _memo["ivs"] = ivs
        if not isinstance(v, IRValue):
            return False
        if id(v) in _memo["ivs"]:
            return True
        if id(v) in _memo:
            return _memo[id(v)]
        _memo[id(v)] = False
        op = self.producer.get(id(v))
        r = op is not None and any(self.depends_on_loop(o, _memo) for o in op.operands)
        _memo[id(v)] = r
        return r

    def loads_of(self, buffer: str) -> int:
        return sum(1 for op in self.ops if op.op == "load" and op.attrs.get("buffer") == buffer)

    def vec_widths(self) -> List[int]:
        return [int(op.result.dtype[-1]) for op in self.ops if op.op == "make_vec"]


# ----------------------------------------------------------------------------- rmsnorm
def _rmsnorm_eps(t: _Trace) -> Tuple[Optional[float], Optional[float]]:
    """eps and the mean divisor from rsqrt(sum / N + eps)."""
    for op in t.ops:
        if op.op not in ("rsqrt", "tv_rsqrt"):
            continue
        add = t.def_of(op.operands[0])
        if add is None or add.op not in ("add", "tv_add"):
            continue
        a, b = add.operands
        eps = t.source_of(b)
        mean = t.def_of(a)
        if eps is None:
            eps, mean = t.source_of(a), t.def_of(b)
        n = None
        if mean is not None and mean.op in ("div", "tv_div"):
            n = t.const_of(mean.operands[1])
        return eps, n
    return None, None


def _match_rmsnorm(t: _Trace, args: tuple) -> Optional[Binding]:
    if t.n_buffers() != 3 or not t.has("rsqrt", "simd_sum"):
        return None
    if t.kinds["exp"] or t.kinds["dot"]:
        return None
    eps, n = _rmsnorm_eps(t)
    if eps is None:
        return None
    dtypes = set(t.buffer_dtypes())
    if len(dtypes) != 1 or not dtypes <= {"float", "bfloat"}:
        return None
    params = {"eps": eps}
    if n:
        params["hidden"] = int(n)
    x = _first_tensor(args, 2)
    if x is not None:
        shp = x.layout.shape
        params["rows"] = product(shp[0])
        params["hidden"] = product(shp[1])
    vw = [c for op in t.ops if op.op == "tv_load" for _, c in op.attrs["groups"]]
    if vw:
        params["vector_run"] = max(vw)
    return Binding("rmsnorm", dtypes.pop(), params)


def _first_tensor(args, rank: int) -> Optional[Tensor]:
    for a in args or ():
        if isinstance(a, Tensor) and a.layout is not None:
            s = a.layout.shape
            if isinstance(s, tuple) and len(s) == rank:
                return a
    return None


# ----------------------------------------------------------------------------- sdpa
_MASK_GT = {"cmp_gt": False, "cmp_ugt": False, "cmp_lt": True, "cmp_ult": True}


def _causal_mask(t: _Trace) -> bool:
    """Find `where(score, -big, key > row)`: a select whose taken value is a constant at or
    below -1e20 under a strict comparison with the loop-dependent (key) side greater.
    Returns False without such a select; raises for a mask of another shape, which no
    sm_100a kernel here implements (e.g. key >= row, or a mask not tied to the key loop)."""
    for op in t.ops:
        if op.op != "select":
            continue
        _false, taken, cond = op.operands
        c = t.const_of(taken)
        if c is None or c > -1e20:
            continue
        cop = t.def_of(cond)
        if cop is None or cop.op not in _MASK_GT:
            raise EnigmaError("attention mask: only `key > query` (causal) masks are supported")
        hi, lo = cop.operands
        if _MASK_GT[cop.op]:
            hi, lo = lo, hi
        if t.depends_on_loop(hi) and not t.depends_on_loop(lo):
            return True
        raise EnigmaError("attention mask: only `key > query` (causal) masks are supported")
    return False


def _match_sdpa(t: _Trace, args: tuple) -> Optional[Binding]:
    if t.n_buffers() != 4 or not t.has("exp", "fmax"):
        return None
    dtype = t.buffer_dtypes()[0]
    if dtype not in ("float", "bfloat"):
        return None
    if t.has("simd_sum", "dot", "threadgroup_alloc"):
        # GQA decode attention over an interleaved [kv_head, token, K|V] buffer,
        # no 1/sqrt(D) scale, running max initialised from buffer 2.
        return Binding("sdpa", dtype, {"scale": 1.0, "causal": False}, layout="gqa_interleaved")
    if t.has("dot") and t.kinds["scf_for"] >= 1:
        widths = t.vec_widths()
        d = t.loads_of(t.b.args[0][0]) or (widths[0] if widths else None)
        scale = None
        for op in t.ops:
            if op.op == "rsqrt":
                c = t.const_of(op.operands[0])
                if c:
                    scale = 1.0 / math.sqrt(c)
            elif op.op in ("mul", "tv_mul") and scale is None:
                # score * scale with the scale a Scalar parameter or function constant
                for o in op.operands:
                    src = t.source_of(o)
                    if isinstance(src, dict):
                        scale = src
        params = {"scale": scale if scale is not None else 1.0, "causal": _causal_mask(t)}
        if d:
            params["head_dim"] = d
        q = _first_tensor(args, 2)
        if q is not None:
            params["seq_q"] = q.layout.shape[0]
            params["head_dim"] = q.layout.shape[1]
        return Binding("sdpa", dtype, params, layout="rows")
    return None


# ----------------------------------------------------------------------------- gemm
def _match_gemm(t: _Trace, args: tuple) -> Optional[Binding]:
    if len(t.b.args) != 3:
        return None
    dtype = t.b.args[0][2]
    tiles = [op for op in t.ops if op.op == "tile_gemm"]
    if tiles:
        # One enigma.gemm tile op over tiles staged from A and B (enigma/ops/gemm.py:51-167;
        # tests/metal/test_new_features_runtime.py:25-56): Out = A @ B for the whole tile.
        if len(tiles) != 1 or t.kinds["exp"]:
            return None
        a = tiles[0].attrs
        if dtype != "float" or a["accum_dtype"] != "float":
            raise EnigmaError("enigma.gemm tile op: only fp32 tiles have an sm_100a binding")
        return Binding("gemm", dtype, {"M": a["M"], "N": a["N"], "K": a["K"],
                                       "transpose_A": a["transpose_A"],
                                       "transpose_B": a["transpose_B"]}, layout="tile")
    if t.has("async_copy_2d_d2t"):
        uints = [c for c in t.consts("uint") if isinstance(c, int)]
        # The example names K and the B/C row pitch with metal_cast(..., "uint").
        ops2d = [op for op in t.ops if op.op == "async_copy_2d_d2t"]
        k = t.const_of(ops2d[0].operands[3]) if ops2d else None
        n = t.const_of(ops2d[1].operands[3]) if len(ops2d) > 1 else None
        params = {}
        if k:
            params["K"] = int(k)
        if n:
            params["N"] = int(n)
        params["tile_consts"] = sorted(set(uints))[:8]
        return Binding("gemm", dtype, params, layout="async_tiles")
    if t.has("dot", "make_vec") and not t.kinds["exp"]:
        widths = t.vec_widths()
        if not widths or len(set(widths)) != 1:
            return None
        k = widths[0]
        c_name = t.b.args[2][0]
        reads_c = any(op.op == "load" and op.attrs.get("buffer") == c_name for op in t.ops)
        params = {"K": k, "accumulate": bool(reads_c)}
        # the row pitch of B / C is the uint constant the kernel names `n`
        ncands = [c for c in t.consts("uint") if isinstance(c, int) and c > 3 and c != k]
        if ncands:
            params["N"] = ncands[0]
        return Binding("gemm", dtype, params, layout="dense")
    return None


# ----------------------------------------------------------------------------- decode layer
def _match_decode(t: _Trace, args: tuple) -> Optional[Binding]:
    if len(t.b.args) < 20 or not t.has("rsqrt", "exp", "simd_sum", "scf_for"):
        return None
    from .. import decode_layer
    return decode_layer.bind_from_trace(t)


# ----------------------------------------------------------------------------- elementwise
_EW_OPS = {"add": 0, "sub": 1, "mul": 2, "fmax": 3, "fmin": 4}
_EW_ALLOWED = {"tv_load", "tv_store", "load", "store", "const", "cast", "add", "sub", "mul",
               "div", "mod", "thread_position_in_grid", "thread_position_in_threadgroup",
               "threadgroup_position_in_grid", "threads_per_threadgroup"}


def _match_elementwise(t: _Trace, args: tuple) -> Optional[Binding]:
    """C = A op B, one element per thread (examples/vector_add.py) or per TV value
    (examples/vector_add_tv.py:13-55): exactly one value op combining the two loads."""
    if len(t.b.args) != 3:
        return None
    dtypes = {a[2] for a in t.b.args}
    if len(dtypes) != 1 or not dtypes <= {"float", "bfloat"}:
        return None
    kinds = set(t.kinds)
    tv = {"tv_add": 0, "tv_sub": 1, "tv_mul": 2}
    if kinds & {"tv_load"}:
        ops = [k for k in kinds if k in tv]
        if len(ops) != 1 or t.kinds[ops[0]] != 1 or t.kinds["tv_load"] != 2 or \
                t.kinds["tv_store"] != 1 or kinds - _EW_ALLOWED - set(tv):
            return None
        runs = [c for op in t.ops if op.op == "tv_load" for _, c in op.attrs["groups"]]
        return Binding("elementwise", dtypes.pop(), {"op": tv[ops[0]], "vector_run": max(runs)},
                       layout="tv")
    if t.kinds["load"] != 2 or t.kinds["store"] != 1 or kinds - _EW_ALLOWED - {"fmax", "fmin"}:
        return None
    store = next(op for op in t.ops if op.op == "store")
    val = t.def_of(store.operands[1])
    if val is None or val.op not in _EW_OPS:
        return None
    srcs = [t.def_of(o) for o in val.operands]
    if not all(s is not None and s.op == "load" for s in srcs):
        return None
    return Binding("elementwise", dtypes.pop(), {"op": _EW_OPS[val.op]}, layout="naive")


_MATCHERS = (_match_decode, _match_rmsnorm, _match_sdpa, _match_gemm, _match_elementwise)


def recognize(builder: KernelBuilder, args: tuple = ()) -> Binding:
    t = _Trace(builder)
    for m in _MATCHERS:
        b = m(t, args)
        if b is not None:
            return b
    raise EnigmaError(
        f"no sm_100a implementation for kernel '{builder.kernel_name}': the B200 backend runs "
        f"the hot-path operators (RMSNorm, SDPA, GEMM, the Qwen decode layer) and has no "
        f"general code generator or CPU fallback")
