"""Kernel tracer: records what an @enigma.kernel body does as a small SSA IR.

Running the kernel's Python body with proxy arguments produces a list of
IROp records (with nested regions for loops and branches).  Nothing here
generates device code: the IR is what the recognizer (enigma.compiler.
recognize) fingerprints to bind the kernel to one of the hand-written
sm_100a kernels, and what `dump_ir` prints.

The intrinsic surface is the reference's (enigma/_tracing.py and the names
re-exported by enigma/__init__.py): math, SIMD-group and quad reductions,
comparisons, grid queries, casts, threadgroup memory, atomics, control flow
(for_range with carried values, if_, while_), predicated access, register
tensors, pipelines, async copies and simdgroup matrices.  Most intrinsics
are generated from the name tables below rather than written one by one.
"""
from __future__ import annotations

import threading
from dataclasses import dataclass, field
from typing import Any, Dict, List, Optional, Sequence

from .tensor import Tensor  # noqa: F401  (re-exported: kernels import it from here)

_local = threading.local()


class EnigmaError(Exception):
    """User-facing error of the Enigma front end."""


def get_builder() -> "Optional[KernelBuilder]":
    return getattr(_local, "builder", None)


def _require_builder(what: str) -> "KernelBuilder":
    b = get_builder()
    if b is None:
        raise EnigmaError(f"{what}() can only be used inside an @enigma.kernel trace")
    return b


# ----------------------------------------------------------------------------- IR
@dataclass(eq=False)
class IRValue:
    """An SSA value of the trace.  `_tv_groups` marks a per-thread vector of
    values produced by Tensor.load() (its contiguous runs)."""

    name: str
    dtype: str
    _tv_groups: Any = field(default=None, repr=False)

    # arithmetic ---------------------------------------------------------
    def __add__(self, o):
        return self if _is_zero(o) else _arith("add", self, o)

    def __radd__(self, o):
        return self if _is_zero(o) else _arith("add", o, self)

    def __sub__(self, o):
        return _arith("sub", self, o)

    def __rsub__(self, o):
        return _arith("sub", o, self)

    def __mul__(self, o):
        return self if _is_one(o) else _arith("mul", self, o)

    def __rmul__(self, o):
        return self if _is_one(o) else _arith("mul", o, self)

    def __truediv__(self, o):
        return _arith("div", self, o)

    def __rtruediv__(self, o):
        return _arith("div", o, self)

    def __floordiv__(self, o):
        return _arith("div", self, o)

    def __mod__(self, o):
        return _arith("mod", self, o)

    def __neg__(self):
        return _emit("neg", [self], self.dtype)

    def __invert__(self):
        return _emit("bitnot", [self], self.dtype)

    def __or__(self, o):
        return _binop("bitor", self, o)

    def __ror__(self, o):
        return _binop("bitor", o, self)

    def __and__(self, o):
        return _binop("bitand", self, o)

    def __rand__(self, o):
        return _binop("bitand", o, self)

    def __xor__(self, o):
        return _binop("bitxor", self, o)

    def __rxor__(self, o):
        return _binop("bitxor", o, self)

    def __lshift__(self, o):
        return _binop("shl", self, o)

    def __rshift__(self, o):
        return _binop("shr", self, o)


@dataclass(eq=False)
class IROp:
    op: str
    result: Optional[IRValue]
    operands: List[Any]
    attrs: Dict[str, Any] = field(default_factory=dict)
    regions: List[List["IROp"]] = field(default_factory=list)


def _is_zero(x) -> bool:
    return isinstance(x, int) and not isinstance(x, bool) and x == 0


def _is_one(x) -> bool:
    return isinstance(x, int) and not isinstance(x, bool) and x == 1


class KernelBuilder:
    """Collects the IROps of one kernel; loop and branch bodies are regions."""

    def __init__(self, kernel_name: str):
        self.kernel_name = kernel_name
        self.ops: List[IROp] = []
        self.args: List[tuple] = []          # (name, buffer_index, metal_dtype)
        self.scalar_params: List[tuple] = []
        self._counter = 0
        self._stack: List[List[IROp]] = [self.ops]
        self._consts: Dict[tuple, IRValue] = {}
        self._special: Dict[str, IRValue] = {}

    def new_value(self, dtype: str) -> IRValue:
        v = IRValue(f"_v{self._counter}", dtype)
        self._counter += 1
        return v

    def record(self, op: IROp) -> None:
        self._stack[-1].append(op)

    def _push_region(self) -> List[IROp]:
        region: List[IROp] = []
        self._stack.append(region)
        return region

    def _pop_region(self) -> List[IROp]:
        assert len(self._stack) > 1, "cannot pop the root region"
        self._consts.clear()  # constants are scoped to the region that made them
        return self._stack.pop()

    def make_const(self, dtype: str, value) -> IRValue:
        key = (dtype, value)
        if key not in self._consts:
            v = IRValue(f"_c{value}", dtype)
            self.record(IROp("const", v, [], {"value": value}))
            self._consts[key] = v
        return self._consts[key]

    def _special_value(self, op: str, name: str) -> IRValue:
        if op not in self._special:
            v = IRValue(name, "uint")
            self.record(IROp(op, v, []))
            self._special[op] = v
        return self._special[op]

    def get_thread_position_in_grid(self) -> IRValue:
        return self._special_value("thread_position_in_grid", "tid")

    def get_thread_idx(self) -> IRValue:
        return self._special_value("thread_position_in_threadgroup", "tidx")

    def get_block_idx(self) -> IRValue:
        return self._special_value("threadgroup_position_in_grid", "bidx")

    def get_block_dim(self) -> IRValue:
        return self._special_value("threads_per_threadgroup", "bdim")

    # iteration helpers for the recognizer --------------------------------
    def walk(self):
        """Every op of the trace, depth first (regions after their parent)."""
        stack = list(reversed(self.ops))
        while stack:
            op = stack.pop()
            yield op
            for region in reversed(op.regions):
                stack.extend(reversed(region))

    def __enter__(self):
        _local.builder = self
        return self

    def __exit__(self, *exc):
        _local.builder = None


def _ensure_ir(x) -> IRValue:
    """Python scalars become constants: bool -> i1, int -> uint, float -> float."""
    if isinstance(x, IRValue):
        return x
    b = _require_builder("constant")
    if isinstance(x, bool):
        return b.make_const("i1", int(x))
    if isinstance(x, int):
        return b.make_const("uint", x)
    if isinstance(x, float):
        v = b.new_value("float")  # float constants are not shared
        b.record(IROp("const", v, [], {"value": float(x), "dtype": "float"}))
        return v
    raise TypeError(f"Cannot convert {type(x).__name__} to IRValue")


def _emit(op: str, operands: Sequence, dtype: str, attrs: Optional[dict] = None) -> IRValue:
    b = _require_builder(op)
    res = b.new_value(dtype)
    b.record(IROp(op, res, list(operands), dict(attrs or {})))
    return res


def _binop(op: str, a, b) -> IRValue:
    a, b = _ensure_ir(a), _ensure_ir(b)
    return _emit(op, [a, b], a.dtype)


def _arith(op: str, a, b) -> IRValue:
    """Binary arithmetic; if either side is a per-thread TV vector the op is
    element-wise over it ("tv_<op>") and the result keeps its runs."""
    a, b = _ensure_ir(a), _ensure_ir(b)
    groups = a._tv_groups if a._tv_groups is not None else b._tv_groups
    if groups is None:
        return _emit(op, [a, b], a.dtype)
    dtype = a.dtype if a._tv_groups is not None else b.dtype
    res = _emit("tv_" + op, [a, b], dtype)
    res._tv_groups = groups
    return res


def _unary(op: str, x, result_dtype: Optional[str] = None) -> IRValue:
    x = _ensure_ir(x)
    res = _emit(op, [x], result_dtype or x.dtype)
    res._tv_groups = x._tv_groups
    return res


def _ternary(op: str, a, b, c, result_dtype: Optional[str] = None) -> IRValue:
    a, b, c = _ensure_ir(a), _ensure_ir(b), _ensure_ir(c)
    return _emit(op, [a, b, c], result_dtype or a.dtype)


# ----------------------------------------------------------------------------- intrinsic tables
_UNARY = ("sqrt abs ceil floor round trunc sign saturate fract rsqrt exp exp2 log log2 log10 "
          "sin cos tan asin acos atan sinh cosh tanh popcount clz ctz reverse_bits "
          "abs_diff_unary").split()
_PREDICATES = "isnan isinf isfinite signbit isnormal".split()
_BINARY = ("fmin fmax pow fmod atan2 step copysign imin imax abs_diff add_sat sub_sat mul_hi "
           "rotate").split()
_TERNARY = "clamp fma mix smoothstep iclamp mad_sat".split()
_REDUCTIONS = ["simd_" + n for n in ("sum product min max and or xor prefix_exclusive_sum "
                                     "prefix_inclusive_sum prefix_exclusive_product "
                                     "prefix_inclusive_product").split()]
_REDUCTIONS += ["quad_" + n for n in ("sum product min max and or xor prefix_exclusive_sum "
                                      "prefix_inclusive_sum").split()]
_SHUFFLES = [p + n for p in ("simd_", "quad_")
             for n in ("shuffle", "shuffle_up", "shuffle_down", "shuffle_xor", "broadcast")]
_COMPARES = "eq ne lt le gt ge ult ule ugt uge".split()
_GRID_XYZ = ("thread_position_in_grid_xyz thread_position_in_threadgroup "
             "threadgroup_position_in_grid threads_per_threadgroup threads_per_grid "
             "threadgroups_per_grid grid_size").split()
_GRID_SCALAR = ("thread_index_in_threadgroup thread_index_in_simdgroup "
                "simdgroup_index_in_threadgroup threads_per_simdgroup "
                "simdgroups_per_threadgroup").split()

_g = globals()
for _n in _UNARY + _REDUCTIONS:
    _g[_n] = (lambda op: lambda x: _unary(op, x))(_n)
for _n in _PREDICATES:
    _g[_n] = (lambda op: lambda x: _unary(op, x, "i1"))(_n)
for _n in _BINARY:
    _g[_n] = (lambda op: lambda a, b: _binop(op, a, b))(_n)
for _n in _TERNARY:
    _g[_n] = (lambda op: lambda a, b, c: _ternary(op, a, b, c))(_n)
for _n in _SHUFFLES:
    _g[_n] = (lambda op: lambda value, lane: _emit(op, [_ensure_ir(value), _ensure_ir(lane)],
                                                   _ensure_ir(value).dtype))(_n)
for _n in _COMPARES:
    _g["cmp_" + _n] = (lambda op: lambda a, b: _emit(op, [_ensure_ir(a), _ensure_ir(b)],
                                                     "i1"))("cmp_" + _n)
for _n in _GRID_XYZ:
    _g[_n] = (lambda op: lambda dim="x": _emit(op, [], "uint", {"dim": dim}))(
        "thread_position_in_grid" if _n == "thread_position_in_grid_xyz" else _n)
for _n in _GRID_SCALAR:
    _g[_n] = (lambda op: lambda: _emit(op, [], "uint"))(_n)
del _g, _n


def select(false_val, true_val, condition) -> IRValue:
    """condition ? true_val : false_val (exported as enigma.where)."""
    f, t = _ensure_ir(false_val), _ensure_ir(true_val)
    return _emit("select", [f, t, _ensure_ir(condition)], t.dtype)


def extract_bits(value, offset: int, bits: int) -> IRValue:
    v = _ensure_ir(value)
    return _emit("extract_bits", [v], v.dtype, {"offset": offset, "bits": bits})


def insert_bits(base, insert, offset: int, bits: int) -> IRValue:
    b = _ensure_ir(base)
    return _emit("insert_bits", [b, _ensure_ir(insert)], b.dtype, {"offset": offset, "bits": bits})


def function_constant(dtype: str, index: int) -> IRValue:
    return _emit("function_constant", [], dtype, {"index": int(index)})


def metal_cast(x, dtype: str) -> IRValue:
    """Convert a value (or Python scalar) to `dtype`.  A Python scalar becomes a
    constant of that dtype, so the recognizer can read shape constants back."""
    if not isinstance(x, IRValue):
        b = _require_builder("metal_cast")
        if dtype in ("float", "half", "bfloat", "f32", "f16", "bf16"):
            v = b.new_value(dtype)
            b.record(IROp("const", v, [], {"value": float(x), "dtype": dtype}))
            return v
        return b.make_const(dtype, int(x))
    res = _emit("cast", [x], dtype)
    res._tv_groups = x._tv_groups
    return res


def as_type(x, dtype: str) -> IRValue:
    return _emit("bitcast", [_ensure_ir(x)], dtype)


def make_vec(*elems, dtype: Optional[str] = None) -> IRValue:
    vals = [_ensure_ir(e) for e in elems]
    base = dtype or vals[0].dtype
    return _emit("make_vec", vals, f"{base}{len(vals)}")


def make_float2(a, b):
    return make_vec(a, b, dtype="float")


def make_float3(a, b, c):
    return make_vec(a, b, c, dtype="float")


def make_float4(a, b, c, d):
    return make_vec(a, b, c, d, dtype="float")


def _scalar_of(dtype: str) -> str:
    return dtype.rstrip("0123456789") or dtype


def vec_extract(v, i: int) -> IRValue:
    v = _ensure_ir(v)
    return _emit("vec_extract", [v], _scalar_of(v.dtype), {"index": int(i)})


def dot(a, b) -> IRValue:
    a = _ensure_ir(a)
    return _emit("dot", [a, _ensure_ir(b)], _scalar_of(a.dtype))


def length(a):
    a = _ensure_ir(a)
    return _emit("length", [a], _scalar_of(a.dtype))


def distance(a, b):
    a = _ensure_ir(a)
    return _emit("distance", [a, _ensure_ir(b)], _scalar_of(a.dtype))


def cross(a, b):
    return _binop("cross", a, b)


def normalize(a):
    return _unary("normalize", a)


def reflect(i, n):
    return _binop("reflect", i, n)


def refract(i, n, eta):
    return _ternary("refract", i, n, eta)


def faceforward(n, i, nref):
    return _ternary("faceforward", n, i, nref)


def matmul(a, b, result_dtype: Optional[str] = None):
    a = _ensure_ir(a)
    return _emit("matmul", [a, _ensure_ir(b)], result_dtype or a.dtype)


def transpose(m, result_dtype: Optional[str] = None):
    m = _ensure_ir(m)
    return _emit("transpose", [m], result_dtype or m.dtype)


def determinant(m, scalar_dtype: Optional[str] = None):
    m = _ensure_ir(m)
    return _emit("determinant", [m], scalar_dtype or "float")


_PACKS = ["pack_float_to_" + n for n in
          "snorm4x8 unorm4x8 snorm2x16 unorm2x16 srgb_unorm4x8 unorm10a2".split()]
_UNPACKS = ["unpack_" + n + "_to_float" for n in
            "snorm4x8 unorm4x8 snorm2x16 unorm2x16 srgb_unorm4x8 unorm10a2".split()]
for _n in _PACKS:
    globals()[_n] = (lambda op: lambda v: _emit(op, [_ensure_ir(v)], "uint"))(_n)
for _n in _UNPACKS:
    globals()[_n] = (lambda op: lambda v: _emit(op, [_ensure_ir(v)], "float4"))(_n)
del _n


# ----------------------------------------------------------------------------- memory
def record_load(t: Tensor, index) -> IRValue:
    return _emit("load", [_ensure_ir(index)], t.metal_dtype, t._attrs())


def record_store(t: Tensor, index, value) -> None:
    _require_builder("store").record(
        IROp("store", None, [_ensure_ir(index), _ensure_ir(value)], t._attrs()))


def _vec_dtype(dtype: str, n: int) -> str:
    return f"{dtype}{n}"


def record_tv_load(t: Tensor, runs, n_elem: int) -> IRValue:
    total = sum(c for _, c in runs)
    vector = len(runs) == 1 and total in (2, 3, 4) and runs[0][0] % total == 0
    res = _emit("tv_load", [], _vec_dtype(t.metal_dtype, total) if vector else t.metal_dtype,
                {"buffer": t.name, "buffer_index": t.buffer_index, "base_offset": t.base_offset,
                 "groups": list(runs), "dtype": t.metal_dtype, "num_elements": n_elem})
    res._tv_groups = list(runs)
    return res


def record_tv_store(t: Tensor, value, runs, n_elem: int) -> None:
    _require_builder("store").record(IROp(
        "tv_store", None, [_ensure_ir(value)],
        {"buffer": t.name, "buffer_index": t.buffer_index, "base_offset": t.base_offset,
         "groups": list(runs), "dtype": t.metal_dtype, "num_elements": n_elem}))


def record_atomic(kind: str, t: Tensor, index, vals, order) -> Optional[IRValue]:
    ops = [_ensure_ir(index)] + [_ensure_ir(v) for v in vals]
    attrs = dict(t._attrs(), order=order)
    if kind == "atomic_store":
        _require_builder(kind).record(IROp(kind, None, ops, attrs))
        return None
    return _emit(kind, ops, "bool" if kind == "atomic_compare_exchange_weak" else t.metal_dtype,
                 attrs)


def _atomic_fn(kind):
    def fn(buf: Tensor, index, *vals, order="relaxed"):
        return record_atomic(kind, buf, index, vals, order)
    fn.__name__ = kind
    return fn


for _n in ("atomic_load atomic_store atomic_exchange atomic_fetch_add atomic_fetch_sub "
           "atomic_fetch_min atomic_fetch_max atomic_fetch_and atomic_fetch_or atomic_fetch_xor "
           "atomic_compare_exchange_weak").split():
    globals()[_n] = _atomic_fn(_n)
del _n

_shared_counter = 0


def threadgroup_alloc(dtype: str, size: int) -> Tensor:
    """Threadgroup (CUDA: shared) memory of `size` elements, as a Tensor."""
    global _shared_counter
    b = _require_builder("threadgroup_alloc")
    _shared_counter += 1
    name = f"_shared{_shared_counter}"
    b.record(IROp("threadgroup_alloc", None, [], {"buffer": name, "dtype": dtype,
                                                   "size": int(size)}))
    return Tensor(name, -1, dtype, address_space="threadgroup", shape=int(size))


def barrier(flags: str = "mem_threadgroup") -> None:
    _require_builder("barrier").record(IROp("barrier", None, [], {"flags": flags}))


def simd_barrier(flags: str = "mem_threadgroup") -> None:
    _require_builder("simd_barrier").record(IROp("simd_barrier", None, [], {"flags": flags}))


def load_if(buf: Tensor, index, mask, default=0) -> IRValue:
    """buf[index] where mask holds, else default (an unconditional load then a select)."""
    mask = _ensure_ir(mask)
    d = _ensure_ir(default)
    if d.dtype != buf.metal_dtype:
        d = metal_cast(d, buf.metal_dtype)
    return select(d, buf[index], mask)


def store_if(buf: Tensor, index, value, mask) -> None:
    with if_(mask):
        buf[index] = value


# ----------------------------------------------------------------------------- control flow
class Carry:
    """Loop-carried slots of for_range(init=[...]): read/write inside the body;
    after the loop, reads give the loop results."""

    __slots__ = ("_slots", "_closed")

    def __init__(self, initial):
        self._slots = list(initial)
        self._closed = False

    def __len__(self):
        return len(self._slots)

    def __getitem__(self, i):
        return self._slots[i]

    def __setitem__(self, i, value):
        if self._closed:
            raise EnigmaError("Cannot assign to carry[] outside the for_range body")
        self._slots[i] = _ensure_ir(value)

    def _close(self, results):
        self._slots = list(results)
        self._closed = True


class _ForRange:
    def __init__(self, lo, hi, step=1, dtype="int", init=None):
        self.b = _require_builder("for_range")
        self.bounds = [_ensure_ir(lo), _ensure_ir(hi), _ensure_ir(step)]
        self.dtype = dtype
        self.iv = self.b.new_value(dtype)
        self.init = [_ensure_ir(v) for v in (init or [])]
        self.iter_args, self.results = [], []
        for v in self.init:
            a = self.b.new_value(v.dtype)
            a._tv_groups = v._tv_groups
            r = self.b.new_value(v.dtype)
            r._tv_groups = v._tv_groups
            self.iter_args.append(a)
            self.results.append(r)
        self.carry = Carry(self.iter_args) if init is not None else None

    def __enter__(self):
        self.body = self.b._push_region()
        return self.iv if self.carry is None else (self.iv, self.carry)

    def __exit__(self, *exc):
        self.b._pop_region()
        attrs = {"iv": self.iv, "dtype": self.dtype}
        if self.carry is not None:
            attrs.update(iter_args=self.iter_args, yield_vals=list(self.carry._slots),
                         results=self.results)
        self.b.record(IROp("scf_for", None, self.bounds + self.init, attrs, [self.body]))
        if self.carry is not None:
            self.carry._close(self.results)


def for_range(lo, hi, step=1, dtype: str = "int", init=None) -> _ForRange:
    """Traced loop over [lo, hi) by step; with init=[...] yields (iv, carry)."""
    return _ForRange(lo, hi, step, dtype, init)


class _Block:
    """One branch of an if_: a context manager that fills its region."""

    def __init__(self, b, region):
        self.b, self.region, self.used = b, region, False

    def __enter__(self):
        self.used = True
        self.b._stack.append(self.region)
        return self

    def __exit__(self, *exc):
        self.b._pop_region()


class _If:
    def __init__(self, cond):
        self.b = _require_builder("if_")
        self.cond = _ensure_ir(cond)
        self.then_r, self.else_r = [], []

    def __enter__(self):
        self.then_b, self.else_b = _Block(self.b, self.then_r), _Block(self.b, self.else_r)
        self.implicit = self.b._push_region()  # body of a plain `with if_(c):`
        return (self.then_b, self.else_b)

    def __exit__(self, *exc):
        self.b._pop_region()
        then_r = self.then_r if self.then_b.used else self.implicit
        if self.then_b.used and self.implicit:
            then_r = self.implicit + self.then_r
        self.b.record(IROp("scf_if", None, [self.cond], {}, [then_r, self.else_r]))


def if_(condition) -> _If:
    """`with if_(c):` body, or `with if_(c) as (then_b, else_b):` two branches."""
    return _If(condition)


class _While:
    def __init__(self, cond_fn):
        self.b = _require_builder("while_")
        self.cond_fn = cond_fn
        self.before, self.after = [], []

    def __enter__(self):
        self.b._stack.append(self.before)
        self.cond = self.cond_fn()
        self.b._pop_region()
        self.b._stack.append(self.after)
        return self

    def __exit__(self, *exc):
        self.b._pop_region()
        self.b.record(IROp("scf_while", None, [], {"cond_result": self.cond},
                           [self.before, self.after]))


def while_(cond_fn) -> _While:
    return _While(cond_fn)


def _flatten_carry(v, out):
    """Loop-carried leaves of a value: IRValues and Python numbers (lists / tuples are
    walked); returns a rebuild spec, or None for a value passed through unchanged (a Tensor,
    a RegisterTensor, ...)."""
    if isinstance(v, IRValue):
        out.append(v)
        return ("v",)
    if isinstance(v, (bool, int, float)):
        out.append(_ensure_ir(v))
        return ("v",)
    if isinstance(v, (list, tuple)):
        specs = [_flatten_carry(e, out) for e in v]
        if any(sp is None for sp in specs):
            # a container holding something that cannot be carried: carry nothing from it
            del out[len(out) - sum(_count(sp) for sp in specs if sp is not None):]
            return None
        return ("seq", type(v), specs)
    return None


def _count(spec) -> int:
    return 1 if spec[0] == "v" else sum(_count(sp) for sp in spec[2])


def _rebuild(spec, leaves, pos):
    if spec[0] == "v":
        return leaves[pos], pos + 1
    items = []
    for sp in spec[2]:
        it, pos = _rebuild(sp, leaves, pos)
        items.append(it)
    return (items if spec[1] is list else spec[1](items)), pos


def _enigma_carry_loop(lo, hi, step, body, *values):
    """A loop rewritten from `for i in enigma.range(...)` (compiler/loops.py): `body(i,
    *values)` returns the new values; IRValues and numbers (also inside lists / tuples)
    become loop-carried slots of one traced loop, anything else is passed through.
    Returns the values after the loop."""
    leaves: List[IRValue] = []
    specs = [_flatten_carry(v, leaves) for v in values]
    if not leaves:
        with for_range(lo, hi, step) as iv:
            body(iv, *values)
        return values
    with for_range(lo, hi, step, init=leaves) as (iv, carry):
        cur, pos = [], 0
        for v, sp in zip(values, specs):
            if sp is None:
                cur.append(v)
            else:
                r, pos = _rebuild(sp, [carry[i] for i in range(len(leaves))], pos)
                cur.append(r)
        res = body(iv, *cur)
        res = res if isinstance(res, tuple) else (res,)
        new: List[IRValue] = []
        for v, sp in zip(res, specs):
            if sp is not None:
                got = []
                sp2 = _flatten_carry(v, got)
                if sp2 is None or len(got) != _count(sp):
                    raise EnigmaError("enigma.range(): a loop-carried value changed its structure "
                                      "inside the loop")
                new.extend(got)
        for i, v in enumerate(new):
            carry[i] = v
    finals = [carry[i] for i in range(len(leaves))]
    out, pos = [], 0
    for v, sp in zip(values, specs):
        if sp is None:
            out.append(v)
        else:
            r, pos = _rebuild(sp, finals, pos)
            out.append(r)
    return tuple(out)


class _EnigmaRange:
    """`for i in enigma.range(lo, hi, step)`: a traced loop.

    Kernel bodies are rewritten before tracing (compiler/loops.py) so that such loops
    carry the values they rebind (through _enigma_carry_loop).  This generator is what runs
    when a body could not be rewritten (no source): it traces the body once with a symbolic
    induction variable and keeps rebound values by name only.  Outside a trace it is a
    plain range.
    """

    def __call__(self, *args):
        b = get_builder()
        if b is None:
            return range(*[int(a) for a in args])
        lo, hi, step = (0, args[0], 1) if len(args) == 1 else (tuple(args) + (1,))[:3]
        return self._trace(b, _ensure_ir(lo), _ensure_ir(hi), _ensure_ir(step))

    @staticmethod
    def _trace(b, lo, hi, step):
        iv = b.new_value("int")
        body = b._push_region()
        try:
            yield iv
        finally:
            b._pop_region()
            b.record(IROp("scf_for", None, [lo, hi, step], {"iv": iv, "dtype": "int",
                                                             "unrolled_by_python": False},
                          [body]))


class _EnigmaRangeConstexpr:
    """`enigma.range_constexpr(n)`: always unrolled at trace time."""

    def __call__(self, *args):
        return range(*args)


# ----------------------------------------------------------------------------- helpers
def copy(src: Tensor, dst: Tensor, count: int, src_offset=0, dst_offset=0, mask_fn=None,
         coalesced_width: int = 1) -> None:
    """Element copy src -> dst; with coalesced_width > 1 each thread moves a
    strided slice.  Recorded as one op."""
    _require_builder("copy").record(IROp(
        "copy", None, [_ensure_ir(src_offset), _ensure_ir(dst_offset)],
        {"src": src.name, "dst": dst.name, "count": int(count), "masked": mask_fn is not None,
         "coalesced_width": int(coalesced_width)}))


class RegisterTensor:
    """Per-thread register array of a fixed shape (index with ints)."""

    def __init__(self, shape, dtype="float", fill=0.0):
        self.b = _require_builder("register_tensor")
        self.shape = tuple(shape) if isinstance(shape, (tuple, list)) else (shape,)
        self.dtype = dtype
        n = 1
        for s in self.shape:
            n *= s
        init = metal_cast(fill, dtype)
        self._vals = [init] * n

    def _flat(self, idx):
        idx = idx if isinstance(idx, tuple) else (idx,)
        k, mul = 0, 1
        for i, s in reversed(list(zip(idx, self.shape))):
            k += int(i) * mul
            mul *= s
        return k

    def __getitem__(self, idx):
        return self._vals[self._flat(idx)]

    def __setitem__(self, idx, value):
        self._vals[self._flat(idx)] = _ensure_ir(value)

    def size(self):
        return len(self._vals)


def register_tensor(shape, dtype: str = "float", fill=0.0) -> RegisterTensor:
    return RegisterTensor(shape, dtype, fill)


class Pipeline:
    """Multi-stage threadgroup buffer ring (producer/consumer stages)."""

    def __init__(self, dtype: str, stage_size: int, stages: int = 2):
        self.stages = int(stages)
        self.stage_size = int(stage_size)
        self.buffer = threadgroup_alloc(dtype, self.stage_size * self.stages)
        _require_builder("pipeline").record(IROp(
            "pipeline", None, [], {"buffer": self.buffer.name, "stages": self.stages,
                                   "stage_size": self.stage_size}))

    def stage_offset(self, i):
        return (i % self.stages) * self.stage_size if isinstance(i, int) else \
            (_ensure_ir(i) % self.stages) * self.stage_size


def pipeline(dtype: str, stage_size: int, stages: int = 2) -> Pipeline:
    return Pipeline(dtype, stage_size, stages)


def async_copy_to_threadgroup(dst: Tensor, src: Tensor, count: int, dst_offset=0, src_offset=0):
    return _emit("async_copy", [_ensure_ir(dst_offset), _ensure_ir(src_offset)], "event",
                 {"dst": dst.name, "src": src.name, "count": int(count)})


def async_copy_commit():
    _require_builder("async_copy_commit").record(IROp("async_copy_commit", None, []))


def async_copy_wait(*events):
    _require_builder("async_copy_wait").record(IROp("async_copy_wait", None, list(events)))


def _async_2d(kind, dst, dst_off, dst_stride, src, src_off, src_stride, width, height):
    return _emit(kind, [_ensure_ir(dst_off), _ensure_ir(dst_stride), _ensure_ir(src_off),
                        _ensure_ir(src_stride), _ensure_ir(width), _ensure_ir(height)], "event",
                 {"dst": dst.name, "src": src.name})


def async_copy_2d_d2t(dst, dst_off, dst_stride, src, src_off, src_stride, width, height):
    """2-D device -> threadgroup tile copy (rows of `width` elements, `height` rows)."""
    return _async_2d("async_copy_2d_d2t", dst, dst_off, dst_stride, src, src_off, src_stride,
                     width, height)


def async_copy_2d_t2d(dst, dst_off, dst_stride, src, src_off, src_stride, width, height):
    return _async_2d("async_copy_2d_t2d", dst, dst_off, dst_stride, src, src_off, src_stride,
                     width, height)


def async_copy_1d_d2t(dst, dst_off, src, src_off, count):
    return _emit("async_copy_1d_d2t", [_ensure_ir(dst_off), _ensure_ir(src_off),
                                       _ensure_ir(count)], "event", {"dst": dst.name,
                                                                     "src": src.name})


def async_copy_1d_t2d(dst, dst_off, src, src_off, count):
    return _emit("async_copy_1d_t2d", [_ensure_ir(dst_off), _ensure_ir(src_off),
                                       _ensure_ir(count)], "event", {"dst": dst.name,
                                                                     "src": src.name})


def simdgroup_matrix_load(buf: Tensor, elements_per_row: int, elem: str = "float",
                          rows: int = 8, cols: int = 8) -> IRValue:
    """Load an 8x8 (rows x cols) matrix fragment from `buf` (row pitch elements_per_row)."""
    return _emit("simdgroup_matrix_load", [_ensure_ir(elements_per_row)],
                 f"simdgroup_{elem}{rows}x{cols}", {"buffer": buf.name})


def simdgroup_matrix_store(matrix: IRValue, buf: Tensor, elements_per_row: int) -> None:
    _require_builder("simdgroup_matrix_store").record(IROp(
        "simdgroup_matrix_store", None, [matrix, _ensure_ir(elements_per_row)],
        {"buffer": buf.name}))


def simdgroup_multiply_accumulate(a, b, c) -> IRValue:
    return _emit("simdgroup_multiply_accumulate", [a, b, c], c.dtype)


def make_filled_simdgroup_matrix(value, elem: str = "float", rows: int = 8,
                                 cols: int = 8) -> IRValue:
    return _emit("make_filled_simdgroup_matrix", [_ensure_ir(value)],
                 f"simdgroup_{elem}{rows}x{cols}")
