"""Layout algebra: Layout = (Shape, Stride), coordinate -> offset.

Host-side only.  It decides the thread x value partition (make_layout_tv),
the tile split (zipped_divide) and therefore the vector width of every
per-thread load the recognizer hands to the CUDA kernels.

The operations keep the reference's exact semantics (enigma/core.py), which
differ from upstream CuTe in places that matter for bit-exact tables:
  * coalesce drops size-1 modes and sorts the rest by (stride, shape) before
    merging (core.py:283-309), so its result is stride-ordered;
  * complement / composition work on that sorted form (core.py:312-417);
  * zipped_divide is per-mode and purely arithmetic (core.py:452-478);
  * make_layout_tv orders thread and value modes by their smallest stride
    (core.py:537-575).
tests/golden/layout_tables.json (generated from the reference itself by
tests/golden/make_golden.py) pins every one of them.
"""
from __future__ import annotations

from typing import List, Tuple

from .tuple import (Coord, Shape, Stride, ceil_div, compact_col_major, compact_order, crd2idx,
                    depth, flatten, gcd, is_int, is_tuple, product)
from .tuple import rank as _rank


class Swizzle:
    """XOR swizzle Swizzle<B, M, S>: offset ^= (offset >> S) & (((1 << B) - 1) << M)."""

    __slots__ = ("bits", "base", "shift")

    def __init__(self, bits: int, base: int, shift: int):
        for name, v in (("bits", bits), ("base", base), ("shift", shift)):
            if v < 0:
                raise ValueError(f"Swizzle {name} must be non-negative, got {v}")
        self.bits, self.base, self.shift = bits, base, shift

    def __call__(self, offset: int) -> int:
        if self.bits == 0:
            return offset
        mask = ((1 << self.bits) - 1) << self.base
        return offset ^ ((offset >> self.shift) & mask)

    def __repr__(self):
        return f"Swizzle(bits={self.bits}, base={self.base}, shift={self.shift})"

    def __eq__(self, other):
        if not isinstance(other, Swizzle):
            return NotImplemented
        return (self.bits, self.base, self.shift) == (other.bits, other.base, other.shift)


class Layout:
    """(Shape, Stride); default stride is packed column-major."""

    __slots__ = ("shape", "stride")

    def __init__(self, shape: Shape, stride: Stride = None):
        self.shape = shape
        self.stride = compact_col_major(shape) if stride is None else stride

    def __call__(self, coord: Coord) -> int:
        return crd2idx(coord, self.shape, self.stride)

    def size(self, mode=None) -> int:
        return product(_select_mode(self.shape, mode))

    def rank(self) -> int:
        return _rank(self.shape)

    def depth(self) -> int:
        return depth(self.shape)

    def cosize(self) -> int:
        """1 + the largest offset (0 for an empty layout); zero or negative strides add nothing."""
        if self.size() == 0:
            return 0
        top = sum((s - 1) * d for s, d in zip(flatten(self.shape), flatten(self.stride))
                  if s > 0 and d > 0)
        return top + 1

    def __repr__(self):
        return f"{_fmt(self.shape)}:{_fmt(self.stride)}"

    def __eq__(self, other):
        if not isinstance(other, Layout):
            return NotImplemented
        return self.shape == other.shape and self.stride == other.stride

    def __hash__(self):
        return hash((self.shape, self.stride))


class SwizzledLayout:
    """A Layout followed by a Swizzle of its offsets (shared-memory tiles)."""

    __slots__ = ("layout", "swizzle")

    def __init__(self, layout: Layout, swizzle: Swizzle):
        self.layout, self.swizzle = layout, swizzle

    def __call__(self, coord) -> int:
        return self.swizzle(self.layout(coord))

    shape = property(lambda self: self.layout.shape)
    stride = property(lambda self: self.layout.stride)

    def size(self, mode=None) -> int:
        return self.layout.size(mode)

    def rank(self) -> int:
        return self.layout.rank()

    def depth(self) -> int:
        return self.layout.depth()

    def cosize(self) -> int:
        return self.layout.cosize()

    def __repr__(self):
        return f"SwizzledLayout({self.layout!r}, {self.swizzle!r})"

    def __eq__(self, other):
        if not isinstance(other, SwizzledLayout):
            return NotImplemented
        return self.layout == other.layout and self.swizzle == other.swizzle


def swizzle(layout: Layout, bits: int, base: int, shift: int) -> SwizzledLayout:
    return SwizzledLayout(layout, Swizzle(bits, base, shift))


def _fmt(x) -> str:
    return str(x) if is_int(x) else "(" + ",".join(map(_fmt, x)) + ")"


def _select_mode(shape, mode):
    if mode is None:
        return shape
    for m in (mode if isinstance(mode, (list, tuple)) else (mode,)):
        if is_tuple(shape):
            shape = shape[m]
    return shape


def _as_layout(shapes: List[int], strides: List[int]) -> Layout:
    """1 leaf -> scalar layout, several -> flat tuple layout."""
    if len(shapes) == 1:
        return Layout(shapes[0], strides[0])
    return Layout(tuple(shapes), tuple(strides))


def _modes(x) -> tuple:
    return x if is_tuple(x) else (x,)


# ----------------------------------------------------------------------------- constructors
def make_layout(shape: Shape, stride: Stride = None) -> Layout:
    return Layout(shape, stride)


def make_ordered_layout(shape: Shape, order: Tuple[int, ...]) -> Layout:
    return Layout(shape, compact_order(shape, order))


def make_identity_layout(shape: Shape) -> Layout:
    return Layout(shape, compact_col_major(shape))


def size(x, mode=None) -> int:
    """Size of a Layout, a Tensor (anything with .layout) or a plain shape."""
    if isinstance(x, Layout) or hasattr(x, "layout"):
        return x.size(mode)
    return product(_select_mode(x, mode))


def cosize(x: Layout) -> int:
    return x.cosize()


# ----------------------------------------------------------------------------- coalesce
def coalesce(layout: Layout) -> Layout:
    """Drop size-1 leaves, order by (stride, shape), merge packed neighbours."""
    leaves = sorted(((s, d) for s, d in zip(flatten(layout.shape), flatten(layout.stride))
                     if s != 1), key=lambda sd: (sd[1], sd[0]))
    if not leaves:
        return Layout(1, 0)
    shapes, strides = [leaves[0][0]], [leaves[0][1]]
    for s, d in leaves[1:]:
        if d == strides[-1] * shapes[-1]:
            shapes[-1] *= s
        else:
            shapes.append(s)
            strides.append(d)
    return _as_layout(shapes, strides)


# ----------------------------------------------------------------------------- complement
def complement(layout: Layout, cosize_val: int = None) -> Layout:
    """Layout enumerating the offsets in [0, cosize_val) that `layout` skips."""
    c = coalesce(layout)
    if cosize_val is None:
        cosize_val = c.cosize()
    holes_s, holes_d = [], []
    covered = 1
    for d, s in sorted(((d, s) for d, s in zip(flatten(c.stride), flatten(c.shape)) if d != 0),
                       key=lambda ds: ds[0]):
        if d > covered:
            holes_s.append(d // covered)
            holes_d.append(covered)
        covered = d * s
    if covered < cosize_val:
        holes_s.append(ceil_div(cosize_val, covered))
        holes_d.append(covered)
    if not holes_s:
        return Layout(1, cosize_val)
    return _as_layout(holes_s, holes_d)


# ----------------------------------------------------------------------------- composition
def composition(a, b) -> Layout:
    """(a o b)(c) = a(b(c)), computed mode by mode of b against coalesce(a)."""
    if not (isinstance(a, Layout) and isinstance(b, Layout)):
        raise TypeError(
            f"composition not implemented for ({type(a).__name__}, {type(b).__name__})")
    ac = coalesce(a)
    if is_tuple(b.shape) and is_tuple(b.stride):
        parts = [_compose_mode(ac, s, d) for s, d in zip(b.shape, b.stride)]
        return Layout(tuple(p[0] for p in parts), tuple(p[1] for p in parts))
    return Layout(*_compose_mode(ac, b.shape, b.stride))


def _compose_mode(a: Layout, bs: Shape, bd: Stride):
    """Compose coalesced `a` with the single mode (bs : bd) of b.

    Walks a's leaves; for each leaf the number of b-steps it can absorb
    depends on whether b's stride is a multiple of the leaf stride, the
    leaf stride a multiple of b's stride, or neither (gcd split).  This is
    the reference's rule (core.py:366-417) and is kept step for step so the
    resulting tables are identical.
    """
    if is_tuple(bs):
        parts = [_compose_mode(a, s, d) for s, d in zip(bs, bd)]
        return tuple(p[0] for p in parts), tuple(p[1] for p in parts)
    if bd == 0:
        return bs, 0
    out_s, out_d = [], []
    left = bs
    for sa, da in zip(flatten(a.shape), flatten(a.stride)):
        if left <= 1:
            break
        if da == 0:
            continue
        if bd % da == 0:
            scale = bd // da
            n = min(left, ceil_div(sa, scale) if scale > 0 else sa)
            step = da * scale
        elif da % bd == 0:
            n = min(left, da // bd)
            step = bd
        else:
            g = gcd(da, bd)
            n = min(left, da // g)
            step = g
        if n > 1:
            out_s.append(n)
            out_d.append(step)
        left = ceil_div(left, max(n, 1))
    if not out_s:
        return 1, 0
    if len(out_s) == 1:
        return out_s[0], out_d[0]
    return tuple(out_s), tuple(out_d)


# ----------------------------------------------------------------------------- inverses
def right_inverse(layout: Layout) -> Layout:
    c = coalesce(layout)
    fs, fd = list(flatten(c.shape)), list(flatten(c.stride))
    inv_s, inv_d = [0] * len(fs), [0] * len(fs)
    running = 1
    for i in sorted(range(len(fd)), key=lambda k: fd[k]):
        inv_s[i], inv_d[i] = fs[i], running
        running *= fs[i]
    return _as_layout(inv_s, inv_d)


def left_inverse(layout: Layout) -> Layout:
    return right_inverse(make_layout(layout.shape, layout.stride))


# ----------------------------------------------------------------------------- divide
def _tiler_layout(tiler) -> Layout:
    return tiler if isinstance(tiler, Layout) else Layout(tiler)


def logical_divide(layout: Layout, tiler) -> Layout:
    """((tile), (rest)): compose `layout` with tiler ++ complement(tiler, size)."""
    t = _tiler_layout(tiler)
    rest = complement(t, size(layout))
    return composition(layout, Layout((t.shape, rest.shape), (t.stride, rest.stride)))


def zipped_divide(layout: Layout, tiler) -> Layout:
    """Per-mode split into ((tile modes), (rest modes)); missing tiler modes are 1."""
    if isinstance(tiler, Layout):
        tshape = _modes(tiler.shape)
    elif isinstance(tiler, (int, tuple)):
        tshape = _modes(tiler)
    else:
        tshape = (tiler,)
    shapes, strides = _modes(layout.shape), _modes(layout.stride)
    tile_s, tile_d, rest_s, rest_d = [], [], [], []
    for i, (s, d) in enumerate(zip(shapes, strides)):
        t = tshape[i] if i < len(tshape) else 1
        n = product(t)
        tile_s.append(t)
        tile_d.append(d)
        rest_s.append(product(s) // n)
        rest_d.append(d * n)
    if len(tile_s) == 1:
        return Layout((tile_s[0], rest_s[0]), (tile_d[0], rest_d[0]))
    return Layout((tuple(tile_s), tuple(rest_s)), (tuple(tile_d), tuple(rest_d)))


# ----------------------------------------------------------------------------- product
def blocked_product(a: Layout, b: Layout) -> Layout:
    """a repeated at every element of b, b's strides scaled by cosize(a)."""
    span = a.cosize()
    shapes = flatten(a.shape) + flatten(b.shape)
    strides = flatten(a.stride) + tuple(d * span for d in flatten(b.stride))
    return _as_layout(list(shapes), list(strides))


# ----------------------------------------------------------------------------- recast
def recast_layout(new_bits: int, old_bits: int, layout: Layout) -> Layout:
    """Re-express `layout` in elements of new_bits (e.g. 4 fp32 -> 1 128-bit).

    The first unit-stride leaf of extent > 1 shrinks by the ratio and every
    stride > 1 is divided by it.
    """
    if new_bits == old_bits:
        return layout
    ratio = new_bits // old_bits
    fs, fd = list(flatten(layout.shape)), list(flatten(layout.stride))
    for i in range(len(fd)):
        if fd[i] == 1 and fs[i] > 1:
            fs[i] //= ratio
            fd = [d // ratio if d > 1 else d for d in fd]
            break
    return Layout(_refold(layout.shape, iter(fs)), _refold(layout.shape, iter(fd)))


def _refold(ref: Shape, leaves):
    """Rebuild the nesting of `ref` from a flat iterator of leaves."""
    if is_int(ref):
        return next(leaves)
    return tuple(_refold(r, leaves) for r in ref)


# ----------------------------------------------------------------------------- TV layout
def make_layout_tv(thr_layout: Layout, val_layout: Layout) -> Tuple[Shape, Layout]:
    """Thread-value layout: (tiler, tv) where tv((t, v)) is the column-major
    offset inside the tile of value v of thread t.

    Per mode i the tile extent is |thr_i| * |val_i|.  Thread modes (and value
    modes) are listed in order of their smallest stride; a thread step in
    mode i advances |val_i| elements of that mode, a value step one element.
    """
    ts, td = _modes(thr_layout.shape), _modes(thr_layout.stride)
    vs, vd = _modes(val_layout.shape), _modes(val_layout.stride)
    n = len(ts)
    assert len(vs) == n
    tiler = tuple(product(ts[i]) * product(vs[i]) for i in range(n))
    mode_stride, acc = [], 1
    for extent in tiler:
        mode_stride.append(acc)
        acc *= extent

    def by_stride(strides):
        key = [s if is_int(s) else min(flatten(s)) for s in strides]
        return sorted(range(n), key=lambda i: key[i])

    to, vo = by_stride(td), by_stride(vd)
    tv = Layout(
        (tuple(ts[i] for i in to), tuple(vs[i] for i in vo)),
        (tuple(product(vs[i]) * mode_stride[i] for i in to), tuple(mode_stride[i] for i in vo)),
    )
    return tiler, tv
