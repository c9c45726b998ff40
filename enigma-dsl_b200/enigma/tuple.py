"""Hierarchical integer tuples (CuTe "IntTuple") — pure host-side math.

Same function names and results as the reference's enigma/tuple.py
(crd2idx :63, idx2crd :79, compact_col_major :91, compact_order :102,
shape_div :137, ...).  The results must agree bit for bit because the
layout algebra built on them decides every offset a kernel touches; the
golden tables under tests/golden/ pin that.
"""
from __future__ import annotations

from typing import Any, Sequence, Tuple, Union

Int = int
Shape = Union[int, Tuple["Shape", ...]]
Stride = Union[int, Tuple["Stride", ...]]
Coord = Union[int, Tuple["Coord", ...]]


def is_int(x: Any) -> bool:
    return isinstance(x, int)


def is_tuple(x: Any) -> bool:
    return isinstance(x, tuple)


def rank(x: Shape) -> int:
    return len(x) if is_tuple(x) else 1


def depth(x: Shape) -> int:
    if not is_tuple(x):
        return 0
    return 1 + max(map(depth, x), default=0)


def flatten(x: Shape) -> Tuple[int, ...]:
    """Leaves of a nested tuple, left to right."""
    out = []
    stack = [x]
    while stack:
        top = stack.pop()
        if is_tuple(top):
            stack.extend(reversed(top))
        else:
            out.append(top)
    return tuple(out)


def product(x: Shape) -> int:
    p = 1
    for v in flatten(x):
        p *= v
    return p


def inner_product(a: Shape, b: Stride) -> int:
    fa, fb = flatten(a), flatten(b)
    assert len(fa) == len(fb)
    return sum(u * v for u, v in zip(fa, fb))


def crd2idx(crd: Coord, shape: Shape, stride: Stride) -> int:
    """Coordinate -> offset.  An integer coordinate against a tuple shape is
    first unfolded colexicographically (mode 0 fastest)."""
    if is_tuple(crd):
        return sum(crd2idx(c, s, d) for c, s, d in zip(crd, shape, stride))
    if is_tuple(shape):
        total, rest = 0, crd
        for s, d in zip(shape, stride):
            n = product(s)
            total += crd2idx(rest % n, s, d)
            rest //= n
        return total
    return crd * stride


def idx2crd(idx: int, shape: Shape) -> Coord:
    """Linear index -> coordinate congruent with `shape` (colexicographic)."""
    if not is_tuple(shape):
        return idx % shape
    out = []
    for s in shape:
        n = product(s)
        out.append(idx2crd(idx % n, s))
        idx //= n
    return tuple(out)


def compact_col_major(shape: Shape, current: int = 1) -> Stride:
    """Strides of the packed column-major layout of `shape` (mode 0 fastest).
    Leaves of extent <= 0 get stride 0."""
    if not is_tuple(shape):
        return current if shape > 0 else 0
    strides = []
    for s in shape:
        strides.append(compact_col_major(s, current))
        current *= product(s)
    return tuple(strides)


def compact_order(shape: Shape, order: Tuple[int, ...]) -> Stride:
    """Packed strides where order[i] ranks mode i (0 = innermost)."""
    n = len(shape) if is_tuple(shape) else 1
    if n == 1:
        return compact_col_major(shape)
    strides = [0] * n
    running = 1
    for dim in sorted(range(n), key=lambda i: order[i]):
        strides[dim] = running
        running *= product(shape[dim])
    return tuple(strides)


def prefix_product(shape: Shape, init: int = 1) -> Tuple[int, ...]:
    out, cur = [], init
    for s in flatten(shape):
        out.append(cur)
        cur *= s
    return tuple(out)


def ceil_div(a: int, b: int) -> int:
    return -(-a // b)


def gcd(a: int, b: int) -> int:
    while b:
        a, b = b, a % b
    return a


def shape_div(a: int, b: int) -> int:
    """CuTe shape division: a / b when b divides, at least 1 otherwise."""
    if b == 1:
        return a
    if a < b:
        return 1
    return max(1, a // b)


def elem_scale(a: Shape, b: Shape) -> Shape:
    if is_int(a) and is_int(b):
        return a * b
    if is_int(a):
        return tuple(elem_scale(a, v) for v in b)
    if is_int(b):
        return tuple(elem_scale(u, b) for u in a)
    return tuple(elem_scale(u, v) for u, v in zip(a, b))


def select(x: Shape, mode: Union[int, Sequence[int]]) -> Shape:
    if isinstance(mode, (list, tuple)):
        return tuple(x[m] for m in mode)
    return x[mode]


def repeat_like(val: Any, ref: Shape) -> Shape:
    if not is_tuple(ref):
        return val
    return tuple(repeat_like(val, r) for r in ref)


def is_congruent(a: Shape, b: Shape) -> bool:
    if is_int(a) and is_int(b):
        return a == b
    if is_tuple(a) and is_tuple(b) and len(a) == len(b):
        return all(map(is_congruent, a, b))
    return False


def is_compatible(a: Shape, b: Shape) -> bool:
    return product(a) == product(b)
