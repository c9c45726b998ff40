"""Tensor = named kernel buffer + Layout + base offset.

At @jit time a Tensor is pure layout algebra (zipped_divide, composition
with a TV layout).  Inside an @enigma.kernel trace, indexing with a runtime
value records index arithmetic, and load()/store() record one vectorised
access of all the view's elements, grouped into contiguous runs.  Those runs
are what the recognizer reads to learn each thread's vector width.

Behaviour follows the reference's enigma/tensor.py: slicing (:61-124),
run grouping (_group_contiguous :368-380), vector promotion of a single
aligned run of 2-4 elements (:151-156), tensor_composition (:252-277) and
the oversize-tiler error of tensor_zipped_divide (:280-317).
"""
from __future__ import annotations

from typing import Any, List, Tuple

from .core import Layout
from .core import zipped_divide as _zipped_divide
from .tuple import flatten, idx2crd, is_int, is_tuple, product


class Tensor:
    def __init__(self, name: str, buffer_index: int, metal_dtype: str,
                 layout: "Layout | None" = None, base_offset: Any = 0,
                 address_space: str = "device", shape: "int | None" = None):
        self.name = name
        self.buffer_index = buffer_index
        self.metal_dtype = metal_dtype
        self.layout = layout
        self.base_offset = base_offset
        self.address_space = address_space
        self._static_shape = shape

    shape = property(lambda self: self.layout.shape)
    stride = property(lambda self: self.layout.stride)
    element_type = property(lambda self: self.metal_dtype)

    def size(self, mode=None):
        if self.layout is None:
            return self._static_shape or 0
        return self.layout.size(mode)

    def _attrs(self):
        return {"buffer": self.name, "buffer_index": self.buffer_index,
                "address_space": self.address_space, "dtype": self.metal_dtype,
                "shape": self._static_shape}

    # ------------------------------------------------------------------ indexing
    def __getitem__(self, coord):
        from . import _tracing as tr

        if not isinstance(coord, tuple):
            if isinstance(coord, (tr.IRValue, int)):
                return tr.record_load(self, coord)
            coord = (coord,)
        if self.layout is None:
            raise TypeError("Layout algebra requires a Layout on the Tensor")
        shapes = self.layout.shape if is_tuple(self.layout.shape) else (self.layout.shape,)
        strides = self.layout.stride if is_tuple(self.layout.stride) else (self.layout.stride,)
        offset = self.base_offset
        keep_s, keep_d = [], []
        for c, s, d in zip(coord, shapes, strides):
            if c is None:
                keep_s.append(s)
                keep_d.append(d)
            elif is_tuple(c) and is_tuple(s):
                sub_s, sub_d = [], []
                for j, cc in enumerate(c):
                    ss, dd = s[j], (d[j] if is_tuple(d) else d)
                    if cc is None:
                        sub_s.append(ss)
                        sub_d.append(dd)
                    else:
                        offset = _offset_add(offset, cc, ss, dd)
                if sub_s:
                    keep_s.append(sub_s[0] if len(sub_s) == 1 else tuple(sub_s))
                    keep_d.append(sub_d[0] if len(sub_d) == 1 else tuple(sub_d))
            else:
                offset = _offset_add(offset, c, s, d)
        if not keep_s:
            return offset
        lay = Layout(keep_s[0] if len(keep_s) == 1 else tuple(keep_s),
                     keep_d[0] if len(keep_d) == 1 else tuple(keep_d))
        return Tensor(self.name, self.buffer_index, self.metal_dtype, lay, base_offset=offset,
                      address_space=self.address_space)

    def __setitem__(self, coord, value):
        from . import _tracing as tr

        if isinstance(coord, tuple) and len(coord) == 1:
            coord = coord[0]
        if isinstance(coord, (tr.IRValue, int)):
            tr.record_store(self, coord, value)
            return
        raise TypeError("Use .store() for TV-layout kernels")

    # ------------------------------------------------------------------ vector access
    def value_runs(self) -> List[Tuple[int, int]]:
        """Contiguous (start, length) runs of this view's element offsets."""
        fs, fd = flatten(self.layout.shape), flatten(self.layout.stride)
        return _group_contiguous(_compute_value_offsets(fs, fd, product(self.layout.shape)))

    def load(self):
        from . import _tracing as tr
        return tr.record_tv_load(self, self.value_runs(), product(self.layout.shape))

    def store(self, value):
        from . import _tracing as tr
        tr.record_tv_store(self, value, self.value_runs(), product(self.layout.shape))

    def __repr__(self):
        return f"Tensor({self.name}, layout={self.layout}, offset={self.base_offset})"

    # ------------------------------------------------------------------ atomics
    def _atomic(self, kind, index, *vals, order="relaxed"):
        from . import _tracing as tr
        return tr.record_atomic(kind, self, index, vals, order)

    def atomic_load(self, index, order="relaxed"):
        return self._atomic("atomic_load", index, order=order)

    def atomic_store(self, index, value, order="relaxed"):
        self._atomic("atomic_store", index, value, order=order)

    def atomic_exchange(self, index, value, order="relaxed"):
        return self._atomic("atomic_exchange", index, value, order=order)

    def atomic_fetch_add(self, index, value, order="relaxed"):
        return self._atomic("atomic_fetch_add", index, value, order=order)

    def atomic_fetch_sub(self, index, value, order="relaxed"):
        return self._atomic("atomic_fetch_sub", index, value, order=order)

    def atomic_fetch_min(self, index, value, order="relaxed"):
        return self._atomic("atomic_fetch_min", index, value, order=order)

    def atomic_fetch_max(self, index, value, order="relaxed"):
        return self._atomic("atomic_fetch_max", index, value, order=order)

    def atomic_fetch_and(self, index, value, order="relaxed"):
        return self._atomic("atomic_fetch_and", index, value, order=order)

    def atomic_fetch_or(self, index, value, order="relaxed"):
        return self._atomic("atomic_fetch_or", index, value, order=order)

    def atomic_fetch_xor(self, index, value, order="relaxed"):
        return self._atomic("atomic_fetch_xor", index, value, order=order)

    def atomic_compare_exchange_weak(self, index, expected, desired,
                                     success_order="relaxed", failure_order="relaxed"):
        return self._atomic("atomic_compare_exchange_weak", index, expected, desired,
                            order=(success_order, failure_order))


def tensor_composition(tensor: Tensor, tv_layout: Layout, tiler) -> Tensor:
    """Per-thread view: the TV layout's tile-linear strides become memory strides.

    A tile-linear stride k is unfolded to a coordinate of the tiler (mode 0
    fastest) and mapped through the tensor's own mode strides.
    """
    mode_d = tensor.layout.stride if is_tuple(tensor.layout.stride) else (tensor.layout.stride,)
    tshape = tiler if is_tuple(tiler) else (tiler,)

    def to_memory(k):
        if not is_int(k):
            return tuple(to_memory(e) for e in k)
        crd = idx2crd(k, tshape)
        if is_tuple(crd):
            return sum(c * d for c, d in zip(crd, mode_d))
        return crd * mode_d[0]

    lay = Layout(tv_layout.shape, (to_memory(tv_layout.stride[0]), to_memory(tv_layout.stride[1])))
    return Tensor(tensor.name, tensor.buffer_index, tensor.metal_dtype, lay,
                  base_offset=tensor.base_offset)


def tensor_zipped_divide(tensor: Tensor, tiler) -> Tensor:
    """zipped_divide of the tensor's layout; a tile larger than the tensor in
    any mode is an error (it would silently produce an empty grid)."""
    from ._tracing import EnigmaError

    tshape = tensor.layout.shape if is_tuple(tensor.layout.shape) else (tensor.layout.shape,)
    if isinstance(tiler, Layout):
        tl = tiler.shape if is_tuple(tiler.shape) else (tiler.shape,)
    elif isinstance(tiler, (int, tuple)):
        tl = tiler if is_tuple(tiler) else (tiler,)
    else:
        tl = (tiler,)
    for i, (have, want) in enumerate(zip(tshape, tl)):
        if product(have) < product(want):
            raise EnigmaError(
                f"Tiler shape exceeds tensor shape in mode {i}: tensor has {product(have)} "
                f"elements but tiler requires {product(want)}. The tile must fit within the "
                f"tensor in every dimension.")
    return Tensor(tensor.name, tensor.buffer_index, tensor.metal_dtype,
                  _zipped_divide(tensor.layout, tiler), base_offset=tensor.base_offset)


def make_identity_tensor(shape) -> Tensor:
    return Tensor("__identity__", -1, "uint", Layout(shape))


# ----------------------------------------------------------------------------- helpers
def _offset_add(base, idx, shape, stride):
    """base + offset of coordinate `idx` in mode (shape : stride).

    A Python int is folded now; a traced value records index arithmetic
    (component = idx % s, idx //= s per leaf) in the current kernel trace.
    """
    if is_int(idx):
        if is_tuple(shape):
            crd = idx2crd(idx, shape)
            leaves = flatten((crd,) if is_int(crd) else crd)
            return base + sum(c * d for c, d in zip(leaves, flatten(stride)))
        return base + idx * stride
    fs = flatten(shape) if is_tuple(shape) else (shape,)
    fd = flatten(stride) if is_tuple(stride) else (stride,)
    acc, rest = None, idx
    for s, d in zip(fs, fd):
        if len(fs) > 1:
            comp, rest = rest % s, rest // s
        else:
            comp = rest
        term = comp * d
        acc = term if acc is None else acc + term
    if acc is None:
        return base
    if is_int(base) and base == 0:
        return acc
    return base + acc


def _compute_value_offsets(flat_shape, flat_stride, n_elem):
    out = []
    for v in range(n_elem):
        off, rest = 0, v
        for s, d in zip(flat_shape, flat_stride):
            off += (rest % s) * d
            rest //= s
        out.append(off)
    return out


def _group_contiguous(offsets):
    """[(start, count)] runs of consecutive offsets, in order."""
    runs: List[List[int]] = []
    for o in offsets:
        if runs and o == runs[-1][0] + runs[-1][1]:
            runs[-1][1] += 1
        else:
            runs.append([o, 1])
    return [(s, c) for s, c in runs]
