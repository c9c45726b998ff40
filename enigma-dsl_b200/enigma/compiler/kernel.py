"""@enigma.kernel / @enigma.jit and tracing entry points.

Same surface as the reference's enigma/compiler/kernel.py: a @jit host
function runs layout algebra and calls `kernel(...).launch(grid=, block=)`,
which traces the kernel (:80-102); an annotated kernel compiled on its own
is traced with one proxy per parameter, Scalar parameters becoming a load
of a one-element buffer (:115-154).
"""
from __future__ import annotations

import inspect
import threading
from typing import Callable, Optional, Tuple

from .._tracing import IROp, KernelBuilder
from ..tensor import Tensor
from ..typing import Numeric, Scalar

_jit_local = threading.local()


class _JitContext:
    """Receives the trace and launch configuration of one @jit run."""

    def __init__(self):
        self.builder: Optional[KernelBuilder] = None
        self.grid: Optional[Tuple[int, ...]] = None
        self.block: Optional[Tuple[int, ...]] = None
        self.args: tuple = ()

    def __enter__(self):
        _jit_local.ctx = self
        return self

    def __exit__(self, *exc):
        _jit_local.ctx = None


def _get_jit_context() -> Optional[_JitContext]:
    return getattr(_jit_local, "ctx", None)


class KernelDef:
    def __init__(self, fn: Callable):
        self.fn = fn
        self.name = fn.__name__
        self._sig = inspect.signature(fn)
        self._traced = None

    @property
    def traced_fn(self) -> Callable:
        """The body that is traced: `fn` with its enigma.range loops carrying values
        (compiler/loops.py), rewritten once."""
        if self._traced is None:
            from .loops import rewrite_range_loops
            self._traced = rewrite_range_loops(self.fn)
        return self._traced

    def __call__(self, *args, **kwargs) -> "KernelHandle":
        return KernelHandle(self, args, kwargs)

    def __repr__(self):
        return f"<enigma.kernel {self.name}>"


def kernel(fn: Callable) -> KernelDef:
    return KernelDef(fn)


class JitDef:
    def __init__(self, fn: Callable):
        self.fn = fn
        self.name = fn.__name__

    def __repr__(self):
        return f"<enigma.jit {self.name}>"


def jit(fn: Callable) -> JitDef:
    return JitDef(fn)


class KernelHandle:
    def __init__(self, kernel_def: KernelDef, args: tuple, kwargs: dict):
        self.kernel_def, self.args, self.kwargs = kernel_def, args, kwargs

    def launch(self, grid: Tuple[int, ...], block: Tuple[int, ...]):
        ctx = _get_jit_context()
        if ctx is None:
            raise RuntimeError("kernel.launch() called outside enigma.compile() context")
        b = KernelBuilder(self.kernel_def.name)
        seen = set()
        for a in self.args:
            if isinstance(a, Tensor) and a.buffer_index >= 0 and a.name not in seen:
                b.args.append((a.name, a.buffer_index, a.metal_dtype))
                seen.add(a.name)
        with b:
            self.kernel_def.traced_fn(*self.args, **self.kwargs)
        ctx.builder, ctx.grid, ctx.block, ctx.args = b, tuple(grid), tuple(block), self.args


def _metal_dtype(ann) -> str:
    if isinstance(ann, (Scalar, Numeric)):
        return ann.metal_name
    if isinstance(ann, type) and issubclass(ann, Numeric):
        return ann.metal_name
    raise TypeError(f"Unsupported kernel parameter annotation: {ann!r}")


def trace_kernel(kdef: KernelDef) -> KernelBuilder:
    """Trace an annotated kernel: one buffer proxy per parameter."""
    b = KernelBuilder(kdef.name)
    proxies = []
    with b:
        for idx, p in enumerate(kdef._sig.parameters.values()):
            if p.annotation is inspect.Parameter.empty:
                raise TypeError(f"Kernel parameter '{p.name}' needs a type annotation")
            dt = _metal_dtype(p.annotation)
            b.args.append((p.name, idx, dt))
            if isinstance(p.annotation, Scalar):
                b.scalar_params.append((p.name, idx, dt))
                buf = Tensor(p.name, idx, dt)
                v = b.new_value(dt)
                v.name = f"_scalar_{p.name}"
                b.record(IROp("load", v, [b.make_const("uint", 0)], buf._attrs()))
                proxies.append(v)
            else:
                proxies.append(Tensor(p.name, idx, dt))
        kdef.traced_fn(*proxies)
    return b
