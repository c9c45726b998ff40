"""enigma.compile: trace, then bind to an sm_100a kernel.

Signature and result type follow the reference (enigma/compiler/compiler.py:
30-93).  Where the reference lowers the trace to MSL and runs xcrun, this
build recognises the traced kernel (recognize.py) and records the binding;
`metal_source` carries a readable dump of the trace instead of MSL, and no
metallib exists (metallib_path / metallib_bytes are None).
"""
from __future__ import annotations

import sys
from dataclasses import dataclass
from typing import Optional, Tuple

from .kernel import JitDef, KernelDef, _JitContext, trace_kernel
from .recognize import Binding, recognize


@dataclass
class CompiledKernel:
    kernel_name: str
    metallib_path: Optional[str] = None
    metallib_bytes: Optional[bytes] = None
    metal_source: str = ""
    mlir_source: Optional[str] = None
    grid: Optional[Tuple[int, ...]] = None
    block: Optional[Tuple[int, ...]] = None
    scalar_params: list = None  # type: ignore[assignment]
    num_params: Optional[int] = None
    param_names: Optional[list] = None
    cuda_kernel: Optional[Binding] = None
    param_dtypes: Optional[list] = None

    @property
    def kernel_source(self) -> str:
        return self.metal_source

    @property
    def has_metallib(self) -> bool:
        return False

    def export_metal(self, path: str = None) -> str:
        """Write the trace dump (the B200 build has no MSL) and return the path."""
        path = path or f"{self.kernel_name}.ir.txt"
        with open(path, "w") as f:
            f.write(self.metal_source)
        return path


def format_ir(builder) -> str:
    lines = [f"// enigma trace of {builder.kernel_name}: args {builder.args}"]

    def emit(ops, depth):
        for op in ops:
            res = f"{op.result.name}:{op.result.dtype} = " if op.result is not None else ""
            if op.op == "scf_for" and op.attrs.get("results"):
                # loop-carried values: results = scf_for(bounds, inits) {iv, iter_args ...
                # yield}
                res = ", ".join(f"{r.name}:{r.dtype}" for r in op.attrs["results"]) + " = "
            opnds = ", ".join(getattr(o, "name", repr(o)) for o in op.operands)
            attrs = {k: v for k, v in op.attrs.items() if k not in ("iv", "iter_args",
                                                                     "yield_vals", "results")}
            lines.append("  " * depth + f"{res}{op.op}({opnds}) {attrs if attrs else ''}".rstrip())
            for r in op.regions:
                head = "{"
                if op.op == "scf_for" and "iv" in op.attrs:
                    carried = op.attrs.get("iter_args") or []
                    head = "{ (" + ", ".join([op.attrs["iv"].name] + [a.name for a in carried]) + ")"
                lines.append("  " * depth + head)
                emit(r, depth + 1)
                if op.op == "scf_for" and op.attrs.get("yield_vals"):
                    lines.append("  " * (depth + 1) + "yield(" + ", ".join(
                        getattr(v, "name", repr(v)) for v in op.attrs["yield_vals"]) + ")")
                lines.append("  " * depth + "}")

    emit(builder.ops, 1)
    return "\n".join(lines) + "\n"


def compile(fn, *args, keep_metal_source=False, dump_ir=False, dump_mlir=False, work_dir=None,
            vec_width=0, emit_only=None) -> CompiledKernel:
    """Compile an @enigma.kernel (annotated) or @enigma.jit (TV layout) function."""
    if isinstance(fn, JitDef):
        with _JitContext() as ctx:
            fn.fn(*args)
        if ctx.builder is None:
            raise RuntimeError(f"@jit function '{fn.name}' did not launch any kernel. "
                               f"Call kernel_fn(...).launch(grid=..., block=...) inside it.")
        builder, grid, block = ctx.builder, ctx.grid, ctx.block
        tensors = tuple(args)
    elif isinstance(fn, KernelDef):
        builder, grid, block, tensors = trace_kernel(fn), None, None, ()
    else:
        raise TypeError(f"Expected @enigma.kernel or @enigma.jit, got {type(fn).__name__}")
    text = format_ir(builder)
    if dump_ir:
        print(text, file=sys.stderr)
    binding = recognize(builder, tensors)
    return CompiledKernel(
        kernel_name=builder.kernel_name, metal_source=text, grid=grid, block=block,
        scalar_params=list(builder.scalar_params), num_params=len(builder.args),
        param_names=[a[0] for a in builder.args], param_dtypes=[a[2] for a in builder.args],
        cuda_kernel=binding)
