"""MetalRuntime: the reference's dispatch API, backed by libenigma_cuda.so.

Python signatures, bind-order rules and error messages follow the
reference's enigma/runtime_dispatch/runtime.py:
  execute(compiled, inputs, output_size, grid, threads, *, scalars,
          output_sizes, constants, output_shapes, output_dtypes)   (:318-523)
  prepare(compiled, inputs, output_size) -> PreparedKernel          (:529-599)
  PreparedKernel.dispatch / dispatch_timed / read_output / release  (:602-656)
  device_capabilities()                                              (:525)
Bind order is inputs, Scalar params at their buffer index, outputs last;
inputs + scalars + outputs must equal the kernel's parameter count.

Buffers: numpy arrays / bytes are copied to device memory the library
allocates (the reference copies host arrays into shared buffers, swift
:91-103); torch CUDA tensors are bound zero-copy (the analogue of the
reference's mlx interop) and must outlive the call.  Outputs come back as
bytes, or as torch tensors when output_shapes / output_dtypes are torch
shapes and dtypes.  Dispatch is synchronous like the reference's
waitUntilCompleted; `grid` is Metal-style total threads per axis.
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass
from typing import Any, List, Optional, Tuple

import numpy as np

from .. import _native
from ..compiler.compiler import CompiledKernel
from . import handwritten as _handwritten
from . import launch as _launch

_SCALAR_NP = {
    "float": "float32", "f32": "float32", "half": "float16", "f16": "float16",
    "bfloat": "float32", "bf16": "float32", "char": "int8", "i8": "int8", "uchar": "uint8",
    "u8": "uint8", "short": "int16", "i16": "int16", "ushort": "uint16", "u16": "uint16",
    "int": "int32", "i32": "int32", "uint": "uint32", "u32": "uint32", "long": "int64",
    "i64": "int64", "ulong": "uint64", "u64": "uint64", "bool": "uint8", "i1": "uint8",
}


def _gpu_error(msg: str, **ctx) -> RuntimeError:
    parts = [f"enigma GPU error: {msg}"] + [f"  {k}: {v}" for k, v in ctx.items()]
    return RuntimeError("\n".join(parts))


def _merge_scalar_buffers(inputs, scalars, scalar_params, num_outputs=0):
    """Place one-element scalar buffers at their declared slots among the inputs."""
    if not scalar_params:
        if scalars:
            raise RuntimeError(f"execute: got {len(scalars)} scalars but kernel has no Scalar params")
        return list(inputs)
    if len(scalars) != len(scalar_params):
        raise RuntimeError(f"execute: expected {len(scalar_params)} scalars "
                           f"(one per Scalar param), got {len(scalars)}")
    total = len(inputs) + len(scalar_params) + num_outputs
    n_merged = total - num_outputs
    slots: list = [None] * n_merged
    for k, (_name, bi, dt) in sorted(enumerate(scalar_params), key=lambda e: e[1][1]):
        if bi >= total:
            raise RuntimeError(f"scalar buffer_index {bi} exceeds total slots {total}")
        if bi >= n_merged:
            raise RuntimeError(f"scalar buffer_index {bi} lands in output region "
                               f"(merged_slots={n_merged}, total={total})")
        slots[bi] = np.asarray([scalars[k]], dtype=_SCALAR_NP.get(dt, "float32"))
    it = iter(inputs)
    return [s if s is not None else next(it) for s in slots]


@dataclass
class DeviceCapabilities:
    """Capabilities of the CUDA device (fields of the reference's dataclass kept)."""

    gpu_family: str
    gpu_family_raw: int
    supports_async_copy: bool
    supports_simdgroup_matrix: bool
    simdgroup_size: int
    max_threadgroup_memory: int
    max_threads_per_threadgroup: int
    device_name: str
    sm_count: int = 0
    total_memory: int = 0

    @property
    def is_m3_or_newer(self) -> bool:
        """The async-copy / tensor-core features the M3 gate protects exist on sm_100."""
        return self.supports_async_copy

    def require_m3(self, feature: str) -> None:
        if not self.is_m3_or_newer:
            raise RuntimeError(f"enigma: {feature} requires async copy support. "
                               f"Current device: {self.device_name} ({self.gpu_family})")


def _torch_mod():
    try:
        import torch
        return torch
    except ImportError:  # pragma: no cover
        return None


class _DeviceBuffers:
    """Device memory for one bind list: owned allocations and borrowed tensors."""

    def __init__(self, stream):
        self.stream = stream
        self.ptrs: List[int] = []
        self.nbytes: List[int] = []
        self._owned: List[int] = []

    def add_host(self, data) -> None:
        arr = np.ascontiguousarray(data if not isinstance(data, (bytes, bytearray))
                                   else np.frombuffer(data, dtype=np.uint8))
        p = ctypes.c_void_p()
        _native.call("enigma_alloc", ctypes.byref(p), max(arr.nbytes, 16))
        self._owned.append(p.value)
        if arr.nbytes:
            _native.call("enigma_upload", p.value, arr.ctypes.data, arr.nbytes, self.stream)
        self.ptrs.append(p.value)
        self.nbytes.append(arr.nbytes)

    def add_tensor(self, t) -> None:
        if not t.is_contiguous():
            raise _gpu_error("torch inputs must be contiguous")
        self.ptrs.append(t.data_ptr())
        self.nbytes.append(t.numel() * t.element_size())

    def add_empty(self, nbytes: int) -> None:
        p = ctypes.c_void_p()
        _native.call("enigma_alloc", ctypes.byref(p), max(int(nbytes), 16))
        self._owned.append(p.value)
        _native.call("enigma_memset", p.value, 0, int(nbytes), self.stream)
        self.ptrs.append(p.value)
        self.nbytes.append(int(nbytes))

    def read(self, slot: int, nbytes: int) -> bytes:
        out = np.empty(nbytes, dtype=np.uint8)
        if nbytes:
            _native.call("enigma_download", out.ctypes.data, self.ptrs[slot], nbytes, self.stream)
        _native.call("enigma_synchronize", self.stream)
        return out.tobytes()

    def free(self) -> None:
        for p in self._owned:
            _native.lib().enigma_free(p)
        self._owned.clear()


class MetalRuntime:
    """Dispatch runtime (name kept from the reference so its callers run unchanged)."""

    def __init__(self, dylib_path: Optional[str] = None, device: int = 0):
        if dylib_path is not None:
            import os
            os.environ["ENIGMA_CUDA_LIB"] = str(dylib_path)
        self._lib = _native.lib()
        self.device = int(device)
        _native.call("enigma_init", self.device)
        s = ctypes.c_void_p()
        _native.call("enigma_stream_create", ctypes.byref(s))
        self._stream = s.value

    # ------------------------------------------------------------------ helpers
    @staticmethod
    def _binding(compiled: CompiledKernel, inputs=()):
        b = getattr(compiled, "cuda_kernel", None)
        if b is None:
            # A bare CompiledKernel around one of the reference's hand-written Metal kernels.
            b = _handwritten.bind(compiled.kernel_name, getattr(compiled, "metal_source", ""),
                                  list(inputs))
        if b is None:
            raise _gpu_error("compiled kernel has no sm_100a binding (was it built by "
                             "enigma.compile?)", kernel=compiled.kernel_name)
        return b

    @staticmethod
    def _check_bind_count(where, compiled, n_in, n_sc, n_out):
        num = getattr(compiled, "num_params", None)
        if num is None:
            return
        total = n_in + n_sc + n_out
        if total != num:
            names = getattr(compiled, "param_names", None) or []
            hint = f"  kernel '{compiled.kernel_name}' params: {names}\n" if names else ""
            raise _gpu_error(
                f"{where}: kernel '{compiled.kernel_name}' has {num} parameter(s), but got "
                f"{n_in} input(s) + {n_sc} scalar(s) + {n_out} output buffer(s) = {total}.\n"
                f"{hint}Outputs are appended AFTER inputs in the bind list. Pass every kernel "
                f"parameter exactly once across inputs= / scalars= / output_size(s)/_shapes.")

    def _bind(self, merged_inputs, out_sizes, out_tensors=None):
        """Device buffers in bind order.  CUDA tensors (inputs, and outputs when given) are
        borrowed; the runtime's stream first waits for the work torch has queued on them
        (the stream is non-blocking, so it would not otherwise order after torch's)."""
        torch = _torch_mod()
        bufs = _DeviceBuffers(self._stream)
        borrowed = False
        try:
            for x in merged_inputs:
                if torch is not None and isinstance(x, torch.Tensor):
                    if not x.is_cuda:
                        x = x.contiguous().numpy() if x.dtype != torch.bfloat16 else \
                            x.contiguous().view(torch.int16).numpy()
                        bufs.add_host(x)
                    else:
                        bufs.add_tensor(x)
                        borrowed = True
                else:
                    bufs.add_host(x)
            if out_tensors is not None:
                for t in out_tensors:
                    bufs.add_tensor(t)
                borrowed = True
            else:
                for sz in out_sizes:
                    bufs.add_empty(sz)
        except Exception:
            bufs.free()
            raise
        if borrowed:
            ev = torch.cuda.Event()
            ev.record(torch.cuda.current_stream(self.device))
            torch.cuda.ExternalStream(self._stream, device=self.device).wait_event(ev)
        return bufs

    # ------------------------------------------------------------------ execute
    def execute(self, compiled: CompiledKernel, inputs: List[Any], output_size=None,
                grid: Tuple[int, int, int] = (1, 1, 1), threads: Tuple[int, int, int] = (1, 1, 1),
                *, scalars: Optional[List] = None, output_sizes: Optional[List[int]] = None,
                constants: Optional[dict] = None, output_shapes: Optional[List[tuple]] = None,
                output_dtypes: Optional[List] = None):
        """One shot: bind (copying host inputs), launch, wait, read back, free."""
        binding = self._binding(compiled, inputs)
        torch_out = output_shapes is not None
        if torch_out:
            if output_dtypes is None or len(output_dtypes) != len(output_shapes):
                raise _gpu_error("execute: output_shapes requires output_dtypes of matching length")
            torch = _torch_mod()
            out_sizes = [int(np.prod(s)) * torch.empty((), dtype=d).element_size()
                         for s, d in zip(output_shapes, output_dtypes)]
            multi = len(output_shapes) > 1
        elif output_sizes is not None:
            out_sizes, multi = [int(s) for s in output_sizes], True
        else:
            if output_size is None:
                raise _gpu_error("execute: must pass output_size, output_sizes, or output_shapes")
            out_sizes, multi = [int(output_size)], False
        scalar_params = getattr(compiled, "scalar_params", None) or []
        self._check_bind_count("execute", compiled, len(inputs), len(scalars or []),
                               len(out_sizes))
        merged = _merge_scalar_buffers(inputs, scalars or [], scalar_params, len(out_sizes))
        scalar_slots = {sp[1] for sp in scalar_params}
        values = {"scalars": {sp[1]: v for sp, v in zip(scalar_params, scalars or [])},
                  "constants": {int(k): (v[1] if isinstance(v, tuple) else v)
                                for k, v in (constants or {}).items()}}
        out_tensors = None
        if torch_out:
            # Outputs are torch tensors on this device: the kernels write them in place.
            out_tensors = [torch.zeros(shp, dtype=dt, device=f"cuda:{self.device}")
                           for shp, dt in zip(output_shapes, output_dtypes)]
        bufs = self._bind(merged, out_sizes, out_tensors)
        try:
            keep = [i for i in range(len(bufs.ptrs)) if i not in scalar_slots]
            p = _launch.plan(binding, [bufs.nbytes[i] for i in keep], tuple(grid), tuple(threads),
                             values)
            try:
                p.fn([bufs.ptrs[i] for i in keep], self._stream)
                _native.call("enigma_synchronize", self._stream)
            except _native.EnigmaCudaError as e:
                raise _gpu_error(f"dispatch failed: {e}", kernel=compiled.kernel_name, grid=grid,
                                 threads=threads, plan=p.describe, return_code=e.status) from e
            first_out = len(merged)
            if torch_out:
                return out_tensors if multi else out_tensors[0]
            outs = [bufs.read(first_out + k, sz) for k, sz in enumerate(out_sizes)]
            return outs if multi else outs[0]
        finally:
            bufs.free()

    def device_capabilities(self) -> DeviceCapabilities:
        name = ctypes.create_string_buffer(256)
        _native.call("enigma_device_name", self.device, name, 256)
        sm, smem, thr, mem = (ctypes.c_int64() for _ in range(4))
        ma, mi = ctypes.c_int32(), ctypes.c_int32()
        _native.call("enigma_device_attrs", self.device, ctypes.byref(sm), ctypes.byref(smem),
                     ctypes.byref(thr), ctypes.byref(mem), ctypes.byref(ma), ctypes.byref(mi))
        return DeviceCapabilities(
            gpu_family=f"sm_{ma.value}{mi.value}", gpu_family_raw=ma.value * 10 + mi.value,
            supports_async_copy=ma.value >= 9, supports_simdgroup_matrix=ma.value >= 8,
            simdgroup_size=32, max_threadgroup_memory=smem.value,
            max_threads_per_threadgroup=thr.value, device_name=name.value.decode(),
            sm_count=sm.value, total_memory=mem.value)

    # ------------------------------------------------------------------ prepare
    def prepare(self, compiled: CompiledKernel, inputs: List[Any], output_size: int
                ) -> "PreparedKernel":
        """Bind once (inputs copied to the device) for repeated dispatch."""
        binding = self._binding(compiled, inputs)
        n_sc = len(getattr(compiled, "scalar_params", None) or [])
        num = getattr(compiled, "num_params", None)
        if num is not None and len(inputs) + n_sc + 1 != num:
            names = getattr(compiled, "param_names", None) or []
            hint = f"  kernel '{compiled.kernel_name}' params: {names}\n" if names else ""
            raise _gpu_error(
                f"prepare: kernel '{compiled.kernel_name}' has {num} parameter(s), but got "
                f"{len(inputs)} input(s) + {n_sc} scalar(s) + 1 output buffer = "
                f"{len(inputs) + n_sc + 1}.\n{hint}The output is appended AFTER inputs in the "
                f"bind list.")
        bufs = self._bind(list(inputs), [int(output_size)])
        return PreparedKernel(self, compiled, binding, bufs, int(output_size))

    def release(self):
        if getattr(self, "_stream", None):
            self._lib.enigma_stream_destroy(self._stream)
            self._stream = None


Runtime = MetalRuntime


class PreparedKernel:
    """Device-resident buffers of one bind list, for timing loops."""

    def __init__(self, rt: MetalRuntime, compiled, binding, bufs: _DeviceBuffers, output_size):
        self._rt, self._compiled, self._binding = rt, compiled, binding
        self._bufs, self._output_size = bufs, output_size
        self._plans = {}

    def _plan(self, grid, threads):
        key = (tuple(grid), tuple(threads))
        if key not in self._plans:
            self._plans[key] = _launch.plan(self._binding, self._bufs.nbytes, *key)
        return self._plans[key]

    def dispatch(self, grid: Tuple[int, int, int], threads: Tuple[int, int, int]) -> None:
        p = self._plan(grid, threads)
        try:
            p.fn(self._bufs.ptrs, self._rt._stream)
            _native.call("enigma_synchronize", self._rt._stream)
        except _native.EnigmaCudaError as e:
            raise _gpu_error(f"dispatch failed: {e}", kernel=self._compiled.kernel_name,
                             grid=grid, threads=threads, return_code=e.status) from e

    def dispatch_timed(self, grid: Tuple[int, int, int], threads: Tuple[int, int, int]) -> float:
        """Launch once; device time in microseconds from CUDA events on the runtime's stream."""
        p = self._plan(grid, threads)
        ev = [ctypes.c_void_p(), ctypes.c_void_p()]
        for e in ev:
            _native.call("enigma_event_create", ctypes.byref(e))
        try:
            s = self._rt._stream
            _native.call("enigma_event_record", ev[0].value, s)
            p.fn(self._bufs.ptrs, s)
            _native.call("enigma_event_record", ev[1].value, s)
            _native.call("enigma_synchronize", s)
            ms = ctypes.c_float()
            _native.call("enigma_event_elapsed_ms", ev[0].value, ev[1].value, ctypes.byref(ms))
            return ms.value * 1000.0
        except _native.EnigmaCudaError as e:
            raise _gpu_error(f"dispatch failed: {e}", kernel=self._compiled.kernel_name,
                             grid=grid, threads=threads, return_code=e.status) from e
        finally:
            for e in ev:
                _native.lib().enigma_event_destroy(e.value)

    def read_output(self) -> bytes:
        return self._bufs.read(len(self._bufs.ptrs) - 1, self._output_size)

    def release(self):
        self._bufs.free()
