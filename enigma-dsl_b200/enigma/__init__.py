"""Enigma on B200: the Enigma DSL surface with sm_100a CUDA kernels behind it.

Public names follow the reference's enigma/__init__.py.  compile() binds a
traced kernel to a hand-written sm_100a kernel (there is no Metal, MSL or
CPU path); MetalRuntime dispatches it through libenigma_cuda.so.
"""
from . import _tracing as _tr
from ._tracing import (EnigmaError, Carry, Pipeline, RegisterTensor, _EnigmaRange,
                       _EnigmaRangeConstexpr, as_type, async_copy_1d_d2t, async_copy_1d_t2d,
                       async_copy_2d_d2t, async_copy_2d_t2d, async_copy_commit,
                       async_copy_to_threadgroup, async_copy_wait, barrier, copy, cross,
                       determinant, distance, dot, extract_bits, faceforward, for_range,
                       function_constant, if_, insert_bits, length, load_if, make_filled_simdgroup_matrix,
                       make_float2, make_float3, make_float4, make_vec, matmul, metal_cast,
                       normalize, pipeline, reflect, refract, register_tensor, simd_barrier,
                       simdgroup_matrix_load, simdgroup_matrix_store, simdgroup_multiply_accumulate,
                       store_if, threadgroup_alloc, transpose, vec_extract, while_)
from ._tracing import select as where  # noqa: F401
from .compiler.compiler import CompiledKernel, compile  # noqa: A004
from .compiler.kernel import jit, kernel
from .core import (Layout, Swizzle, SwizzledLayout, blocked_product, coalesce, complement,
                   composition, logical_divide, make_identity_layout, make_layout, make_layout_tv,
                   make_ordered_layout, recast_layout, size, swizzle, zipped_divide)
from .runtime_dispatch.runtime import MetalRuntime, PreparedKernel, Runtime
from .tensor import Tensor, make_identity_tensor, tensor_composition, tensor_zipped_divide
from .tuple import product, repeat_like, select
from .typing import (BFloat16, Bool, Float16, Float32, Int8, Int16, Int32, Int64, Scalar, UInt8,
                     UInt16, UInt32, UInt64, b1, bf16, f16, f32, i8, i16, i32, i64, u8, u16, u32,
                     u64)
from . import benchmark, cuda_ops, ops, testing  # noqa: F401
from .ops import (dequantize_int8, gemm, pack_int4x2, pack_uint8x4, unpack_int4x2,
                  unpack_uint8x4)

__version__ = "0.1.0+b200"

# Table-generated intrinsics (math, reductions, shuffles, comparisons, grid queries, atomics,
# pack/unpack) are re-exported by name.
_GENERATED = (_tr._UNARY + _tr._PREDICATES + _tr._BINARY + _tr._TERNARY + _tr._REDUCTIONS
              + _tr._SHUFFLES + ["cmp_" + c for c in _tr._COMPARES] + _tr._GRID_XYZ
              + _tr._GRID_SCALAR + _tr._PACKS + _tr._UNPACKS
              + ["atomic_load", "atomic_store", "atomic_exchange", "atomic_fetch_add",
                 "atomic_fetch_sub", "atomic_fetch_min", "atomic_fetch_max", "atomic_fetch_and",
                 "atomic_fetch_or", "atomic_fetch_xor", "atomic_compare_exchange_weak"])
for _name in _GENERATED:
    globals()[_name] = getattr(_tr, _name)
del _name

range = _EnigmaRange()  # noqa: A001
range_constexpr = _EnigmaRangeConstexpr()


class arch:
    """CUDA-style thread/block index accessors for use inside @enigma.kernel."""

    @staticmethod
    def thread_idx():
        b = _tr._require_builder("arch.thread_idx")
        return (b.get_thread_idx(), 0, 0)

    @staticmethod
    def block_idx():
        b = _tr._require_builder("arch.block_idx")
        return (b.get_block_idx(), 0, 0)

    @staticmethod
    def block_dim():
        b = _tr._require_builder("arch.block_dim")
        return (b.get_block_dim(), 0, 0)


def __getattr__(name: str):
    if name == "thread_position_in_grid":
        b = _tr.get_builder()
        if b is None:
            raise RuntimeError(
                "enigma.thread_position_in_grid can only be used inside @enigma.kernel")
        return b.get_thread_position_in_grid()
    raise AttributeError(f"module 'enigma' has no attribute {name!r}")
