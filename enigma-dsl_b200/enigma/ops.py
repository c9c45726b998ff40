"""Tile-level helpers used inside @enigma.kernel bodies (trace-time only).

Same names and semantics as the reference's enigma/ops/gemm.py and
enigma/ops/quant.py: `gemm` records C += A @ B over an M x N x K tile
(one 8x8x8 matrix multiply-accumulate when the shape allows, a scalar
triple loop into a RegisterTensor otherwise); the quant helpers record
bit packing and int8 dequantisation.  Whole-matrix GEMMs run on the sm_100a
tensor cores through enigma.cuda_ops.gemm / the recognizer, not through this
tile helper.
"""
from __future__ import annotations

from typing import Optional

from ._tracing import (EnigmaError, IROp, RegisterTensor, _ensure_ir, _require_builder, cmp_ge,
                       extract_bits, fma, insert_bits, make_filled_simdgroup_matrix, metal_cast,
                       select, simdgroup_matrix_load, simdgroup_matrix_store,
                       simdgroup_multiply_accumulate)
from .tensor import Tensor


def gemm(A_s, B_s, C, *, M: int, N: int, K: int, transpose_A: bool = False,
         transpose_B: bool = False, accum_dtype: str = "float",
         use_simdgroup: Optional[bool] = None) -> None:
    """Record C += A @ B over an M x N tile with reduction K.

    Besides the per-element ops, a `tile_gemm` marker op carries the tile's shape and
    transpose flags: the recognizer binds a kernel built around one tile GEMM to the
    fp32 GEMM kernel (enigma_gemm_f32_trans)."""
    b = _require_builder("gemm")
    if M <= 0 or N <= 0 or K <= 0:
        raise EnigmaError(f"gemm: M/N/K must be positive, got M={M}, N={N}, K={K}")
    matrix_ok = (M, N, K) == (8, 8, 8) and accum_dtype in ("float", "half") \
        and not (transpose_A or transpose_B)
    if use_simdgroup is True and not matrix_ok:
        raise EnigmaError(f"gemm: use_simdgroup=True but shape ({M}x{N}x{K}, elem={accum_dtype}) "
                          f"is not 8x8x8 (or transpose flags set). The simdgroup path currently "
                          f"supports a single 8x8x8 tile only.")
    b.record(IROp("tile_gemm", None, [], {"M": int(M), "N": int(N), "K": int(K),
                                          "transpose_A": bool(transpose_A),
                                          "transpose_B": bool(transpose_B),
                                          "accum_dtype": accum_dtype}))
    if matrix_ok if use_simdgroup is None else use_simdgroup:
        if not isinstance(C, Tensor):
            raise EnigmaError("gemm: simdgroup path requires C to be a Tensor (threadgroup or "
                              "device buffer); got RegisterTensor. Pass use_simdgroup=False to "
                              "use the scalar accumulator path.")
        a = simdgroup_matrix_load(A_s, 8, accum_dtype)
        b = simdgroup_matrix_load(B_s, 8, accum_dtype)
        c = simdgroup_matrix_load(C, 8, accum_dtype)
        simdgroup_matrix_store(simdgroup_multiply_accumulate(a, b, c), C, 8)
        return
    if isinstance(C, Tensor):
        raise EnigmaError("gemm: scalar fallback path requires C to be a RegisterTensor of shape "
                          "(M, N). Pass `enigma.register_tensor((M, N), ...)` for C.")
    for m in range(M):
        for n in range(N):
            acc = C[m, n]
            for k in range(K):
                a = A_s[k * M + m] if transpose_A else A_s[m * K + k]
                b = B_s[n * K + k] if transpose_B else B_s[k * N + n]
                acc = fma(a, b, acc)
            C[m, n] = acc


def _as_uint(v):
    v = _ensure_ir(v)
    return v if v.dtype == "uint" else metal_cast(v, "uint")


def pack_uint8x4(b0, b1, b2, b3):
    """Four bytes into one uint, lane 0 in the low byte."""
    _require_builder("pack_uint8x4")
    out = metal_cast(0, "uint")
    for shift, val in zip((0, 8, 16, 24), (b0, b1, b2, b3)):
        out = insert_bits(out, _as_uint(val), shift, 8)
    return out


def unpack_uint8x4(packed):
    _require_builder("unpack_uint8x4")
    v = _as_uint(packed)
    return tuple(extract_bits(v, sh, 8) for sh in (0, 8, 16, 24))


def pack_int4x2(lo, hi):
    """Two signed nibbles (two's complement) into the low byte of a uint."""
    _require_builder("pack_int4x2")
    out = insert_bits(metal_cast(0, "uint"), _as_uint(lo), 0, 4)
    return insert_bits(out, _as_uint(hi), 4, 4)


def unpack_int4x2(packed):
    """Inverse of pack_int4x2: nibbles sign-extended (subtract 16 when >= 8)."""
    _require_builder("unpack_int4x2")
    v = _as_uint(packed)
    eight, sixteen = metal_cast(8, "int"), metal_cast(16, "int")

    def sext(nib_u):
        nib = metal_cast(nib_u, "int")
        return select(nib, nib - sixteen, cmp_ge(nib, eight))

    return sext(extract_bits(v, 0, 4)), sext(extract_bits(v, 4, 4))


def dequantize_int8(x, scale, zero_point=0):
    """float(x - zero_point) * scale."""
    _require_builder("dequantize_int8")
    v, s, z = _ensure_ir(x), _ensure_ir(scale), _ensure_ir(zero_point)
    v = v if v.dtype == "int" else metal_cast(v, "int")
    z = z if z.dtype == "int" else metal_cast(z, "int")
    s = s if s.dtype == "float" else metal_cast(s, "float")
    return metal_cast(v - z, "float") * s


__all__ = ["gemm", "pack_uint8x4", "unpack_uint8x4", "pack_int4x2", "unpack_int4x2",
           "dequantize_int8", "RegisterTensor"]
