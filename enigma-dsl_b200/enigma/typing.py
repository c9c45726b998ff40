"""Element-type annotations for @enigma.kernel parameters.

Names and Metal type names match the reference (enigma/typing.py:18-119):
`enigma.f32` annotates a device buffer of float, `enigma.Scalar(enigma.f32)`
a single value the runtime packs into a one-element buffer.  The CUDA side
only needs the element size and kind (CUDA_TYPES below).
"""
from __future__ import annotations


class Numeric:
    width: int = 0
    metal_name: str = ""

    def __repr__(self):
        return f"enigma.{type(self).__name__}"


def _numeric(name: str, width: int, metal: str):
    return type(name, (Numeric,), {"width": width, "metal_name": metal})


Float32 = _numeric("Float32", 32, "float")
Float16 = _numeric("Float16", 16, "half")
BFloat16 = _numeric("BFloat16", 16, "bfloat")
Int8 = _numeric("Int8", 8, "char")
UInt8 = _numeric("UInt8", 8, "uchar")
Int16 = _numeric("Int16", 16, "short")
UInt16 = _numeric("UInt16", 16, "ushort")
Int32 = _numeric("Int32", 32, "int")
UInt32 = _numeric("UInt32", 32, "uint")
Int64 = _numeric("Int64", 64, "long")
UInt64 = _numeric("UInt64", 64, "ulong")
Bool = _numeric("Bool", 1, "bool")

f32, f16, bf16 = Float32(), Float16(), BFloat16()
i8, u8, i16, u16 = Int8(), UInt8(), Int16(), UInt16()
i32, u32, i64, u64 = Int32(), UInt32(), Int64(), UInt64()
b1 = Bool()


class Scalar:
    """A by-value kernel parameter (`n: enigma.Scalar(enigma.u32)`)."""

    def __init__(self, dtype: Numeric):
        if isinstance(dtype, type) and issubclass(dtype, Numeric):
            dtype = dtype()
        if not isinstance(dtype, Numeric):
            raise TypeError(f"Scalar() needs an enigma numeric type, got {dtype!r}")
        self.dtype = dtype
        self.metal_name = dtype.metal_name
        self.width = dtype.width

    def __repr__(self):
        return f"enigma.Scalar({self.dtype!r})"


# Metal type name -> (bytes, numpy dtype name)
CUDA_TYPES = {
    "float": (4, "float32"), "half": (2, "float16"), "bfloat": (2, "bfloat16"),
    "char": (1, "int8"), "uchar": (1, "uint8"), "short": (2, "int16"), "ushort": (2, "uint16"),
    "int": (4, "int32"), "uint": (4, "uint32"), "long": (8, "int64"), "ulong": (8, "uint64"),
    "bool": (1, "uint8"),
}
