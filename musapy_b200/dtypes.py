"""musapy dtypes: the 15 types of rust/musapy-core/src/dtype.rs:25-41, their
string aliases (rust/musapy-python/src/dtype.rs:40-64), promotion, and the
numpy / torch equivalents used at the host boundary.
"""
from __future__ import annotations

import numpy as np
import torch

from . import errors

try:  # bfloat16 for numpy; optional (bf16 data then travels as raw uint16)
    import ml_dtypes as _mld

    _NP_BF16 = np.dtype(_mld.bfloat16)
except Exception:  # pragma: no cover - exercised only without ml_dtypes
    _NP_BF16 = None


class Dtype:
    __slots__ = ("code", "name", "itemsize")

    def __init__(self, spec) -> None:
        d = parse(spec)
        self.code = d.code
        self.name = d.name
        self.itemsize = d.itemsize

    @classmethod
    def _make(cls, code: int, name: str, itemsize: int) -> "Dtype":
        obj = cls.__new__(cls)
        obj.code = code
        obj.name = name
        obj.itemsize = itemsize
        return obj

    def element_size(self) -> int:
        return self.itemsize

    def is_floating(self) -> bool:
        return self.code in (F16, F32, F64, BF16)

    def is_integer(self) -> bool:
        return I8 <= self.code <= U64

    def is_complex(self) -> bool:
        return self.code in (C64, C128)

    def __eq__(self, other) -> bool:
        if isinstance(other, Dtype):
            return self.code == other.code
        if isinstance(other, str):
            d = _ALIASES.get(other.lower())
            return d is not None and d.code == self.code
        return NotImplemented

    def __hash__(self) -> int:
        return hash(self.code)

    def __repr__(self) -> str:
        return f"musapy.{self.name}"

    def __str__(self) -> str:
        return self.name

    def __format__(self, fmt: str) -> str:
        return format(self.name, fmt)


BOOL, I8, I16, I32, I64, U8, U16, U32, U64, F16, F32, F64, BF16, C64, C128 = range(15)

_TABLE = [
    (BOOL, "bool", 1), (I8, "int8", 1), (I16, "int16", 2), (I32, "int32", 4), (I64, "int64", 8),
    (U8, "uint8", 1), (U16, "uint16", 2), (U32, "uint32", 4), (U64, "uint64", 8),
    (F16, "float16", 2), (F32, "float32", 4), (F64, "float64", 8), (BF16, "bfloat16", 2),
    (C64, "complex64", 8), (C128, "complex128", 16),
]
BY_CODE = [Dtype._make(c, n, s) for c, n, s in _TABLE]

bool_, int8, int16, int32, int64, uint8, uint16, uint32, uint64 = BY_CODE[:9]
float16, float32, float64, bfloat16, complex64, complex128 = BY_CODE[9:]

_ALIASES = {
    "bool": bool_, "b1": bool_, "bool8": bool_,
    "int8": int8, "i8": int8, "int16": int16, "i16": int16,
    "int32": int32, "i32": int32, "int64": int64, "i64": int64,
    "uint8": uint8, "u8": uint8, "uint16": uint16, "u16": uint16,
    "uint32": uint32, "u32": uint32, "uint64": uint64, "u64": uint64,
    "float16": float16, "half": float16, "f16": float16,
    "float32": float32, "single": float32, "f32": float32,
    "float64": float64, "double": float64, "f64": float64,
    "bfloat16": bfloat16, "bf16": bfloat16,
    "complex64": complex64, "c64": complex64, "complex128": complex128, "c128": complex128,
}


def parse(spec) -> Dtype:
    if isinstance(spec, Dtype):
        return spec
    if isinstance(spec, str):
        d = _ALIASES.get(spec.lower())
        if d is None:
            raise errors.DtypeError(f"unknown dtype '{spec}'")
        return d
    if isinstance(spec, np.dtype) or (isinstance(spec, type) and issubclass(spec, np.generic)):
        return from_numpy(np.dtype(spec))
    if isinstance(spec, torch.dtype):
        return from_torch(spec)
    raise errors.DtypeError(f"cannot interpret {spec!r} as a dtype")


_NP = {
    BOOL: np.dtype(np.bool_), I8: np.dtype(np.int8), I16: np.dtype(np.int16), I32: np.dtype(np.int32),
    I64: np.dtype(np.int64), U8: np.dtype(np.uint8), U16: np.dtype(np.uint16), U32: np.dtype(np.uint32),
    U64: np.dtype(np.uint64), F16: np.dtype(np.float16), F32: np.dtype(np.float32),
    F64: np.dtype(np.float64), C64: np.dtype(np.complex64), C128: np.dtype(np.complex128),
}
if _NP_BF16 is not None:
    _NP[BF16] = _NP_BF16


def to_numpy(d: Dtype) -> np.dtype:
    """numpy dtype with the same bytes (bf16 -> ml_dtypes.bfloat16 or uint16 bits)."""
    if d.code == BF16 and _NP_BF16 is None:
        return np.dtype(np.uint16)
    return _NP[d.code]


def from_numpy(nd: np.dtype) -> Dtype:
    nd = np.dtype(nd)
    if _NP_BF16 is not None and nd == _NP_BF16:
        return bfloat16
    for code, v in _NP.items():
        if v == nd:
            return BY_CODE[code]
    raise errors.DtypeError(f"numpy dtype {nd} has no musapy equivalent")


_TORCH = {
    BOOL: torch.bool, I8: torch.int8, I16: torch.int16, I32: torch.int32, I64: torch.int64,
    U8: torch.uint8, U16: torch.uint16, U32: torch.uint32, U64: torch.uint64,
    F16: torch.float16, F32: torch.float32, F64: torch.float64, BF16: torch.bfloat16,
    C64: torch.complex64, C128: torch.complex128,
}


def to_torch(d: Dtype) -> torch.dtype:
    return _TORCH[d.code]


def from_torch(td: torch.dtype) -> Dtype:
    for code, v in _TORCH.items():
        if v == td:
            return BY_CODE[code]
    raise errors.DtypeError(f"torch dtype {td} has no musapy equivalent")


def promote(a: Dtype, b: Dtype, all_gpu: bool = True) -> Dtype:
    """Result dtype of a binary op (dtype.rs:302-338); all_gpu selects the
    narrow-first rule musapy uses when every input lives on the device."""
    key = (a.code, b.code, bool(all_gpu))
    d = _PROMOTE_CACHE.get(key)
    if d is None:
        from ._lib import LIB

        code = LIB.mpb_promote(a.code, b.code, 1 if all_gpu else 0)
        if code < 0:
            raise errors.DtypeError(f"cannot promote {a} with {b}")
        d = _PROMOTE_CACHE[key] = BY_CODE[code]
    return d


_PROMOTE_CACHE: dict = {}
