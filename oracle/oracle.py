"""TEST INFRASTRUCTURE ONLY - numpy-facing wrapper of the C parity oracle.

Restates the CPU path of musapy's operator layer on numpy arrays:
promotion (rust/musapy-core/src/dtype.rs:206-338), the cast-then-compute
order of the 3-phase skeletons (rust/musapy-ops/src/op_builder.rs:315-532),
broadcast strides (rust/musapy-ops/src/broadcast.rs:24-92), the per-axis
iteration of multi-axis reductions and the transpose+merge of multi-axis
argmax/argmin (rust/musapy-ops/src/reduction.rs:118-223). The arithmetic
itself runs in oracle.c (built by oracle/Makefile).

Only tests/, __graft_entry__.smoke() and bench.py's CPU legs import this
module; the product never does.
"""
from __future__ import annotations

import ctypes
import math
import os
import subprocess

import numpy as np

try:
    import ml_dtypes as _mld

    NP_BF16 = np.dtype(_mld.bfloat16)
except Exception:  # pragma: no cover
    NP_BF16 = None

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "_build", "liboracle.so")

BOOL, I8, I16, I32, I64, U8, U16, U32, U64, F16, F32, F64, BF16, C64, C128 = range(15)
NAMES = ["bool", "int8", "int16", "int32", "int64", "uint8", "uint16", "uint32", "uint64",
         "float16", "float32", "float64", "bfloat16", "complex64", "complex128"]
OPS = {"add": 0, "sub": 1, "mul": 2, "div": 3, "pow": 4, "eq": 10, "ne": 11, "lt": 12, "gt": 13, "le": 14,
       "ge": 15, "sin": 20, "cos": 21, "exp": 22, "log": 23, "abs": 24, "sign": 25, "neg": 26}
RED = {"sum": 0, "prod": 1, "max": 2, "min": 3, "mean": 4, "argmax": 5, "argmin": 6}

_NP = {BOOL: np.dtype(np.bool_), I8: np.dtype(np.int8), I16: np.dtype(np.int16), I32: np.dtype(np.int32),
       I64: np.dtype(np.int64), U8: np.dtype(np.uint8), U16: np.dtype(np.uint16), U32: np.dtype(np.uint32),
       U64: np.dtype(np.uint64), F16: np.dtype(np.float16), F32: np.dtype(np.float32), F64: np.dtype(np.float64),
       BF16: NP_BF16 if NP_BF16 is not None else np.dtype(np.uint16), C64: np.dtype(np.complex64),
       C128: np.dtype(np.complex128)}


def build() -> str:
    """Compile liboracle.so (make) when missing or stale."""
    src = os.path.join(HERE, "oracle.c")
    if not os.path.exists(LIB_PATH) or os.path.getmtime(src) > os.path.getmtime(LIB_PATH):
        subprocess.run(["make", "-C", HERE], check=True, capture_output=True)
    return LIB_PATH


_LIB = None


def lib() -> ctypes.CDLL:
    global _LIB
    if _LIB is None:
        build()
        L = ctypes.CDLL(LIB_PATH)
        vp, ip, i64p = ctypes.c_void_p, ctypes.c_int, ctypes.POINTER(ctypes.c_int64)
        L.or_binary.argtypes = [ip, ip, vp, vp, vp, ip, i64p, i64p, i64p]
        L.or_compare.argtypes = [ip, ip, vp, vp, vp, ip, i64p, i64p, i64p]
        L.or_unary.argtypes = [ip, ip, vp, vp, ip, i64p, i64p]
        L.or_clamp.argtypes = [ip, vp, vp, ctypes.c_double, ctypes.c_double, ip, i64p, i64p]
        L.or_cast.argtypes = [ip, ip, vp, vp, ip, i64p, i64p]
        L.or_reduce.argtypes = [ip, ip, vp, vp, ip, i64p, i64p, ip, ctypes.c_int64, ctypes.c_int64]
        L.or_cumsum.argtypes = [ip, vp, vp, ip, i64p, i64p, ip]
        L.or_set_threads.argtypes = [ip]
        L.or_max_threads.restype = ip
        L.or_double_to_f16.restype = ctypes.c_uint16
        L.or_double_to_f16.argtypes = [ctypes.c_double]
        L.or_double_to_bf16.restype = ctypes.c_uint16
        L.or_double_to_bf16.argtypes = [ctypes.c_double]
        _LIB = L
    return _LIB


def set_threads(n: int) -> None:
    lib().or_set_threads(int(n))


def max_threads() -> int:
    return int(lib().or_max_threads())


def code_of(nd: np.dtype) -> int:
    nd = np.dtype(nd)
    for c, v in _NP.items():
        if v == nd:
            return c
    raise TypeError(f"no musapy dtype for numpy {nd}")


def np_of(code: int) -> np.dtype:
    return _NP[code]


# ------------------------------------------------------------- promotion
_CAT = [0, 1, 1, 1, 1, 2, 2, 2, 2, 3, 3, 3, 3, 4, 4]
_W = [8, 8, 16, 32, 64, 8, 16, 32, 64, 16, 32, 64, 16, 32, 64]


def promote(a: int, b: int, all_gpu: bool = False) -> int:
    """promote / jax_promote of rust/musapy-core/src/dtype.rs:206-338."""
    if a == b:
        return a

    def int_of(w):
        return {8: I8, 16: I16, 32: I32, 64: I64}[w]

    def float_of(w):
        return {16: F16, 32: F32, 64: F64}[w]

    def complex_of(w):
        return C64 if w <= 32 else C128

    def jax(a, b):
        if a == BOOL:
            return b
        if b == BOOL:
            return a
        ca, cb, pa, pb = _CAT[a], _CAT[b], _W[a], _W[b]
        if ca == cb:
            if ca == 3 and pa == pb:
                return F32
            return a if pa >= pb else b
        if {ca, cb} == {1, 2}:
            iw = pa if ca == 1 else pb
            uw = pb if ca == 1 else pa
            return int_of(iw if iw > uw else min(uw * 2, 64))
        if ca in (1, 2) and cb == 3:
            return BF16 if b == BF16 else float_of(pb)
        if cb in (1, 2) and ca == 3:
            return BF16 if a == BF16 else float_of(pa)
        if ca in (1, 2) and cb == 4:
            return complex_of(max(pa, pb, 32))
        if cb in (1, 2) and ca == 4:
            return complex_of(max(pa, pb, 32))
        return complex_of(max(pa, pb))

    j = jax(a, b)
    if not all_gpu:
        return j
    ca, cb, pa, pb = _CAT[a], _CAT[b], _W[a], _W[b]
    if ca != cb:
        return j
    if ca == 3 and pa == pb and {a, b} == {F16, BF16}:
        return j
    return a if pa <= pb else b


# ---------------------------------------------------------------- helpers
def _i64(vals):
    vals = [int(v) for v in vals]
    return (ctypes.c_int64 * max(1, len(vals)))(*vals)


def _estrides(x: np.ndarray):
    return [s // x.itemsize for s in x.strides]


def _ptr(x: np.ndarray):
    return x.ctypes.data if x.size else None


def cast(x: np.ndarray, dst: int) -> np.ndarray:
    """cpu_cast (op_builder.rs:2052-2160) into a new contiguous array."""
    x = np.asarray(x)
    src = code_of(x.dtype)
    out = np.empty(x.shape, dtype=_NP[dst])
    if x.size:
        lib().or_cast(src, dst, _ptr(x), _ptr(out), x.ndim, _i64(x.shape), _i64(_estrides(x)))
    return out


def _as(x: np.ndarray, code: int) -> np.ndarray:
    return x if code_of(x.dtype) == code else cast(x, code)


def broadcast_shape(*shapes):
    return np.broadcast_shapes(*shapes)


def binary(op: str, a: np.ndarray, b: np.ndarray, compute: int | None = None, all_gpu: bool = False,
           out: np.ndarray | None = None) -> np.ndarray:
    """binary_elementwise on the CPU path: cast to the promoted dtype, then
    c[i] = op(a[off_a], b[off_b]) in that dtype (into `out` when given: a
    C-contiguous array of the result's shape and dtype)."""
    a, b = np.asarray(a), np.asarray(b)
    cd = compute if compute is not None else promote(code_of(a.dtype), code_of(b.dtype), all_gpu)
    a2, b2 = _as(a, cd), _as(b, cd)
    shape = broadcast_shape(a2.shape, b2.shape)
    av, bv = np.broadcast_to(a2, shape), np.broadcast_to(b2, shape)
    if out is None:
        out = np.empty(shape, dtype=_NP[cd])
    elif out.shape != tuple(shape) or out.dtype != _NP[cd] or not out.flags.c_contiguous:
        raise ValueError("binary: out must be C-contiguous with the result's shape and dtype")
    if out.size:
        lib().or_binary(OPS[op], cd, _ptr(av), _ptr(bv), _ptr(out), len(shape), _i64(shape),
                        _i64(_estrides(av)), _i64(_estrides(bv)))
    return out


def compare(op: str, a: np.ndarray, b: np.ndarray, compute: int | None = None, all_gpu: bool = False) -> np.ndarray:
    a, b = np.asarray(a), np.asarray(b)
    cd = compute if compute is not None else promote(code_of(a.dtype), code_of(b.dtype), all_gpu)
    a2, b2 = _as(a, cd), _as(b, cd)
    shape = broadcast_shape(a2.shape, b2.shape)
    av, bv = np.broadcast_to(a2, shape), np.broadcast_to(b2, shape)
    out = np.empty(shape, dtype=np.uint8)
    if out.size:
        lib().or_compare(OPS[op], cd, _ptr(av), _ptr(bv), _ptr(out), len(shape), _i64(shape),
                         _i64(_estrides(av)), _i64(_estrides(bv)))
    return out.view(np.bool_)


def unary(op: str, a: np.ndarray) -> np.ndarray:
    a = np.asarray(a)
    d = code_of(a.dtype)
    od = d
    if op == "abs" and d in (C64, C128):
        od = F32 if d == C64 else F64
    out = np.empty(a.shape, dtype=_NP[od])
    if out.size:
        lib().or_unary(OPS[op], d, _ptr(a), _ptr(out), a.ndim, _i64(a.shape), _i64(_estrides(a)))
    return out


def clamp(a: np.ndarray, lo: float, hi: float) -> np.ndarray:
    a = np.asarray(a)
    d = code_of(a.dtype)
    out = np.empty(a.shape, dtype=a.dtype)
    if out.size:
        lib().or_clamp(d, _ptr(a), _ptr(out), float(lo), float(hi), a.ndim, _i64(a.shape), _i64(_estrides(a)))
    return out


def compute_dtype(d: int, op: str) -> int:
    """reduction_compute_dtype (op_builder.rs:2209-2225)."""
    if d in (F32, F64, C64, C128):
        return d
    if d in (F16, BF16):
        return F32
    return F64 if op == "mean" else I64


def _reduce_axis(op: str, x: np.ndarray, axis: int | None, keepdims: bool) -> np.ndarray:
    """reduction_axis on the CPU device for one axis (or None)."""
    cd = compute_dtype(code_of(x.dtype), op)
    x = _as(x, cd)
    if axis is None:
        x = np.ascontiguousarray(x).reshape(-1)
        kshape, kstr, kax, L = (x.size,), [1], 0, x.size
        out_shape = (1,) * 0 if not keepdims else None
    else:
        kshape, kstr, kax, L = x.shape, _estrides(x), axis, x.shape[axis]
    out_d = I64 if op in ("argmax", "argmin") else cd
    if axis is None:
        oshape = ()
    else:
        oshape = tuple(s for i, s in enumerate(x.shape) if i != axis)
    M = int(np.prod(oshape)) if oshape else 1
    out = np.zeros(max(M, 1), dtype=_NP[out_d])
    if M > 0 and L > 0:
        lib().or_reduce(RED[op], cd, _ptr(x), _ptr(out), len(kshape), _i64(kshape), _i64(kstr), kax, L, M)
    out = out[:M].reshape(oshape) if oshape else out[:1].reshape(())
    if keepdims:
        full = list(x.shape)
        if axis is None:
            full = [1] * x.ndim if False else [1] * len(full)
        else:
            full[axis] = 1
        out = out.reshape(full)
    return out


def reduce(op: str, x: np.ndarray, axis=None, keepdims: bool = False) -> np.ndarray:
    """reduce_multi / arg_reduce_multi (reduction.rs:118-223) on the CPU path."""
    x = np.asarray(x)
    nd = x.ndim
    if axis is None:
        r = _reduce_axis(op, x, None, False)
        return r.reshape((1,) * nd) if keepdims else r
    axes = [axis] if isinstance(axis, (int, np.integer)) else list(axis)
    axes = sorted(a + nd if a < 0 else a for a in axes)
    if len(axes) == 1:
        return _reduce_axis(op, x, axes[0], keepdims)
    if op in ("argmax", "argmin"):
        perm = [i for i in range(nd) if i not in axes] + axes
        t = np.ascontiguousarray(np.transpose(x, perm))
        merged = t.reshape(t.shape[: nd - len(axes)] + (-1,))
        r = _reduce_axis(op, merged, merged.ndim - 1, keepdims)
        if keepdims:
            r = r.reshape(t.shape[: nd - len(axes)] + (1,) * len(axes))
            inv = np.argsort(perm)
            r = np.transpose(r, inv)
        return r
    cur = x
    for ax in axes:
        cur = _reduce_axis(op, cur, ax, True)
    if not keepdims:
        cur = cur.reshape(tuple(s for i, s in enumerate(cur.shape) if i not in axes))
    return cur


def cumsum(x: np.ndarray, axis=None) -> np.ndarray:
    """cumsum_op (op_builder.rs:3144-3363) on the CPU path."""
    x = np.asarray(x)
    d = code_of(x.dtype)
    cd = d if d in (F32, F64) else I64
    x = _as(x, cd)
    if axis is None:
        x = np.ascontiguousarray(x).reshape(-1)
        axis = 0
    axis = axis + x.ndim if axis < 0 else axis
    out = np.empty(x.shape, dtype=_NP[cd])
    if x.size:
        lib().or_cumsum(cd, _ptr(x), _ptr(out), x.ndim, _i64(x.shape), _i64(_estrides(x)), axis)
    return out


def _fill_values(vals: np.ndarray, dst: int) -> np.ndarray:
    """f64 values converted once with Rust `as` semantics (cpu_fill_ptr)."""
    return np.ascontiguousarray(vals.astype(np.float64)) if dst == F64 else cast(vals.astype(np.float64), dst)


def arange_len(start: float, stop: float, step: float) -> int:
    """arange_len (creation.rs:624-633)."""
    if step > 0.0 and start >= stop:
        return 0
    if step < 0.0 and start <= stop:
        return 0
    n = math.ceil((stop - start) / step)
    return int(n) if n > 0 else 0


def arange(start, stop=None, step=1, dtype: int | None = None) -> np.ndarray:
    """ms.arange on the CPU device (creation.rs:469-501, cpu_fill_ptr :324-348):
    element i = start + (i as f64) * step in f64 (no fused multiply-add), then
    `as` the dtype; float64 when any argument is a Python float, else int64
    (the binding's inference, rust/musapy-python/src/ops.rs:752-786)."""
    any_float = any(isinstance(v, float) for v in (start, stop, step))
    start, step = float(start), float(step)
    if stop is None:
        start, stop = 0.0, start
    stop = float(stop)
    if step == 0.0:
        raise ValueError("arange: step must not be zero")
    n = arange_len(start, stop, step)
    if dtype is None:
        dtype = F64 if any_float else I64
    i = np.arange(n, dtype=np.float64)
    return _fill_values(start + i * step, dtype)


def linspace(start, stop, num: int = 50, dtype: int | None = None) -> np.ndarray:
    """ms.linspace on the CPU device (creation.rs:508-521, :350-377)."""
    start, stop = float(start), float(stop)
    dtype = F64 if dtype is None else dtype
    if num == 1:
        return _fill_values(np.array([start]), dtype)
    step = (stop - start) / float(num - 1) if num > 1 else 0.0
    i = np.arange(num, dtype=np.float64)
    return _fill_values(start + i * step, dtype)


def eye(n: int, m: int | None = None, k: int = 0, dtype: int = F32) -> np.ndarray:
    """ms.eye on the CPU device (creation.rs:457-461, :378-400): 1 where
    col - row == k."""
    m = n if m is None else m
    r = np.arange(n, dtype=np.int64)[:, None]
    c = np.arange(m, dtype=np.int64)[None, :]
    return _fill_values((c - r == k).astype(np.float64), dtype)


def f16_bits(x: float) -> int:
    return int(lib().or_double_to_f16(float(x)))


def bf16_bits(x: float) -> int:
    return int(lib().or_double_to_bf16(float(x)))
