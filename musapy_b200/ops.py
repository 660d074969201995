"""musapy's operator surface over the B200 engine.

Each op follows the 3-phase skeleton of rust/musapy-ops/src/op_builder.rs:
phase A validates (device, broadcast, promotion, dtype whitelist, out=,
alias), phase B launches one call of the C-ABI (libmusapy_b200), phase C
wraps the output. Differences from the reference, all deliberate:

* promotion casts are fused into the kernels' loads instead of materialising
  a converted copy (op_builder.rs:410-417);
* f16 / bf16 are accepted for arithmetic, comparison, unary math, clamp,
  casts and reductions (the reference rejects them: op_builder.rs:904-962,
  rust/musapy-python/src/ops.rs:491-493), and integer comparisons too;
* cumsum has no 256^3 length limit (op_builder.rs:3291-3300);
* multi-axis sum/prod/max/min/mean reduce in one pass instead of one pass per
  axis (rust/musapy-ops/src/reduction.rs:118-155); max/min/argmax/argmin
  results are identical, sums agree within the float tolerance.
"""
from __future__ import annotations

import builtins
import math
import numbers

import numpy as np
import torch

from . import dtypes as _dt
from . import errors
from . import streams as _streams
from ._lib import LIB, NATIVE, OPS, RED_OPS, check, i64arr
from .array import Array, _alloc, contiguous_strides, empty, parse_device, reshape

_ARITH_OK = {_dt.F32, _dt.F64, _dt.C64, _dt.C128, _dt.F16, _dt.BF16}
_UNARY_OK = {_dt.F32, _dt.F64, _dt.F16, _dt.BF16}


def _stream(dev: int) -> int:
    return _streams.current_stream(dev).cuda_stream


def _out(shape, d, dev: int) -> Array:
    """An op's result: device and dtype follow the inputs (input_array in
    musapy's resolution chain, resolution.rs:224-230)."""
    return _alloc(shape, d, dev, "input_array", "input_array")


def _launch(op: str, dev: int, *arrays) -> int:
    """CUDA stream for a launch of `op` touching `arrays` on `dev`: waits for
    other streams' pending work on those buffers, checks the stream is not
    poisoned and records the op context (streams.launch)."""
    return _streams.launch(op, dev, *arrays)


def _scalar_like(x, other: Array) -> Array:
    """Python scalar -> 0-d device array (dtype of the array operand, or
    complex128/float64 when the scalar cannot be represented)."""
    if isinstance(x, Array):
        return x
    if isinstance(x, (numbers.Number, np.generic)):
        d = other.dtype
        if isinstance(x, complex) and not d.is_complex():
            d = _dt.complex128
        elif isinstance(x, float) and not (d.is_floating() or d.is_complex()):
            d = _dt.float64
        v = complex(x)
        if isinstance(x, (bool, np.bool_)) or (isinstance(x, numbers.Integral) and builtins.abs(int(x)) <= (1 << 53)) \
                or not isinstance(x, numbers.Integral):
            # written on the device by the fill kernel: no host -> device copy
            # (which would wait for the host) in the middle of a stream of ops
            return full((), v if d.is_complex() else v.real, d, other._dev)
        from .array import array as _array

        return _array(x, dtype=d, device=other._dev)  # integers beyond 2^53: exact host conversion
    raise TypeError(f"unsupported operand {type(x).__name__}")


def _coerce_pair(a, b):
    if not isinstance(a, Array) and not isinstance(b, Array):
        raise TypeError("at least one operand must be a musapy Array")
    if not isinstance(a, Array):
        a = _scalar_like(a, b)
    if not isinstance(b, Array):
        b = _scalar_like(b, a)
    return a, b


def _broadcast_shape(a: Array, b: Array) -> tuple:
    """broadcast_shape (broadcast.rs:24-55): align from the right; extents
    must match or be 1. (Same rule as mpb_broadcast_shape, without a library
    call on the per-op path; the two are tested against each other.)"""
    sa, sb = a._shape, b._shape
    if sa == sb:
        return sa
    na, nb = len(sa), len(sb)
    n = na if na > nb else nb
    out = []
    for i in range(n):
        da = sa[i - n + na] if i >= n - na else 1
        db = sb[i - n + nb] if i >= n - nb else 1
        if da == db or db == 1:
            out.append(da)
        elif da == 1:
            out.append(db)
        else:
            raise errors.ShapeError(f"broadcast: incompatible shapes {list(sa)} and {list(sb)}")
    return tuple(out)


def _bstrides(a: Array, shape) -> tuple:
    """broadcast_strides (broadcast.rs:57-92): the view's strides on `shape`,
    0 where a dim is added or stretched from 1."""
    if a._shape == shape:
        return a._strides
    n, na = len(shape), len(a._shape)
    st = []
    for i in range(n):
        j = i - (n - na)
        if j < 0 or (a._shape[j] == 1 and shape[i] != 1):
            st.append(0)
        else:
            st.append(a._strides[j])
    return tuple(st)


def _check_out(out: Array, shape, dtype: _dt.Dtype, dev: int, name: str) -> None:
    if out._shape != tuple(shape):
        raise errors.ShapeError(f"{name}: out shape {list(out.shape)} != expected {list(shape)}")
    if out._dtype != dtype:
        raise errors.DtypeError(f"{name}: out dtype {out.dtype} != expected {dtype}")
    if out._dev != dev:
        raise errors.DeviceError(f"{name}: out device cuda:{out._dev} != input device cuda:{dev}")
    if not out._is_c_contiguous():
        raise errors.ShapeError(f"{name}: out must be C-contiguous")


def _alias(out: Array, *ins: Array) -> bool:
    """musapy's AliasDetected rule: `out` shares its allocation with an input."""
    sid = out._sid
    for x in ins:
        if x._sid == sid:
            return True
    return False


def _same_device(name: str, *arrs: Array) -> int:
    dev = arrs[0]._dev
    for x in arrs[1:]:
        if x._dev != dev:
            raise errors.DeviceError(f"{name}: device mismatch cuda:{dev} vs cuda:{x._dev}")
    return dev


# ------------------------------------------------------------------ binary
def _binary(name: str, a, b, out):
    a, b = _coerce_pair(a, b)
    dev = _same_device(name, a, b)
    shape = _broadcast_shape(a, b)
    d = _dt.promote(a.dtype, b.dtype, all_gpu=True)
    if d.code not in _ARITH_OK:
        raise errors.DtypeError(
            f"{name}: promoted dtype {d} not supported (compute whitelist: float16/bfloat16/float32/float64/complex64/complex128)"
        )
    if name == "pow" and d.is_complex():
        raise errors.DtypeError(f"pow: not supported for complex dtype {d}")
    if out is not None:
        _check_out(out, shape, d, dev, name)
        if _alias(out, a, b):
            raise errors.MemoryError("out= aliases an input buffer (AliasDetected)")
        res = out
    else:
        res = _out(shape, d, dev)
    rc = NATIVE.elementwise_bc(
        OPS[name], shape, a._ptr, a._dtype.code, a._shape, a._strides, b._ptr, b._dtype.code, b._shape, b._strides,
        res._ptr, d.code, d.code, 0.0, 0.0, _launch(name, dev, a, b, res),
    )
    check(rc, name)
    return res


def add(a, b, out=None):
    """``ms.add(a, b, out=None)`` (ops.rs:106; op_builder.rs:315)."""
    return _binary("add", a, b, out)


def sub(a, b, out=None):
    return _binary("sub", a, b, out)


def mul(a, b, out=None):
    return _binary("mul", a, b, out)


def div(a, b, out=None):
    return _binary("div", a, b, out)


def pow(a, b, out=None):  # noqa: A001
    return _binary("pow", a, b, out)


# ------------------------------------------------------------- comparisons
def _compare(name: str, a, b, out):
    a, b = _coerce_pair(a, b)
    dev = _same_device(name, a, b)
    shape = _broadcast_shape(a, b)
    d = _dt.promote(a.dtype, b.dtype, all_gpu=True)
    if d.is_complex() and name not in ("eq", "ne"):
        raise errors.DtypeError(f"{name}: not supported for complex dtype {d} (complex has no total order)")
    if out is not None:
        _check_out(out, shape, _dt.bool_, dev, name)
        if _alias(out, a, b):
            raise errors.MemoryError("out= aliases an input buffer (AliasDetected)")
        res = out
    else:
        res = _out(shape, _dt.bool_, dev)
    rc = NATIVE.elementwise_bc(
        OPS[name], shape, a._ptr, a._dtype.code, a._shape, a._strides, b._ptr, b._dtype.code, b._shape, b._strides,
        res._ptr, _dt.BOOL, d.code, 0.0, 0.0, _launch(name, dev, a, b, res),
    )
    check(rc, name)
    return res


def eq(a, b, out=None):
    """``ms.eq`` (op_builder.rs:1338): bool output, compare in the promoted dtype."""
    return _compare("eq", a, b, out)


def ne(a, b, out=None):
    return _compare("ne", a, b, out)


def lt(a, b, out=None):
    return _compare("lt", a, b, out)


def gt(a, b, out=None):
    return _compare("gt", a, b, out)


def le(a, b, out=None):
    return _compare("le", a, b, out)


def ge(a, b, out=None):
    return _compare("ge", a, b, out)


# ------------------------------------------------------------------- unary
def _unary(name: str, a: Array, out, p0: float = 0.0, p1: float = 0.0):
    if not isinstance(a, Array):
        raise TypeError(f"{name}: expected a musapy Array")
    d = a.dtype
    complex_ok = name in ("neg", "abs")
    if not (d.code in _UNARY_OK or (complex_ok and d.is_complex())):
        raise errors.DtypeError(f"{name}: dtype {d} not supported")
    out_d = d
    if name == "abs" and d.is_complex():
        out_d = _dt.float32 if d.code == _dt.C64 else _dt.float64
    dev = a._dev
    if out is not None:
        _check_out(out, a.shape, out_d, dev, name)
        if _alias(out, a):
            raise errors.MemoryError("out= aliases an input buffer (AliasDetected)")
        res = out
    else:
        res = _out(a.shape, out_d, dev)
    rc = NATIVE.elementwise(
        OPS[name], a._shape, a.data_ptr, d.code, a._strides, None, 0, None, res.data_ptr, out_d.code, d.code,
        float(p0), float(p1), _launch(name, dev, a, res),
    )
    check(rc, name)
    return res


def sin(a, out=None):
    return _unary("sin", a, out)


def cos(a, out=None):
    return _unary("cos", a, out)


def exp(a, out=None):
    return _unary("exp", a, out)


def log(a, out=None):
    return _unary("log", a, out)


def abs(a, out=None):  # noqa: A001
    return _unary("abs", a, out)


def sign(a, out=None):
    return _unary("sign", a, out)


def neg(a, out=None):
    return _unary("neg", a, out)


def clamp(a, lo, hi, out=None):
    """``ms.clamp(a, lo, hi)`` (op_builder.rs:740): NaN passes through; bounds
    are rounded to the array dtype first."""
    if isinstance(a, Array) and a.dtype.is_complex():
        raise errors.DtypeError(f"clamp: dtype {a.dtype} not supported")
    return _unary("clamp", a, out, float(lo), float(hi))


# ------------------------------------------------------------------- casts
def _validate_cast(src: _dt.Dtype, dst: _dt.Dtype) -> None:
    """validate_cast_pair (op_builder.rs:904-962), widened to the 16-bit
    floats, bool and every integer width; complex -> real stays rejected."""
    if src.is_complex() and not dst.is_complex():
        raise errors.DtypeError(f"cast: {src} -> {dst} not supported (complex -> real)")
    if src.code == _dt.C128 and dst.code == _dt.C64:
        raise errors.DtypeError("cast: complex128 -> complex64 not supported")


def _cast_into(a: Array, d: _dt.Dtype, out: Array | None = None) -> Array:
    dev = a._dev
    res = out if out is not None else _out(a.shape, d, dev)
    rc = NATIVE.elementwise(
        OPS["cast"], a._shape, a.data_ptr, a.dtype.code, a._strides, None, 0, None, res.data_ptr, d.code, d.code,
        0.0, 0.0, _launch("cast", dev, a, res),
    )
    check(rc, "cast")
    return res


def astype(a: Array, dtype, out=None) -> Array:
    """``Array.astype`` (op_builder.rs:1130): a new contiguous array of `dtype`."""
    d = _dt.parse(dtype)
    if a.dtype != d:
        _validate_cast(a.dtype, d)
    if out is not None:
        _check_out(out, a.shape, d, a._dev, "astype")
        if _alias(out, a):
            raise errors.MemoryError("out= aliases an input buffer (AliasDetected)")
    return _cast_into(a, d, out)


def contiguous(a: Array, out=None) -> Array:
    """``ms.contiguous`` (indexing.rs:181): a C-contiguous copy of a view
    (tiled transpose through shared memory when the view's unit stride is on
    an outer dim). ``out=`` receives the copy instead of a new array."""
    if not isinstance(a, Array):
        raise TypeError("contiguous: expected a musapy Array")
    if out is not None:
        _check_out(out, a.shape, a.dtype, a._dev, "contiguous")
        if _alias(out, a):
            raise errors.MemoryError("out= aliases an input buffer (AliasDetected)")
    return _cast_into(a, a.dtype, out)


# -------------------------------------------------------------- reductions
def _resolve_axes(axis, ndim: int) -> list:
    """resolve_axes (rust/musapy-ops/src/reduction.rs:45-75): normalise
    negatives, reject out-of-range and duplicates, sort ascending."""
    if axis is None:
        return []
    axs = [axis] if isinstance(axis, numbers.Integral) else list(axis)
    out = []
    for ax in axs:
        ax = int(ax)
        n = ax + ndim if ax < 0 else ax
        if n < 0 or n >= ndim:
            raise errors.ShapeError(f"axis {ax} is out of bounds for array of dimension {ndim}")
        out.append(n)
    out.sort()
    for x, y in zip(out, out[1:]):
        if x == y:
            raise errors.ShapeError(f"duplicate value in 'axis' argument: {x}")
    return out


def _compute_dtype(d: _dt.Dtype, kernel: str) -> _dt.Dtype:
    """reduction_compute_dtype (op_builder.rs:2209-2225); 16-bit floats
    accumulate in f32 (an extension)."""
    if d.code in (_dt.F32, _dt.F16, _dt.BF16):
        return _dt.float32
    if d.code == _dt.F64:
        return _dt.float64
    if d.is_complex():
        return d
    return _dt.float64 if kernel == "mean" else _dt.int64


def _widen_int(a: Array) -> Array:
    """Integer inputs narrower than 64 bits (and bool) are widened to int64
    first, as musapy's cast_array does (op_builder.rs:2435-2438)."""
    if a.dtype.is_integer() and a.dtype.code not in (_dt.I64, _dt.U64) or a.dtype.code == _dt.BOOL:
        return _cast_into(a, _dt.int64)
    return a


def _reduce(kernel: str, a: Array, axis, keepdims: bool, out):
    if not isinstance(a, Array):
        raise TypeError(f"{kernel}: expected a musapy Array")
    if a.dtype.is_complex() and kernel in ("max", "min", "argmax", "argmin"):
        raise errors.DtypeError(
            f"{kernel}: ordering reduction not supported for complex dtype {a.dtype} (complex has no total order)"
        )
    axes = _resolve_axes(axis, a.ndim)
    if (kernel in ("max", "min") and axis is not None and len(axes) > 1
            and a.dtype.code in (_dt.F16, _dt.BF16, _dt.F32, _dt.F64)):
        # reduce_multi (reduction.rs:118-223) reduces one axis at a time, in
        # ascending order. For float max/min that order is visible: a NaN at
        # the start of an inner run, or the sign of a zero extremum, decides
        # the outcome per pass, so the passes are kept. The last pass writes
        # into `out` (through a keepdims-shaped view of it) when one is given.
        kshape = tuple(1 if i in axes else s for i, s in enumerate(a.shape))
        rshape = kshape if keepdims else tuple(s for i, s in enumerate(a.shape) if i not in axes)
        if out is not None:
            _check_out(out, rshape, a.dtype, a._dev, kernel)
            if _alias(out, a):
                raise errors.MemoryError("out= aliases an input buffer (AliasDetected)")
        cur = a
        axs = sorted(axes)
        for ax in axs[:-1]:
            cur = _reduce(kernel, cur, ax, True, None)
        cur = _reduce(kernel, cur, axs[-1], True, reshape(out, kshape) if out is not None else None)
        if out is not None:
            return out
        return cur if keepdims else reshape(cur, rshape)
    red = axes if axes else list(range(a.ndim))
    is_arg = kernel in ("argmax", "argmin")
    cd = _compute_dtype(a.dtype, kernel)
    if is_arg:
        out_d = _dt.int64
    elif a.dtype.code in (_dt.F16, _dt.BF16):
        out_d = a.dtype
    else:
        out_d = cd
    if axis is None:
        out_shape = (1,) * a.ndim if keepdims else ()
    else:
        out_shape = tuple(1 if i in red else s for i, s in enumerate(a.shape) if keepdims or i not in red)
    dev = a._dev
    L = 1
    for i in red:
        L *= a.shape[i]
    M = 1
    for s in out_shape:
        M *= s
    if out is not None:
        _check_out(out, out_shape, out_d, dev, kernel)
        if _alias(out, a):
            raise errors.MemoryError("out= aliases an input buffer (AliasDetected)")
        res = out
    else:
        res = _out(out_shape, out_d, dev)
    if M == 0:
        return res
    if L == 0:
        if kernel in ("max", "min", "argmax", "argmin"):
            raise errors.ShapeError(f"{kernel}: zero-size reduction has no identity")
        fillv = {"sum": 0.0, "prod": 1.0, "mean": float("nan")}[kernel]
        check(NATIVE.elementwise(OPS["fill"], out_shape, None, 0, None, None, 0, None, res.data_ptr, out_d.code,
                                 out_d.code, fillv, 0.0, _launch("fill", dev, res)), "fill")
        return res
    src = _widen_int(a)
    in_code = src.dtype.code
    if in_code == _dt.U64 and kernel in ("max", "min", "argmax", "argmin"):
        in_code = _dt.U64
    mask = 0
    for i in red:
        mask |= 1 << i
    op = RED_OPS[kernel]
    shape, strides, ptr = src._shape, src._strides, src.data_ptr
    nbytes = NATIVE.reduce_scratch_bytes(op, shape, strides, ptr, in_code, mask, cd.code)
    scratch = torch.empty(nbytes, dtype=torch.uint8, device=f"cuda:{dev}") if nbytes else None
    rc = NATIVE.reduce(
        op, shape, strides, ptr, in_code, mask, res.data_ptr, out_d.code, cd.code, 1,
        scratch.data_ptr() if scratch is not None else None, nbytes, _launch(kernel, dev, src, res),
    )
    check(rc, kernel)
    return res


def sum(a, axis=None, keepdims=False, out=None):  # noqa: A001
    """``ms.sum`` (rust/musapy-ops/src/reduction.rs:81): integers accumulate
    in int64, floats keep their dtype."""
    return _reduce("sum", a, axis, keepdims, out)


def prod(a, axis=None, keepdims=False, out=None):
    return _reduce("prod", a, axis, keepdims, out)


def max(a, axis=None, keepdims=False, out=None):  # noqa: A001
    return _reduce("max", a, axis, keepdims, out)


def min(a, axis=None, keepdims=False, out=None):  # noqa: A001
    return _reduce("min", a, axis, keepdims, out)


def mean(a, axis=None, keepdims=False, out=None):
    """``ms.mean``: integers average in float64; the divisor is the true
    element count."""
    return _reduce("mean", a, axis, keepdims, out)


def argmax(a, axis=None, keepdims=False, out=None):
    """``ms.argmax`` (reduction.rs:160-223): int64 index of the first maximum;
    several axes index the flattened reduced axes (NumPy 2 semantics)."""
    return _reduce("argmax", a, axis, keepdims, out)


def argmin(a, axis=None, keepdims=False, out=None):
    return _reduce("argmin", a, axis, keepdims, out)


def cumsum(a, axis=None, out=None):
    """``ms.cumsum`` (op_builder.rs:3144): inclusive prefix sum; axis=None
    flattens; integers accumulate in int64."""
    if not isinstance(a, Array):
        raise TypeError("cumsum: expected a musapy Array")
    d = a.dtype
    if d.code in (_dt.F32, _dt.F64):
        cd = d
    elif d.is_integer() or d.code == _dt.BOOL:
        cd = _dt.int64
    else:
        raise errors.DtypeError(f"cumsum: dtype {d} not supported")
    if axis is None:
        src = a if a._is_c_contiguous() else contiguous(a)
        from .array import _view

        src = _view(src, (src.size,), (1,), src._offset)
        ax = 0
    else:
        ax = _resolve_axes(axis, a.ndim)[0]
        src = a
    shape = src.shape
    dev = a._dev
    if out is not None:
        _check_out(out, shape, cd, dev, "cumsum")
        if _alias(out, a):
            raise errors.MemoryError("out= aliases an input buffer (AliasDetected)")
        res = out
    else:
        res = _out(shape, cd, dev)
    if src.size == 0:
        return res
    shape_c, strides_c = i64arr(shape), i64arr(src.strides)
    nbytes = LIB.mpb_cumsum_scratch_bytes(src.ndim, shape_c, strides_c, src.data_ptr, d.code, ax, res.data_ptr, cd.code)
    scratch = torch.empty(nbytes, dtype=torch.uint8, device=f"cuda:{dev}") if nbytes else None
    rc = LIB.mpb_cumsum(src.ndim, shape_c, strides_c, src.data_ptr, d.code, ax, res.data_ptr, cd.code,
                        scratch.data_ptr() if scratch is not None else None, nbytes, _launch("cumsum", dev, src, res))
    check(rc, "cumsum")
    if scratch is not None and _CHECK_SCAN_STATUS[0]:
        check(LIB.mpb_cumsum_status(scratch.data_ptr(), _stream(dev)), "cumsum")
    return res


# Reading the look-back status word synchronises the stream; tests turn it on.
_CHECK_SCAN_STATUS = [False]


def set_scan_status_check(on: bool) -> None:
    _CHECK_SCAN_STATUS[0] = bool(on)


# ---------------------------------------------------------------- creation
def full(shape, fill_value, dtype=None, device=None) -> Array:
    res = empty(shape, dtype, device)
    v = complex(fill_value)
    check(NATIVE.elementwise(OPS["fill"], res._shape, None, 0, None, None, 0, None, res.data_ptr, res.dtype.code,
                             res.dtype.code, v.real, v.imag, _launch("fill", res._dev, res)), "fill")
    return res


def zeros(shape, dtype=None, device=None) -> Array:
    return full(shape, 0.0, dtype, device)


def ones(shape, dtype=None, device=None) -> Array:
    return full(shape, 1.0, dtype, device)


def zeros_like(a: Array) -> Array:
    return full(a.shape, 0.0, a.dtype, a._dev)


def ones_like(a: Array) -> Array:
    return full(a.shape, 1.0, a.dtype, a._dev)


def _arange_len(start: float, stop: float, step: float) -> int:
    """arange_len (creation.rs:624-633)."""
    if step > 0.0 and start >= stop:
        return 0
    if step < 0.0 and start <= stop:
        return 0
    n = math.ceil((stop - start) / step)
    return int(n) if n > 0 else 0


def arange(start, stop=None, step=1, dtype=None, device=None) -> Array:
    """``ms.arange`` (creation.rs:469-501): ``arange(stop)`` or
    ``arange(start, stop, step)``; float64 when any argument is a Python
    float, int64 otherwise (rust/musapy-python/src/ops.rs:752-786), unless
    ``dtype`` is given. Element i is start + i*step evaluated in f64 and
    converted once, as the CPU path does."""
    any_float = any(isinstance(v, float) for v in (start, stop, step))
    start, step = float(start), float(step)
    if stop is None:
        start, stop = 0.0, start
    stop = float(stop)
    if step == 0.0:
        raise errors.ShapeError("arange: step must not be zero")
    n = _arange_len(start, stop, step)
    if dtype is None:
        dtype = _dt.float64 if any_float else _dt.int64
    res = empty((n,), dtype, device)
    check(LIB.mpb_arange(res.data_ptr, res.dtype.code, n, start, step, _launch("arange", res._dev, res)), "arange")
    return res


def linspace(start, stop, num=50, dtype=None, device=None) -> Array:
    """``ms.linspace`` (creation.rs:508-521): ``num`` evenly spaced values from
    start to stop inclusive, float64 unless ``dtype`` is given."""
    num = int(num)
    if num < 0:
        raise errors.ShapeError(f"linspace: num must be non-negative, got {num}")
    res = empty((num,), _dt.float64 if dtype is None else dtype, device)
    check(LIB.mpb_linspace(res.data_ptr, res.dtype.code, num, float(start), float(stop), _launch("linspace", res._dev, res)),
          "linspace")
    return res


def eye(n, m=None, k=0, dtype=None, device=None) -> Array:
    """``ms.eye`` (creation.rs:457-461): an (n, m) matrix with ones on the
    diagonal shifted by k (k > 0 above, k < 0 below); m defaults to n."""
    n = int(n)
    m = n if m is None else int(m)
    if n < 0 or m < 0:
        raise errors.ShapeError(f"eye: negative shape ({n}, {m})")
    res = empty((n, m), dtype, device)
    check(LIB.mpb_eye(res.data_ptr, res.dtype.code, n, m, int(k), _launch("eye", res._dev, res)), "eye")
    return res
