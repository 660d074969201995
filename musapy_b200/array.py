"""Device arrays: a buffer + layout (shape, element strides, element offset) +
dtype + device, the object model of rust/musapy-core/src/array.rs and
layout.rs. Device memory comes from torch's caching allocator (stream
ordered); views share the buffer and only change the layout.
"""
from __future__ import annotations

import builtins
import mmap
import numbers
from typing import Iterable, Sequence

import numpy as np
import torch

from . import dtypes as _dt
from . import errors
from . import streams as _streams

# host transfers from this size on go through the pinned staging ring
# (mpb_copy_h2d / mpb_copy_d2h); smaller ones through torch's copy
_STAGED_COPY_BYTES = 1 << 20


class Device:
    """A CUDA device. "musa:N" is accepted as an alias of "cuda:N" so that
    musapy call sites keep working. A device taken from an array carries how
    it was resolved (`resolution_source`: arg / context / input_array /
    global_default, rust/musapy-python/src/device.rs:40-90)."""

    __slots__ = ("index", "_source")

    def __init__(self, spec="cuda:0", _source=None) -> None:
        self.index = parse_device(spec)
        self._source = _source

    def __repr__(self) -> str:
        if self._source:
            return f"Device(cuda:{self.index})  # resolved from: {self._source}"
        return f"Device(cuda:{self.index})"

    @property
    def resolution_source(self):
        return self._source

    def __str__(self) -> str:
        return f"cuda:{self.index}"

    def __format__(self, fmt: str) -> str:
        return format(str(self), fmt)

    def __eq__(self, other) -> bool:
        if isinstance(other, Device):
            return self.index == other.index
        if isinstance(other, (str, int)):
            try:
                return parse_device(other) == self.index
            except errors.DeviceError:
                return False
        return NotImplemented

    def __hash__(self) -> int:
        return hash(("cuda", self.index))

    @property
    def is_cuda(self) -> bool:
        return True

    @property
    def is_musa(self) -> bool:
        """True: the accelerator device (device.rs:64-68)."""
        return True

    @property
    def musa_id(self) -> int:
        return self.index


def parse_device(spec) -> int:
    if spec is None:
        return _streams.default_device()
    if isinstance(spec, Device):
        return spec.index
    if isinstance(spec, torch.device):
        if spec.type != "cuda":
            raise errors.DeviceError(f"device {spec} is not a CUDA device")
        return spec.index or 0
    if isinstance(spec, int):
        return spec
    s = str(spec).strip().lower()
    if s in ("cuda", "musa", "gpu"):
        return 0
    for p in ("cuda:", "musa:", "gpu:"):
        if s.startswith(p):
            try:
                return int(s[len(p):])
            except ValueError:
                break
    if s == "cpu":
        raise errors.DeviceError(
            "musapy_b200 executes on CUDA devices only; the CPU path of musapy is not part of this engine"
        )
    raise errors.DeviceError(f"cannot parse device '{spec}'")


def set_default_device(spec) -> None:
    """``ms.set_default_device`` (resolution.rs:60-75): this thread's default
    device, inherited by threads that have not chosen one."""
    _streams.set_default_device(parse_device(spec))


def set_default_dtype(spec) -> None:
    _streams.set_default_dtype(_dt.parse(spec))


def default_dtype() -> _dt.Dtype:
    """The innermost ``ms.dtype`` context's dtype, else the global default."""
    return _streams.default_dtype()


def contiguous_strides(shape: Sequence[int]) -> tuple:
    st = []
    acc = 1
    for d in reversed(shape):
        st.append(acc)
        acc *= int(d)
    return tuple(reversed(st))


def _prod(xs: Iterable[int]) -> int:
    p = 1
    for x in xs:
        p *= int(x)
    return p


class Array:
    """A strided view of device memory."""

    __slots__ = ("_buf", "_shape", "_strides", "_offset", "_dtype", "_dev", "_name", "_dev_src", "_dt_src", "_ptr",
                 "_sid")

    def __init__(self, buf: torch.Tensor, shape, strides, offset: int, dtype: _dt.Dtype, device: int,
                 dev_src: str = "input_array", dt_src: str = "input_array") -> None:
        self._buf = buf  # torch uint8 tensor owning the allocation
        self._shape = tuple(int(s) for s in shape)
        self._strides = tuple(int(s) for s in strides)
        self._offset = int(offset)
        self._dtype = dtype
        self._dev = int(device)
        self._name = None
        self._dev_src = dev_src  # how the device / dtype were resolved
        self._dt_src = dt_src
        self._ptr = buf.data_ptr() + self._offset * dtype.itemsize  # device address of element [0, ..., 0]
        self._sid = buf.untyped_storage().data_ptr()  # identity of the allocation (alias checks)

    # ------------------------------------------------------------ metadata
    @property
    def shape(self) -> tuple:
        return self._shape

    @property
    def strides(self) -> tuple:
        """Element strides (may be 0 or negative for views)."""
        return self._strides

    @property
    def offset(self) -> int:
        return self._offset

    @property
    def ndim(self) -> int:
        return len(self._shape)

    @property
    def size(self) -> int:
        return _prod(self._shape)

    @property
    def dtype(self) -> _dt.Dtype:
        return self._dtype

    @property
    def device(self) -> Device:
        return Device(self._dev, self._dev_src)

    @property
    def dtype_resolution_source(self) -> str:
        """arg / context / input_array / global_default / auto_probe (array.rs:59-63)."""
        return self._dt_src

    @property
    def nbytes(self) -> int:
        return self.size * self._dtype.itemsize

    @property
    def name(self):
        return self._name

    @name.setter
    def name(self, value) -> None:
        self._name = value

    def clear_name(self) -> None:
        self._name = None

    @property
    def is_contiguous(self) -> bool:
        return self._is_c_contiguous()

    @property
    def is_0d(self) -> bool:
        return len(self._shape) == 0

    def _is_c_contiguous(self) -> bool:
        acc = 1
        for d, s in zip(reversed(self._shape), reversed(self._strides)):
            if d != 1 and s != acc:
                return False
            acc *= d
        return True

    @property
    def data_ptr(self) -> int:
        """Device address of the logical element [0, ..., 0]."""
        return self._ptr

    def _stream(self) -> int:
        return _streams.current_stream(self._dev).cuda_stream

    @property
    def stream(self):
        """The stream the array was created on (array.rs:73); for arrays that
        wrap foreign memory, the stream that last used it, else the current
        stream of its device."""
        s = getattr(self._buf, "_mpb_owner", None) or getattr(self._buf, "_mpb_stream", None)
        return s if s is not None else _streams.current_stream(self._dev)

    def __len__(self) -> int:
        if not self._shape:
            raise TypeError("len() of a 0-d array")
        return self._shape[0]

    # ------------------------------------------------------------- transfer
    def numpy(self) -> np.ndarray:
        """Copy to host as a numpy array (C order)."""
        a = self if self._is_c_contiguous() else contiguous(self)
        n = a.nbytes
        if n == 0:
            return np.zeros(a._shape, dtype=_dt.to_numpy(a._dtype))
        start = a._offset * a._dtype.itemsize
        handle = _streams.launch("numpy", a._dev, a)
        if n >= _STAGED_COPY_BYTES:
            host = _host_buffer(n)
            from ._lib import LIB, check

            with torch.cuda.device(a._dev):
                check(LIB.mpb_copy_d2h(host.ctypes.data, a._buf.data_ptr() + start, n, handle), "numpy")
        else:
            host = a._buf.narrow(0, start, n).cpu().numpy()
        return host.view(_dt.to_numpy(a._dtype)).reshape(a._shape)

    def tolist(self):
        h = self.numpy()
        if self._dtype.code == _dt.BF16:
            h = h.astype(np.float32)
        return h.tolist()

    def item(self):
        if self.size != 1:
            raise errors.ShapeError(f"item() requires exactly one element, array has {self.size}")
        return self.numpy().reshape(()).item() if self._dtype.code != _dt.BF16 else float(
            self.numpy().astype(np.float32).reshape(()))

    def torch(self) -> torch.Tensor:
        """Zero-copy torch view (strided) of this array."""
        td = _dt.to_torch(self._dtype)
        base = self._buf.view(td) if self._buf.numel() % self._dtype.itemsize == 0 else None
        if base is None:
            raise errors.InteropError("buffer size is not a multiple of the element size")
        return torch.as_strided(base, self._shape, self._strides, self._offset)

    def __dlpack__(self, stream=None):
        return self.torch().__dlpack__(stream=stream)

    def __dlpack_device__(self):
        return self.torch().__dlpack_device__()

    def to(self, device) -> "Array":
        dev = parse_device(device)
        if dev == self._dev:
            return self
        src = self if self._is_c_contiguous() else contiguous(self)
        n = src.nbytes
        buf = torch.empty(max(n, 1), dtype=torch.uint8, device=f"cuda:{dev}")
        if n:
            start = src._offset * src._dtype.itemsize
            buf[:n].copy_(src._buf.narrow(0, start, n))
        return Array(buf, src._shape, contiguous_strides(src._shape), 0, src._dtype, dev)

    # -------------------------------------------------------------- casting
    def astype(self, dtype) -> "Array":
        from . import ops

        return ops.astype(self, dtype)

    def contiguous(self) -> "Array":
        return contiguous(self)

    # --------------------------------------------------------------- dunders
    def __add__(self, o):
        from . import ops
        return ops.add(self, o)

    def __radd__(self, o):
        from . import ops
        return ops.add(o, self)

    def __sub__(self, o):
        from . import ops
        return ops.sub(self, o)

    def __rsub__(self, o):
        from . import ops
        return ops.sub(o, self)

    def __mul__(self, o):
        from . import ops
        return ops.mul(self, o)

    def __rmul__(self, o):
        from . import ops
        return ops.mul(o, self)

    def __truediv__(self, o):
        from . import ops
        return ops.div(self, o)

    def __rtruediv__(self, o):
        from . import ops
        return ops.div(o, self)

    def __pow__(self, o, modulo=None):
        from . import ops
        return ops.pow(self, o)

    def __rpow__(self, o):
        from . import ops
        return ops.pow(o, self)

    def __neg__(self):
        from . import ops
        return ops.neg(self)

    def __abs__(self):
        from . import ops
        return ops.abs(self)

    def __eq__(self, o):  # type: ignore[override]
        from . import ops
        return ops.eq(self, o)

    def __ne__(self, o):  # type: ignore[override]
        from . import ops
        return ops.ne(self, o)

    def __lt__(self, o):
        from . import ops
        return ops.lt(self, o)

    def __gt__(self, o):
        from . import ops
        return ops.gt(self, o)

    def __le__(self, o):
        from . import ops
        return ops.le(self, o)

    def __ge__(self, o):
        from . import ops
        return ops.ge(self, o)

    __hash__ = None  # type: ignore[assignment]

    def __getitem__(self, key):
        return getitem(self, key)

    def __repr__(self) -> str:
        try:
            body = np.array2string(self.numpy(), separator=", ") if self.size <= 64 else f"<{self.size} elements>"
        except Exception:  # pragma: no cover
            body = "<unavailable>"
        return f"Array({body}, dtype={self._dtype.name}, device='cuda:{self._dev}')"

    __str__ = __repr__


# ---------------------------------------------------------------- creation
def empty(shape, dtype=None, device=None) -> Array:
    if isinstance(shape, numbers.Integral):
        shape = (int(shape),)
    shape = tuple(int(s) for s in shape)
    if any(s < 0 for s in shape):
        raise errors.ShapeError(f"negative dimension in {shape}")
    d, dt_src = _streams.resolve_dtype(dtype)
    dev, dev_src = _streams.resolve_device(device)
    return _alloc(shape, d, dev, dev_src, dt_src)


_LAYOUTS: dict = {}
_TORCH_DEVICES: dict = {}
_new_object = object.__new__


def _alloc(shape: tuple, d: _dt.Dtype, dev: int, dev_src: str, dt_src: str) -> Array:
    """A fresh C-contiguous array. `shape` is a tuple of non-negative Python
    ints and `dev` a resolved device index (the per-op output path: no
    parsing, cached strides)."""
    lay = _LAYOUTS.get(shape)
    if lay is None:
        if len(_LAYOUTS) >= 4096:
            _LAYOUTS.clear()
        lay = _LAYOUTS[shape] = (contiguous_strides(shape), _prod(shape))
    tdev = _TORCH_DEVICES.get(dev)
    if tdev is None:
        tdev = _TORCH_DEVICES[dev] = torch.device("cuda", dev)
    n = lay[1] * d.itemsize
    # Round allocations up to 16 bytes so every buffer start is vector aligned.
    buf = torch.empty(max(16, (n + 15) & ~15), dtype=torch.uint8, device=tdev)
    buf._mpb_owner = _streams.current_stream(dev)  # the stream the array belongs to
    a = _new_object(Array)
    a._buf = buf
    a._shape = shape
    a._strides = lay[0]
    a._offset = 0
    a._dtype = d
    a._dev = dev
    a._name = None
    a._dev_src = dev_src
    a._dt_src = dt_src
    a._ptr = a._sid = buf.data_ptr()  # a fresh allocation starts its storage
    return a


def _has_complex(data) -> bool:
    if isinstance(data, complex):
        return True
    if isinstance(data, (list, tuple)):
        return any(_has_complex(x) for x in data)
    return False


def _host_buffer(n: int) -> np.ndarray:
    """A fresh host byte array for a device -> host copy. Large ones are an
    anonymous mapping advised for transparent huge pages: the copy then
    faults in 2 MiB pages instead of 4 KiB ones, which is most of the cost of
    filling fresh memory."""
    if n >= (64 << 20) and hasattr(mmap, "MADV_HUGEPAGE"):
        mm = mmap.mmap(-1, n, flags=mmap.MAP_PRIVATE | mmap.MAP_ANONYMOUS)
        try:
            mm.madvise(mmap.MADV_HUGEPAGE)
        except OSError:
            pass
        return np.frombuffer(mm, dtype=np.uint8)
    return np.empty(n, dtype=np.uint8)


def from_numpy(arr: np.ndarray, device=None, dtype=None) -> Array:
    """Copy a numpy array to the device (dtype kept unless given)."""
    arr = np.asarray(arr)
    d = _dt.from_numpy(arr.dtype) if dtype is None else _dt.parse(dtype)
    if _dt.to_numpy(d) != arr.dtype:
        arr = _np_cast(arr, d)
    if not arr.flags.c_contiguous:  # (np.ascontiguousarray would turn 0-d into 1-d)
        arr = arr.copy(order="C")
    out = empty(arr.shape, d, device)
    n = arr.nbytes
    if n:
        handle = _streams.launch("from_numpy", out._dev, out)
        if n >= _STAGED_COPY_BYTES:
            from ._lib import LIB, check

            with torch.cuda.device(out._dev):
                check(LIB.mpb_copy_h2d(out._buf.data_ptr(), arr.ctypes.data, n, handle), "from_numpy")
        else:
            out._buf[:n].copy_(torch.from_numpy(arr.reshape(-1).view(np.uint8)))
    return out


def _np_cast(arr: np.ndarray, d: _dt.Dtype) -> np.ndarray:
    target = _dt.to_numpy(d)
    if d.code == _dt.BF16 and target == np.dtype(np.uint16):  # no ml_dtypes: round via torch
        t = torch.from_numpy(np.ascontiguousarray(arr, dtype=np.float32)).to(torch.bfloat16)
        return t.view(torch.uint16).numpy()
    return arr.astype(target)


def array(data, dtype=None, device=None) -> Array:
    """``ms.array(data, dtype=None, device=None)`` (rust/musapy-python/src/ops.rs:30-110).

    Without ``dtype`` the default dtype (float32) is used, except that
    Python complex literals give complex128. numpy arrays and torch tensors
    keep their dtype unless ``dtype`` is given.
    """
    if isinstance(data, Array):
        return data.astype(dtype or data.dtype).to(device if device is not None else data._dev)
    if isinstance(data, torch.Tensor):
        return from_numpy(data.detach().cpu().numpy(), device, dtype)
    if isinstance(data, np.ndarray):
        return from_numpy(data, device, dtype)
    if dtype is None and _has_complex(data):
        d, dt_src = _dt.complex128, "input_array"
    else:
        d, dt_src = _streams.resolve_dtype(dtype)
    dev, dev_src = _streams.resolve_device(device)
    if d.code == _dt.BF16:
        host = _np_cast(np.asarray(data, dtype=np.float64), d)
    elif d.is_complex():
        host = np.asarray(data, dtype=_dt.to_numpy(d))
    else:
        host = np.asarray(data)
        if host.dtype.kind == "c":
            raise errors.DtypeError(f"complex data cannot be stored as {d}")
        host = host.astype(_dt.to_numpy(d))
    out = from_numpy(host, dev, d)
    out._dev_src, out._dt_src = dev_src, dt_src
    return out


def from_torch(t: torch.Tensor) -> Array:
    """Zero-copy view of a CUDA tensor's storage as an Array."""
    if not t.is_cuda:
        raise errors.DeviceError("from_torch: tensor must live on a CUDA device")
    d = _dt.from_torch(t.dtype)
    st = t.untyped_storage()
    buf = torch.empty(0, dtype=torch.uint8, device=t.device).set_(st, 0, (st.nbytes(),), (1,))
    return Array(buf, tuple(t.shape), tuple(t.stride()), t.storage_offset(), d, t.device.index or 0)


def from_dlpack(obj) -> Array:
    return from_torch(torch.from_dlpack(obj))


# -------------------------------------------------------------------- views
def _view(a: Array, shape, strides, offset) -> Array:
    """A view of `a`'s allocation (shares its buffer, pointer base and
    allocation identity)."""
    v = _new_object(Array)
    v._buf = a._buf
    v._shape = tuple(int(x) for x in shape)
    v._strides = tuple(int(x) for x in strides)
    v._offset = int(offset)
    v._dtype = a._dtype
    v._dev = a._dev
    v._name = None
    v._dev_src = a._dev_src
    v._dt_src = a._dt_src
    v._ptr = a._ptr + (v._offset - a._offset) * a._dtype.itemsize
    v._sid = a._sid
    return v


def transpose(a: Array, axes=None) -> Array:
    """Permuted view (rust/musapy-ops/src/indexing.rs:30); reverses dims by default."""
    n = a.ndim
    if axes is None:
        axes = list(range(n))[::-1]
    axes = [int(x) + n if int(x) < 0 else int(x) for x in axes]
    if sorted(axes) != list(range(n)):
        raise errors.ShapeError(f"transpose: axes {axes} are not a permutation of {n} dims")
    return _view(a, [a._shape[i] for i in axes], [a._strides[i] for i in axes], a._offset)


def permute(a: Array, dims) -> Array:
    return transpose(a, dims)


def flip(a: Array, axis=None) -> Array:
    axes = range(a.ndim) if axis is None else ([axis] if isinstance(axis, numbers.Integral) else list(axis))
    shape, strides, off = list(a._shape), list(a._strides), a._offset
    for ax in axes:
        ax = int(ax) + a.ndim if int(ax) < 0 else int(ax)
        if not 0 <= ax < a.ndim:
            raise errors.ShapeError(f"flip: axis {ax} out of range")
        if shape[ax] > 0:
            off += (shape[ax] - 1) * strides[ax]
        strides[ax] = -strides[ax]
    return _view(a, shape, strides, off)


def slice(a: Array, ranges) -> Array:  # noqa: A001 - musapy's name
    """``ms.slice(a, [[start, stop, step], ...])``: per-dim slices, leading dims."""
    shape, strides, off = list(a._shape), list(a._strides), a._offset
    for d, r in enumerate(ranges):
        start, stop, step = (list(r) + [None, None, None])[:3]
        st, sp, stp = builtins.slice(start, stop, step).indices(shape[d])
        n = len(range(st, sp, stp))
        off += st * strides[d]
        shape[d] = n
        strides[d] = strides[d] * stp
    return _view(a, shape, strides, off)


def getitem(a: Array, key) -> Array:
    if not isinstance(key, tuple):
        key = (key,)
    if any(k is Ellipsis for k in key):
        i = key.index(Ellipsis)
        fill = a.ndim - (len(key) - 1)
        key = key[:i] + (builtins.slice(None),) * fill + key[i + 1:]
    shape, strides, off = [], [], a._offset
    d = 0
    for k in key:
        if k is None:
            shape.append(1)
            strides.append(0)
            continue
        if d >= a.ndim:
            raise errors.ShapeError("too many indices")
        if isinstance(k, numbers.Integral):
            k = int(k)
            if k < 0:
                k += a._shape[d]
            if not 0 <= k < a._shape[d]:
                raise errors.ShapeError(f"index {k} out of range for dim {d} of extent {a._shape[d]}")
            off += k * a._strides[d]
        elif isinstance(k, builtins.slice):
            st, sp, stp = k.indices(a._shape[d])
            shape.append(len(range(st, sp, stp)))
            strides.append(a._strides[d] * stp)
            off += st * a._strides[d]
        else:
            raise errors.ShapeError(f"unsupported index {k!r}")
        d += 1
    shape += list(a._shape[d:])
    strides += list(a._strides[d:])
    return _view(a, shape, strides, off)


def index_select(a: Array, axis: int, index: int) -> Array:
    """Drop `axis` by selecting one position (indexing.rs index_select)."""
    axis = axis + a.ndim if axis < 0 else axis
    if not 0 <= index < a._shape[axis]:
        raise errors.ShapeError(f"index {index} out of range")
    shape = list(a._shape)
    strides = list(a._strides)
    off = a._offset + index * strides[axis]
    del shape[axis]
    del strides[axis]
    return _view(a, shape, strides, off)


def reshape(a: Array, shape) -> Array:
    if isinstance(shape, numbers.Integral):
        shape = (int(shape),)
    shape = list(shape)
    if shape.count(-1) > 1:
        raise errors.ShapeError("reshape: at most one -1")
    if -1 in shape:
        rest = _prod(s for s in shape if s != -1)
        shape[shape.index(-1)] = a.size // rest if rest else 0
    if _prod(shape) != a.size:
        raise errors.ShapeError(f"reshape: cannot reshape {a.shape} into {tuple(shape)}")
    src = a if a._is_c_contiguous() else contiguous(a)
    return _view(src, shape, contiguous_strides(shape), src._offset)


def squeeze(a: Array, axis=None) -> Array:
    keep = [i for i, s in enumerate(a._shape) if not (s == 1 and (axis is None or i == axis % max(1, a.ndim)))]
    return _view(a, [a._shape[i] for i in keep], [a._strides[i] for i in keep], a._offset)


def broadcast_to(a: Array, shape) -> Array:
    shape = tuple(int(s) for s in shape)
    from ._lib import LIB, i64arr

    st = i64arr([0] * len(shape))
    LIB.mpb_broadcast_strides(a.ndim, i64arr(a._shape), i64arr(a._strides), len(shape), i64arr(shape), st)
    return _view(a, shape, list(st)[: len(shape)], a._offset)


def contiguous(a: Array) -> Array:
    """C-contiguous copy (indexing.rs:181; musapy_copy_transpose2d_* for 2-D
    transposes) through the engine's strided / tiled copy kernel."""
    from . import ops

    return ops._cast_into(a, a._dtype)
