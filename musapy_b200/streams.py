"""Streams: ``ms.Stream``, the ``ms.stream`` / ``ms.device`` / ``ms.dtype``
context managers, cross-stream ordering and stream poisoning.

musapy keeps per-buffer read/write events so that an op on one stream waits
for the work other streams still have on its inputs and outputs
(rust/musapy-core/src/buffer.rs:225-326, ADR L1-8), and marks a stream
poisoned when an asynchronous fault surfaces at synchronize, reporting the
op that was running (stream.rs:311-414). Here a stream is a CUDA stream (a
torch.cuda.Stream, so torch's caching allocator orders frees on it) and the
bookkeeping is per buffer: every buffer remembers the last stream that used
it; an op on stream S touching a buffer last used on P != S makes S wait for
P's work so far (an event recorded on P, waited on S: no host sync) and tells
the allocator the buffer is in use on S. That orders read-after-write,
write-after-read and write-after-write across streams.

Poisoning: ``Stream.synchronize`` turns an asynchronous CUDA error into
``StreamError`` naming the ops launched on the stream since its last
successful synchronize (the op context), and every later op on that stream
raises ``StreamError`` before launching anything.
"""
from __future__ import annotations

import collections
import itertools
import threading

import torch

from . import dtypes as _dt
from . import errors

_ids = itertools.count(1)
_tls = threading.local()
# one Stream object per CUDA stream handle, so that ids and poison persist
_wrappers: dict = {}
_wrappers_lock = threading.Lock()

OP_CONTEXT_DEPTH = 32


def _stack(name: str) -> list:
    st = getattr(_tls, name, None)
    if st is None:
        st = []
        setattr(_tls, name, st)
    return st


class Stream:
    """``ms.Stream(device=None, priority=0)`` (rust/musapy-python/src/stream.rs:14-90).

    ``device`` defaults to the current default device ("cpu" in musapy; this
    engine has CUDA devices only). ``priority`` is the CUDA stream priority
    (lower is higher priority, as in CUDA)."""

    def __init__(self, device=None, priority: int = 0, _torch_stream=None) -> None:
        from .array import parse_device

        self._dev = parse_device(device if device is not None else default_device())
        self._priority = int(priority)
        self._torch = _torch_stream if _torch_stream is not None else torch.cuda.Stream(
            device=f"cuda:{self._dev}", priority=self._priority)
        self._handle = self._torch.cuda_stream
        self._id = next(_ids)
        self._poison = None
        self._ops = collections.deque(maxlen=OP_CONTEXT_DEPTH)
        with _wrappers_lock:
            _wrappers[(self._dev, self._torch.cuda_stream)] = self

    # ------------------------------------------------------------ properties
    @property
    def priority(self) -> int:
        return self._priority

    @property
    def device(self):
        from .array import Device

        return Device(self._dev)

    @property
    def id(self) -> int:
        return self._id

    @property
    def is_poisoned(self) -> bool:
        return self._poison is not None

    @property
    def pending_count(self) -> int:
        """Ops launched since the last synchronize that may still be running."""
        if not self._ops:
            return 0
        try:
            done = self._torch.query()
        except RuntimeError:
            done = False
        return 0 if done else len(self._ops)

    @property
    def cuda_stream(self) -> int:
        return self._handle

    @property
    def torch_stream(self):
        return self._torch

    # --------------------------------------------------------------- control
    def synchronize(self) -> None:
        """Wait for every op on the stream; an asynchronous fault becomes
        StreamError with the op context and poisons the stream."""
        self.check()
        try:
            self._torch.synchronize()
        except RuntimeError as e:
            self._poison = (f"stream {self._id} on cuda:{self._dev} poisoned: {e}; ops since the last "
                            f"synchronize: {self.op_context() or 'none recorded'}")
            raise errors.StreamError(self._poison) from e
        self._ops.clear()

    def check(self) -> None:
        if self._poison is not None:
            raise errors.StreamError(self._poison)

    def op_context(self) -> str:
        return "; ".join(self._ops)

    def _note(self, op: str) -> None:
        self._ops.append(op)

    def __eq__(self, other) -> bool:
        return isinstance(other, Stream) and other._dev == self._dev and other._handle == self._handle

    def __hash__(self) -> int:
        return hash((self._dev, self._handle))

    def __repr__(self) -> str:
        return f"Stream(device=cuda:{self._dev}, priority={self._priority}, id={self._id})"


def _wrap(dev: int, ts) -> Stream:
    key = (dev, ts.cuda_stream)
    with _wrappers_lock:
        s = _wrappers.get(key)
    if s is None:
        s = Stream(dev, getattr(ts, "priority", 0), _torch_stream=ts)
    return s


_raw_stream = getattr(torch._C, "_cuda_getCurrentRawStream", None)


def current_stream(dev: int) -> Stream:
    """The stream ops on `dev` run on: the innermost ``ms.stream`` context for
    that device, else torch's current stream of the device (so torch stream
    contexts and CUDA graph capture are honoured)."""
    st = getattr(_tls, "streams", None)
    if st:
        for s in reversed(st):
            if s._dev == dev:
                return s
    if _raw_stream is not None and _wrappers:
        # the handle alone is cheap; torch builds a Stream object per call
        try:
            s = _wrappers.get((dev, _raw_stream(dev)))
        except RuntimeError:  # CUDA not usable: torch's own call raises below
            s = None
        if s is not None:
            return s
    return _wrap(dev, torch.cuda.current_stream(dev))


def launch(op: str, dev: int, *arrays) -> int:
    """Prepare a launch of `op` on the current stream of `dev` touching
    `arrays` (inputs and outputs): poison check, cross-stream waits, allocator
    stream bookkeeping, op context. Returns the CUDA stream handle.

    Each buffer remembers the Stream that last used it (`_mpb_stream`); the
    Stream objects are unique per CUDA stream, so the common case - the same
    stream again - is one identity test."""
    s = current_stream(dev)
    if s._poison is not None:
        raise errors.StreamError(s._poison)
    capturing = None
    for x in arrays:
        if x is None:
            continue
        buf = x._buf
        last = getattr(buf, "_mpb_stream", None)
        if last is s:
            continue
        if last is not None and last._handle != s._handle:
            if capturing is None:
                capturing = _capturing(s._torch)
            if capturing:
                # inside CUDA graph capture a wait on uncaptured work is not
                # allowed; the capturing code orders its inputs beforehand
                continue
            s._torch.wait_stream(last._torch)
            buf.record_stream(s._torch)
        if not capturing:
            buf._mpb_stream = s
    s._ops.append(op)
    return s._handle


def _capturing(ts) -> bool:
    """Is `ts` (a torch CUDA stream) capturing a CUDA graph?"""
    try:
        with torch.cuda.stream(ts):
            return torch.cuda.is_current_stream_capturing()
    except (RuntimeError, AttributeError, TypeError):
        return False


def mark(dev: int, *arrays) -> None:
    """Record that `arrays` were just written on the current stream of `dev`
    by a torch operation (a copy), without waiting on anything."""
    s = current_stream(dev)
    for x in arrays:
        x._buf._mpb_stream = s


# ----------------------------------------------------- context managers
class _StreamContext:
    """``with ms.stream(s):`` (rust/musapy-python/src/lib.rs:126-131)."""

    def __init__(self, stream: Stream) -> None:
        if not isinstance(stream, Stream):
            raise TypeError("ms.stream() expects an ms.Stream")
        self._s = stream
        self._torch_ctx = None

    def __enter__(self) -> Stream:
        _stack("streams").append(self._s)
        self._torch_ctx = torch.cuda.stream(self._s._torch)
        self._torch_ctx.__enter__()
        return self._s

    def __exit__(self, *exc) -> bool:
        self._torch_ctx.__exit__(*exc)
        _stack("streams").pop()
        return False


def stream(s: Stream) -> _StreamContext:
    return _StreamContext(s)


class _DeviceContext:
    """``with ms.device("cuda:1"):`` (lib.rs:111-116): the default device
    inside the block."""

    def __init__(self, spec) -> None:
        from .array import parse_device

        self._dev = parse_device(spec)

    def __enter__(self):
        from .array import Device

        _stack("devices").append(self._dev)
        return Device(self._dev)

    def __exit__(self, *exc) -> bool:
        _stack("devices").pop()
        return False


def device(spec) -> _DeviceContext:
    return _DeviceContext(spec)


class _DtypeContext:
    """``with ms.dtype("f64"):`` (lib.rs:119-123): the default dtype inside
    the block. ``ms.dtype(spec).dtype`` is the parsed Dtype."""

    def __init__(self, spec) -> None:
        self.dtype = _dt.parse(spec)

    def __enter__(self) -> _dt.Dtype:
        _stack("dtypes").append(self.dtype)
        return self.dtype

    def __exit__(self, *exc) -> bool:
        _stack("dtypes").pop()
        return False

    def __eq__(self, other) -> bool:
        return self.dtype == other

    def __hash__(self) -> int:
        return hash(self.dtype)

    def __repr__(self) -> str:
        return f"dtype({self.dtype.name})"


def dtype(spec) -> _DtypeContext:
    return _DtypeContext(spec)


# ---------------------------------------------------------- resolution
# resolution.rs:1-120 (ADR L0-6..L0-11): the default device and dtype are
# per thread; set_default_* writes the calling thread's value and, until the
# thread has taken its snapshot, the process-wide seed; a thread without a
# value snapshots the seed on first use and is independent afterwards. The
# device has no fallback (DeviceNotConfiguredError), the dtype falls back to
# float32.
_seed = {"device": None, "dtype": None}
_seed_lock = threading.Lock()


def _get_default(kind: str):
    v = getattr(_tls, kind + "_default", None)
    if v is not None:
        return v
    with _seed_lock:
        v = _seed[kind]
    if v is not None:
        setattr(_tls, kind + "_default", v)
        setattr(_tls, kind + "_snap", True)
    return v


def _set_default(kind: str, value) -> None:
    setattr(_tls, kind + "_default", value)
    if not getattr(_tls, kind + "_snap", False):
        with _seed_lock:
            _seed[kind] = value


def set_default_device(dev: int) -> None:
    _set_default("device", dev)


def set_default_dtype(dt: _dt.Dtype) -> None:
    _set_default("dtype", dt)


def resolve_device(arg=None) -> tuple[int, str]:
    """(device index, source): arg > context > global_default >
    DeviceNotConfiguredError (resolution.rs:200-235)."""
    from .array import parse_device

    if arg is not None:
        return parse_device(arg), "arg"
    st = _stack("devices")
    if st:
        return st[-1], "context"
    d = _get_default("device")
    if d is not None:
        return d, "global_default"
    raise errors.DeviceNotConfiguredError(
        "no device: pass device=..., use `with ms.device(...)`, or call ms.set_default_device('musa:0')")


def resolve_dtype(arg=None) -> tuple[_dt.Dtype, str]:
    """(dtype, source): arg > context > global_default > float32 (resolution.rs:240-262)."""
    if arg is not None:
        return _dt.parse(arg), "arg"
    st = _stack("dtypes")
    if st:
        return st[-1], "context"
    d = _get_default("dtype")
    if d is not None:
        return d, "global_default"
    return _dt.float32, "auto_probe"  # the float32 fallback


def default_device() -> int:
    return resolve_device()[0]


def default_dtype() -> _dt.Dtype:
    return resolve_dtype()[0]
