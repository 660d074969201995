"""Host logic of the stream runtime (musapy_b200/streams.py) with fake CUDA
streams: cross-stream waits, poisoning with op context, and the device /
dtype / stream context stacks. No GPU; failures are made on the host (a fake
synchronize that raises, as an asynchronous fault would surface)."""
import threading

import pytest

import musapy_b200 as ms
from musapy_b200 import streams


class FakeTorchStream:
    _next = [1000]

    def __init__(self, fail_sync: str | None = None) -> None:
        FakeTorchStream._next[0] += 16
        self.cuda_stream = FakeTorchStream._next[0]
        self.priority = 0
        self.waited = []
        self.fail_sync = fail_sync
        self.synced = 0

    def wait_stream(self, other) -> None:
        self.waited.append(other.cuda_stream)

    def synchronize(self) -> None:
        self.synced += 1
        if self.fail_sync:
            raise RuntimeError(self.fail_sync)

    def query(self) -> bool:
        return False


class FakeBuf:
    def __init__(self) -> None:
        self.recorded = []

    def record_stream(self, s) -> None:
        self.recorded.append(s.cuda_stream)


class FakeArray:
    def __init__(self) -> None:
        self._buf = FakeBuf()


@pytest.fixture
def on_stream():
    """Run with `s` as the innermost ms.stream for device 0 (the stack the
    context manager maintains; entering torch's stream context needs CUDA)."""
    def push(s):
        streams._stack("streams").append(s)

    yield push
    streams._stack("streams").clear()


def test_cross_stream_use_waits_and_records(on_stream):
    t1, t2 = FakeTorchStream(), FakeTorchStream()
    s1, s2 = ms.Stream(0, _torch_stream=t1), ms.Stream(0, _torch_stream=t2)
    a, b, out = FakeArray(), FakeArray(), FakeArray()
    on_stream(s1)
    assert streams.launch("fill", 0, a) == t1.cuda_stream  # a written on s1
    streams._stack("streams").pop()
    on_stream(s2)
    h = streams.launch("add", 0, a, b, out)
    assert h == t2.cuda_stream
    # a's last use was s1: s2 waits for s1 and the allocator learns a is used on s2
    assert t2.waited == [t1.cuda_stream]
    assert a._buf.recorded == [t2.cuda_stream]
    # b and out were never used: nothing to wait for
    assert b._buf.recorded == [] and out._buf.recorded == []
    # a second op on the same stream waits for nothing new
    streams.launch("mul", 0, a, out)
    assert t2.waited == [t1.cuda_stream]
    assert s2.op_context() == "add; mul"


def test_write_after_read_orders_across_streams(on_stream):
    t1, t2 = FakeTorchStream(), FakeTorchStream()
    s1, s2 = ms.Stream(0, _torch_stream=t1), ms.Stream(0, _torch_stream=t2)
    x = FakeArray()
    on_stream(s1)
    streams.launch("sum", 0, x)  # read on s1
    streams._stack("streams").pop()
    on_stream(s2)
    streams.launch("fill", 0, x)  # overwrite on s2 must wait for the read
    assert t2.waited == [t1.cuda_stream]


def test_async_fault_poisons_with_op_context(on_stream):
    t = FakeTorchStream(fail_sync="CUDA error: an illegal memory access was encountered")
    s = ms.Stream(0, _torch_stream=t)
    on_stream(s)
    streams.launch("add", 0, FakeArray())
    streams.launch("cumsum", 0, FakeArray())
    assert not s.is_poisoned
    with pytest.raises(ms.StreamError, match="illegal memory access") as ei:
        s.synchronize()
    assert "add; cumsum" in str(ei.value)
    assert s.is_poisoned
    # every later op on the stream is refused before launching
    with pytest.raises(ms.StreamError, match="poisoned"):
        streams.launch("mul", 0, FakeArray())
    with pytest.raises(ms.StreamError):
        s.synchronize()
    assert t.synced == 1


def test_successful_synchronize_clears_context(on_stream):
    t = FakeTorchStream()
    s = ms.Stream(0, priority=-1, _torch_stream=t)
    on_stream(s)
    streams.launch("add", 0, FakeArray())
    assert s.pending_count == 1
    s.synchronize()
    assert s.pending_count == 0 and s.op_context() == ""
    assert s.priority == -1 and s.device == "cuda:0" and s.id > 0
    assert "Stream(device=cuda:0" in repr(s)


def test_op_context_is_bounded(on_stream):
    s = ms.Stream(0, _torch_stream=FakeTorchStream())
    on_stream(s)
    for i in range(100):
        streams.launch(f"op{i}", 0, FakeArray())
    ops = s.op_context().split("; ")
    assert len(ops) == streams.OP_CONTEXT_DEPTH and ops[-1] == "op99"


def test_stream_context_requires_stream():
    with pytest.raises(TypeError):
        ms.stream("cuda:0")


def test_device_and_dtype_contexts_nest_and_restore():
    from musapy_b200.array import default_dtype, parse_device

    ms.set_default_device("musa:0")
    base_dev, base_dt = parse_device(None), default_dtype()
    with ms.device("musa:2") as d:
        assert d == "cuda:2" and parse_device(None) == 2
        with ms.device(5):
            assert parse_device(None) == 5
        assert parse_device(None) == 2
        with ms.dtype("f64") as dt:
            assert dt == ms.float64 and default_dtype() == ms.float64
            with ms.dtype("i32"):
                assert default_dtype() == ms.int32
            assert default_dtype() == ms.float64
    assert parse_device(None) == base_dev and default_dtype() == base_dt
    assert ms.dtype("bf16") == ms.bfloat16


def test_contexts_are_per_thread():
    from musapy_b200.array import default_dtype

    seen = {}
    entered, release = threading.Event(), threading.Event()

    def worker():
        with ms.dtype("f16"):
            seen["inner"] = default_dtype()
            entered.set()
            release.wait(5)

    th = threading.Thread(target=worker)
    th.start()
    entered.wait(5)
    seen["main"] = default_dtype()
    release.set()
    th.join(5)
    assert seen["inner"] == ms.float16 and seen["main"] == ms.float32


def test_device_context_rejects_cpu():
    with pytest.raises(ms.DeviceError):
        ms.device("cpu")


def test_resolution_chain_sources():
    """resolve_device / resolve_dtype: arg > context > global_default
    (resolution.rs:200-262); dtype falls back to float32 (auto_probe)."""
    import subprocess
    import sys

    code = ("import musapy_b200 as ms\n"
            "try:\n"
            "    ms.streams.resolve_device()\n"
            "    print('NO_ERROR')\n"
            "except ms.DeviceNotConfiguredError as e:\n"
            "    print('DeviceNotConfiguredError')\n"
            "print(ms.streams.resolve_dtype())\n")
    out = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True, timeout=300).stdout
    assert "DeviceNotConfiguredError" in out and "NO_ERROR" not in out
    assert "auto_probe" in out and "float32" in out
    assert issubclass(ms.DeviceNotConfiguredError, ms.DeviceError)
    ms.set_default_device("cuda:1")
    assert streams.resolve_device() == (1, "global_default")
    assert streams.resolve_device("musa:3") == (3, "arg")
    with ms.device("cuda:2"):
        assert streams.resolve_device() == (2, "context")
        assert streams.resolve_device(0) == (0, "arg")
    with ms.dtype("f64"):
        assert streams.resolve_dtype() == (ms.float64, "context")
        assert streams.resolve_dtype("f16") == (ms.float16, "arg")
    ms.set_default_device("cuda:0")


def test_default_device_thread_inheritance():
    """A new thread snapshots the process seed on first use; its own
    set_default_device does not reach the parent (resolution.rs:55-100)."""
    ms.set_default_device("cuda:0")
    seen = {}

    def child():
        seen["inherited"] = streams.resolve_device()
        ms.set_default_device("cuda:3")
        seen["own"] = streams.resolve_device()

    th = threading.Thread(target=child)
    th.start()
    th.join(10)
    assert seen["inherited"] == (0, "global_default") and seen["own"] == (3, "global_default")
    assert streams.resolve_device() == (0, "global_default")


def test_device_properties_match_binding():
    d = ms.Device("musa:1")
    assert d.is_musa is True and d.musa_id == 1 and str(d) == "cuda:1"
    assert repr(d) == "Device(cuda:1)" and d.resolution_source is None
