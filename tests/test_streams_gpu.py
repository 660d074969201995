"""Streams on the GPU: the reference's multi-stream acceptance cases
(tests/python/test_stream.py:47-230, run there on cpu and musa devices) on
CUDA streams, plus ordering checks that would fail without the automatic
cross-stream waits."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def test_two_streams_independent_arrays(ms):
    s1, s2 = ms.Stream("cuda:0"), ms.Stream("cuda:0")
    with ms.stream(s1):
        a = ms.array([1.0, 2.0, 3.0], dtype="f32")
    with ms.stream(s2):
        b = ms.array([4.0, 5.0, 6.0], dtype="f32")
    s1.synchronize()
    s2.synchronize()
    assert a.tolist() == [1.0, 2.0, 3.0] and b.tolist() == [4.0, 5.0, 6.0]
    assert a.stream == s1 and b.stream == s2


def test_cross_stream_add_and_out(ms):
    s1, s2 = ms.Stream("cuda:0"), ms.Stream("cuda:0")
    with ms.stream(s1):
        a = ms.array([1.0, 2.0, 3.0], dtype="f32")
    with ms.stream(s2):
        b = ms.array([4.0, 5.0, 6.0], dtype="f32")
        out = ms.array([0.0, 0.0, 0.0], dtype="f32")
    with ms.stream(s2):
        c = ms.add(a, b)
        r = ms.add(a, b, out=out)
    s2.synchronize()
    assert c.tolist() == [5.0, 7.0, 9.0] and out.tolist() == [5.0, 7.0, 9.0] and r is out


def test_reader_waits_for_writer_on_other_stream(ms):
    """A long chain of writes on s1, then a reduction on s2 of the final
    buffer: s2 must see every write (it waits for s1's work, no host sync)."""
    n = 1 << 24
    s1, s2 = ms.Stream("cuda:0"), ms.Stream("cuda:0")
    with ms.stream(s1):
        one = ms.ones((n,), dtype="f32")
        x = ms.zeros((n,), dtype="f32")
        y = ms.empty((n,), dtype="f32")
        for _ in range(40):
            ms.add(x, one, out=y)
            x, y = y, x
    with ms.stream(s2):
        total = ms.sum(x, axis=0)
        mx = ms.max(x)
    s2.synchronize()
    assert total.item() == 40.0 * n and mx.item() == 40.0


def test_writer_waits_for_reader_on_other_stream(ms):
    """Write-after-read: s1 reads x twenty times, then s2 overwrites x; every
    read must see the old contents."""
    n = 1 << 24
    s1, s2 = ms.Stream("cuda:0"), ms.Stream("cuda:0")
    x = ms.full((n,), 2.0, dtype="f32")
    with ms.stream(s1):
        sums = [ms.sum(x, axis=0) for _ in range(20)]
    with ms.stream(s2):
        zero = ms.zeros((n,), dtype="f32")
        ms.mul(zero, zero, out=x)
    s1.synchronize()
    s2.synchronize()
    assert all(v.item() == 2.0 * n for v in sums)
    assert ms.max(x).item() == 0.0


def test_interleaved_and_many_streams(ms):
    streams = [ms.Stream("cuda:0") for _ in range(8)]
    vals = []
    for i, s in enumerate(streams):
        with ms.stream(s):
            a = ms.full((1000,), float(i), dtype="f64")
            vals.append(ms.sum(ms.mul(a, a), axis=0))
    for s in streams:
        s.synchronize()
    assert [v.item() for v in vals] == [1000.0 * i * i for i in range(8)]
    for s in streams:
        assert not s.is_poisoned and s.pending_count == 0


def test_stream_reuse_after_sync_and_priority(ms):
    hi = ms.Stream("cuda:0", priority=-1)
    assert hi.priority == -1 and hi.device == "cuda:0"
    with ms.stream(hi):
        a = ms.arange(10, dtype="f32")
    hi.synchronize()
    with ms.stream(hi):
        b = ms.cumsum(a)
    hi.synchronize()
    assert b.tolist() == np.cumsum(np.arange(10, dtype=np.float32)).tolist()


def test_default_stream_ops_follow_torch_current_stream(ms):
    import torch

    side = torch.cuda.Stream()
    with torch.cuda.stream(side):
        a = ms.arange(4, dtype="f32")
        assert ms.streams.current_stream(0).cuda_stream == side.cuda_stream
    torch.cuda.synchronize()
    assert a.tolist() == [0.0, 1.0, 2.0, 3.0]


@pytest.mark.parametrize("nbytes", [(1 << 20) - 1, 1 << 20, (1 << 20) + 3, (100 << 20) + 7, (300 << 20) + 5])
def test_staged_host_transfers_round_trip(ms, nbytes):
    """from_numpy / numpy() through the pinned staging ring (sizes below,
    at and above the threshold, not multiples of 16, larger than the ring)."""
    rng = np.random.default_rng(nbytes % 1000)
    host = rng.integers(0, 256, nbytes, dtype=np.uint8)
    d = ms.from_numpy(host)
    back = d.numpy()
    assert back.dtype == np.uint8 and np.array_equal(back, host)
    # a device-side op in between: the copy-out sees its result
    f = rng.standard_normal(nbytes // 8).astype(np.float64)
    fd = ms.from_numpy(f)
    neg = ms.neg(fd).numpy()
    assert np.array_equal(neg, -f)


def test_staged_copy_waits_for_other_stream(ms):
    n = 1 << 24
    s1 = ms.Stream("cuda:0")
    with ms.stream(s1):
        x = ms.zeros((n,), dtype="f32")
        one = ms.ones((n,), dtype="f32")
        y = ms.empty((n,), dtype="f32")
        for _ in range(30):
            ms.add(x, one, out=y)
            x, y = y, x
    # copied out on the default stream: waits for s1's chain
    h = x.numpy()
    assert h.min() == 30.0 and h.max() == 30.0


def test_from_numpy_views_and_complex(ms):
    rng = np.random.default_rng(3)
    a = rng.standard_normal((1024, 768)) + 1j * rng.standard_normal((1024, 768))
    v = a[::2, ::-3]
    d = ms.from_numpy(v)
    assert np.array_equal(d.numpy(), v)
    z = ms.from_numpy(np.float32(2.5))
    assert z.shape == () and z.item() == 2.5


def test_resolution_sources_on_arrays(ms):
    """The reference's resolution tests (tests/python/test_resolution.py:23-160)
    on the CUDA device: repr(a.device) names how the device was chosen, the
    dtype context sets the default dtype, op results follow their inputs."""
    import threading

    ms.set_default_device("cuda:0")
    a = ms.array([1.0, 2.0], dtype="f32", device="cuda:0")
    assert "resolved from: arg" in repr(a.device)
    b = ms.array([1.0, 2.0], dtype="f32")
    assert "resolved from: global_default" in repr(b.device)
    with ms.device("cuda:0"):
        c = ms.array([1.0], dtype="f32")
        assert "resolved from: context" in repr(c.device)
        with ms.device("musa:0"):
            assert "context" in repr(ms.array([1.0], dtype="f32").device)
    assert "global_default" in repr(ms.array([1.0], dtype="f32").device)
    with ms.dtype("f64"):
        d = ms.array([1.0, 2.0])
        assert d.dtype == "f64" and d.dtype_resolution_source == "context"
    e = ms.array([1.0, 2.0])
    assert e.dtype == "f32" and e.dtype_resolution_source == "auto_probe"
    s = ms.Stream("cuda:0", priority=0)
    with ms.stream(s):
        f = ms.array([1.0], dtype="f32")
        assert f.stream.priority == 0 and f.stream == s
    g = ms.add(a, b)
    assert g.device.resolution_source == "input_array" and g.dtype_resolution_source == "input_array"
    out = {}

    def worker():
        out["dev"] = str(ms.array([1.0], dtype="f32").device)

    t = threading.Thread(target=worker)
    t.start()
    t.join(30)
    assert out["dev"] == "cuda:0"


@pytest.mark.parametrize("nbytes", [16, (1 << 20) + 3, (100 << 20) + 7])
def test_page_locked_host_transfers_take_one_dma(ms, nbytes):
    """mpb_copy_h2d / mpb_copy_d2h with page-locked host buffers (torch
    pin_memory): one DMA each way, returning once the data has moved, so the
    source can be overwritten at once and the destination read at once."""
    import ctypes

    import torch

    from musapy_b200._lib import LIB

    rng = np.random.default_rng(nbytes % 977)
    src = torch.from_numpy(rng.integers(0, 256, nbytes, dtype=np.uint8)).pin_memory()
    want = src.clone()
    dev = torch.empty(nbytes, dtype=torch.uint8, device="cuda")
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    assert LIB.mpb_copy_h2d(dev.data_ptr(), src.data_ptr(), nbytes, stream) == 0
    src.zero_()  # the call returned: the DMA has read the source
    dst = torch.zeros(nbytes, dtype=torch.uint8).pin_memory()
    assert LIB.mpb_copy_d2h(dst.data_ptr(), dev.data_ptr(), nbytes, stream) == 0
    assert torch.equal(dst, want)  # no synchronize needed: the call waited
