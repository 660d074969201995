"""The NVLink record exchange kernels on one GPU (musapy_b200/csrc/peer.cu).

A one-rank exchange sends the record to the rank's own buffer and reads it
back through the same flag-in-line words a multi-rank exchange uses, so the
wire format, both buffer parities, the fused sum / argmax finishes and the
status word are all exercised without a second GPU. The time-limit test
makes one wait run out: a two-rank exchange whose second rank never sends
(nothing else runs), as the bounded waits are meant to handle.
"""
import ctypes
import struct

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

MPB_ERR_TIMEOUT = 6
F32, F64 = 10, 11


@pytest.fixture
def peer(ms):
    from musapy_b200._lib import LIB

    buf = ctypes.c_void_p()
    handle = ctypes.create_string_buffer(int(LIB.mpb_peer_handle_bytes()))
    assert LIB.mpb_peer_alloc(ctypes.byref(buf), handle) == 0
    yield LIB, buf
    torch.cuda.synchronize()
    assert LIB.mpb_peer_free(buf) == 0


def _stream():
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


def _ptrs(*bufs):
    return (ctypes.c_void_p * len(bufs))(*[b.value for b in bufs])


def test_self_allgather_every_record_size_both_parities(peer):
    LIB, buf = peer
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    peers = _ptrs(buf)
    seq = 0
    for rec_bytes in (8, 16, 24, 32):
        for k in range(4):
            seq += 1
            rec = torch.randint(-2**62, 2**62, (rec_bytes // 8,), dtype=torch.int64, device="cuda")
            out = torch.full((rec_bytes // 8,), -1, dtype=torch.int64, device="cuda")
            rc = LIB.mpb_peer_allgather(ctypes.c_void_p(rec.data_ptr()), rec_bytes, peers, 0, 1, seq,
                                        ctypes.c_void_p(out.data_ptr()), ctypes.c_void_p(status.data_ptr()),
                                        _stream())
            assert rc == 0
            assert torch.equal(out, rec), (rec_bytes, k)
    assert int(status.item()) == 0


@pytest.mark.parametrize("out_dt", [F32, F64])
def test_self_sum_finalize(peer, out_dt):
    LIB, buf = peer
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    tdt = torch.float32 if out_dt == F32 else torch.float64
    for seq, total in enumerate([3.5, -1e300 if out_dt == F64 else -1e30, float("nan"), 0.1], start=1):
        partial = torch.tensor([total, 123.0], dtype=torch.float64, device="cuda")
        s = torch.zeros((), dtype=tdt, device="cuda")
        m = torch.zeros((), dtype=tdt, device="cuda")
        rc = LIB.mpb_peer_sum_finalize(ctypes.c_void_p(partial.data_ptr()), _ptrs(buf), 0, 1, seq, 7.0, out_dt,
                                       ctypes.c_void_p(s.data_ptr()), ctypes.c_void_p(m.data_ptr()),
                                       ctypes.c_void_p(status.data_ptr()), _stream())
        assert rc == 0
        want_s = np.array(total, dtype=np.float64).astype(np.float32 if out_dt == F32 else np.float64)
        want_m = np.array(total / 7.0, dtype=np.float64).astype(want_s.dtype)
        np.testing.assert_array_equal(s.cpu().numpy(), want_s)
        np.testing.assert_array_equal(m.cpu().numpy(), want_m)
    assert int(status.item()) == 0


def _bits(v: float) -> int:
    return struct.unpack("<q", struct.pack("<d", v))[0]


@pytest.mark.parametrize("case", ["float", "nan_first", "int", "empty"])
def test_self_arg_combine(peer, case):
    LIB, buf = peer
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    is_int = case == "int"
    recs = {"float": [_bits(2.5), 42], "nan_first": [_bits(float("nan")), 0], "int": [-7, 9],
            "empty": [0, 2**63 - 1]}[case]
    want = {"float": 142, "nan_first": 0, "int": 109, "empty": 0}[case]
    offsets = (ctypes.c_int64 * 1)(100 if case != "nan_first" else 0)
    for seq in (1, 2, 3):  # both parities
        rec = torch.tensor(recs, dtype=torch.int64, device="cuda")
        idx = torch.full((), -1, dtype=torch.int64, device="cuda")
        val = torch.zeros(1, dtype=torch.float64, device="cuda")
        rc = LIB.mpb_peer_arg_combine(ctypes.c_void_p(rec.data_ptr()), _ptrs(buf), 0, 1, seq, offsets, 1,
                                      1 if is_int else 0, ctypes.c_void_p(idx.data_ptr()),
                                      ctypes.c_void_p(val.data_ptr()), ctypes.c_void_p(status.data_ptr()),
                                      _stream())
        assert rc == 0
        assert int(idx.item()) == want, (case, seq)
        if case == "float":
            assert float(val.item()) == 2.5
        if case == "int":
            assert float(val.item()) == -7.0
    assert int(status.item()) == 0


def test_wait_runs_out_and_reports(peer):
    """Rank 0 of a two-rank exchange whose rank 1 never sends: the wait ends
    after its time limit, the status word says so and no result is written;
    the context stays usable."""
    from musapy_b200._lib import LIB

    _, buf0 = peer
    buf1 = ctypes.c_void_p()
    handle = ctypes.create_string_buffer(int(LIB.mpb_peer_handle_bytes()))
    assert LIB.mpb_peer_alloc(ctypes.byref(buf1), handle) == 0
    try:
        status = torch.zeros(1, dtype=torch.int32, device="cuda")
        partial = torch.tensor([1.0, 0.0], dtype=torch.float64, device="cuda")
        s = torch.full((), 5.0, dtype=torch.float64, device="cuda")
        m = torch.full((), 5.0, dtype=torch.float64, device="cuda")
        rc = LIB.mpb_peer_sum_finalize(ctypes.c_void_p(partial.data_ptr()), _ptrs(buf0, buf1), 0, 2, 1, 1.0, F64,
                                       ctypes.c_void_p(s.data_ptr()), ctypes.c_void_p(m.data_ptr()),
                                       ctypes.c_void_p(status.data_ptr()), _stream())
        assert rc == 0
        torch.cuda.synchronize()
        assert int(status.item()) == MPB_ERR_TIMEOUT
        assert float(s.item()) == 5.0 and float(m.item()) == 5.0
        # the device is still usable
        assert float(torch.ones(4, device="cuda").sum().item()) == 4.0
    finally:
        torch.cuda.synchronize()
        assert LIB.mpb_peer_free(buf1) == 0


def test_bad_arguments_are_rejected(peer):
    LIB, buf = peer
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    rec = torch.zeros(2, dtype=torch.int64, device="cuda")
    out = torch.zeros(2, dtype=torch.int64, device="cuda")
    args = lambda nbytes, world, seq: (ctypes.c_void_p(rec.data_ptr()), nbytes, _ptrs(buf), 0, world, seq,  # noqa: E731
                                       ctypes.c_void_p(out.data_ptr()), ctypes.c_void_p(status.data_ptr()), _stream())
    assert LIB.mpb_peer_allgather(*args(12, 1, 1)) != 0  # size not a multiple of 8
    assert LIB.mpb_peer_allgather(*args(40, 1, 1)) != 0  # larger than 32 bytes
    assert LIB.mpb_peer_allgather(*args(16, 17, 1)) != 0  # too many ranks
    assert LIB.mpb_peer_allgather(*args(16, 1, 0)) != 0  # seq starts at 1
    assert LIB.mpb_peer_sum_finalize(ctypes.c_void_p(rec.data_ptr()), _ptrs(buf), 0, 1, 1, 1.0, 5, None, None,
                                     ctypes.c_void_p(status.data_ptr()), _stream()) != 0  # i64 output
