"""The multi-rank peer exchange and combine of sharded full reductions, with
every rank played on one GPU.

A sharded argmax / sum ends with each rank's local record (the product's
mpb_reduce with the *_REC op, or its f64 partial sum) exchanged over peer
memory and combined in rank order by k_peer_arg_combine /
k_peer_sum_finalize. Here those same kernels run as ONE cooperative launch of
`world` blocks on one GPU (mpb_peer_*_emulated), block r playing rank r with
its own exchange buffer, so the wire format, both buffer parities and the
cross-rank first-occurrence and NaN rule of musapy's CPU loop
(rust/musapy-ops/src/op_builder.rs:3543-3578: strict comparison, the first
occurrence wins, a NaN only when it is element 0) are checked against the
oracle over the whole array at world 2, 3 and 8. Ranks that wait on one
another are never separate launches on one GPU; the single cooperative launch
keeps every block resident.
"""
import ctypes

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

F32, F64, I64 = 10, 11, 4
SUM, ARGMAX_REC, ARGMIN_REC = 0, 7, 8
CODE = {np.float32: F32, np.float64: F64, np.int64: I64}
INT64_MAX = np.iinfo(np.int64).max


def _i64(v):
    return (ctypes.c_int64 * max(1, len(v)))(*v)


def _stream():
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


class Ranks:
    """`world` zeroed exchange buffers on this GPU and the exchange counter
    (every call uses the next sequence number, alternating buffer parities)."""

    def __init__(self, LIB, world: int):
        nbytes = int(LIB.mpb_peer_buffer_bytes())
        self.bufs = [torch.zeros(nbytes, dtype=torch.uint8, device="cuda") for _ in range(world)]
        self.ptrs = (ctypes.c_void_p * world)(*[b.data_ptr() for b in self.bufs])
        self.world = world
        self.seq = 0
        self.status = torch.zeros(1, dtype=torch.int32, device="cuda")

    def next(self) -> int:
        self.seq += 1
        return self.seq


def _parts(n: int, world: int):
    """Contiguous [start, stop) blocks, the first n % world one longer (the
    sharded path's row split)."""
    base, extra = divmod(n, world)
    out, s = [], 0
    for r in range(world):
        e = s + base + (1 if r < extra else 0)
        out.append((s, e))
        s = e
    return out


def _local_records(LIB, x: torch.Tensor, parts, is_max: bool) -> torch.Tensor:
    """Each rank's {value bits, local index} record from the product's own
    local reduction; only rank 0 applies the first-element NaN rule; a rank
    without elements sends {0, INT64_MAX}."""
    code = {torch.float32: F32, torch.float64: F64, torch.int64: I64}[x.dtype]
    recs = torch.empty((len(parts), 2), dtype=torch.int64, device="cuda")
    op = ARGMAX_REC if is_max else ARGMIN_REC
    for r, (s, e) in enumerate(parts):
        if e == s:
            recs[r, 0], recs[r, 1] = 0, INT64_MAX
            continue
        part = x[s:e]
        shape, strides = _i64([e - s]), _i64([1])
        need = LIB.mpb_reduce_scratch_bytes(op, 1, shape, strides, part.data_ptr(), code, 1, code)
        scratch = torch.empty(max(1, need), dtype=torch.uint8, device="cuda")
        rc = LIB.mpb_reduce(op, 1, shape, strides, part.data_ptr(), code, 1, recs[r].data_ptr(), I64, code,
                            1 if r == 0 else 0, scratch.data_ptr(), need, torch.cuda.current_stream().cuda_stream)
        assert rc == 0, LIB.mpb_last_error()
    return recs


def _arg_combine(LIB, ranks: Ranks, recs: torch.Tensor, parts, is_max: bool, is_int: bool):
    idx = torch.full((ranks.world,), -1, dtype=torch.int64, device="cuda")
    val = torch.zeros(ranks.world, dtype=torch.float64, device="cuda")
    rc = LIB.mpb_peer_arg_combine_emulated(recs.data_ptr(), ranks.ptrs, ranks.world, ranks.next(),
                                           _i64([s for s, _ in parts]), 1 if is_max else 0, 1 if is_int else 0,
                                           idx.data_ptr(), val.data_ptr(), ranks.status.data_ptr(), _stream())
    assert rc == 0, LIB.mpb_last_error()
    torch.cuda.synchronize()
    assert int(ranks.status.item()) == 0
    return idx.cpu().numpy()


def _case(name: str, n: int, world: int, dtype, rng) -> np.ndarray:
    x = rng.standard_normal(n).astype(dtype) if dtype != np.int64 else rng.integers(-50, 50, n).astype(np.int64)
    parts = _parts(n, world)
    s1, e1 = parts[1]
    if name == "tie_across_ranks":
        # each extreme appears at the end of rank 0 and at the start of rank 1
        # (and of rank 2): rank 0's occurrence is the first one
        hi, lo = x.max() + 3, x.min() - 3
        x[parts[0][1] - 1], x[parts[0][1] - 2] = hi, lo
        x[s1], x[s1 + 1] = hi, lo
        if world > 2:
            x[parts[2][0]], x[parts[2][0] + 1] = hi, lo
    elif name == "tie_later_ranks":
        hi, lo = x.max() + 3, x.min() - 3
        x[s1 + 1], x[s1 + 2] = hi, lo
        x[parts[-1][0]], x[parts[-1][0] + 1] = hi, lo
    elif name == "nan_first_of_rank1":
        x[s1] = np.nan     # not global element 0: never the answer
    elif name == "nan_global_first":
        x[0] = np.nan      # global element 0: the answer
        x[s1 + 2] = np.nan
    elif name == "all_equal":
        x[:] = 1 if dtype == np.int64 else 0.5
    return x


CASES = ["random", "tie_across_ranks", "tie_later_ranks", "nan_first_of_rank1", "nan_global_first", "all_equal"]


@pytest.mark.parametrize("world", [2, 3, 8])
@pytest.mark.parametrize("dtype", [np.float32, np.float64, np.int64])
def test_emulated_arg_combine_matches_oracle(oracle, world, dtype):
    from musapy_b200._lib import LIB

    rng = np.random.default_rng(1000 + world)
    ranks = Ranks(LIB, world)
    for name in CASES:
        if dtype == np.int64 and name.startswith("nan"):
            continue
        for n in (world * 70001 + 3, 5 * world + 1):  # split kernels, and tiny ranks
            host = _case(name, n, world, dtype, rng)
            parts = _parts(n, world)
            x = torch.from_numpy(host).cuda()
            for is_max in (True, False):
                recs = _local_records(LIB, x, parts, is_max)
                got = _arg_combine(LIB, ranks, recs, parts, is_max, dtype == np.int64)
                want = int(oracle.reduce("argmax" if is_max else "argmin", host, None))
                assert (got == want).all(), (name, n, is_max, got, want)


def test_emulated_arg_combine_with_empty_ranks(oracle):
    """More ranks than elements: the empty ranks' records are skipped."""
    from musapy_b200._lib import LIB

    world = 8
    ranks = Ranks(LIB, world)
    for host in (np.array([0.5, -2.0, 7.0, 7.0, 1.0], np.float32), np.array([np.nan, 3.0], np.float32)):
        parts = _parts(host.size, world)
        x = torch.from_numpy(host).cuda()
        for is_max in (True, False):
            recs = _local_records(LIB, x, parts, is_max)
            got = _arg_combine(LIB, ranks, recs, parts, is_max, False)
            want = int(oracle.reduce("argmax" if is_max else "argmin", host, None))
            assert (got == want).all(), (host, is_max, got, want)


@pytest.mark.parametrize("world", [2, 3, 8])
@pytest.mark.parametrize("dtype", [np.float32, np.float64])
def test_emulated_sum_finalize_matches_oracle_on_every_rank(oracle, world, dtype):
    from musapy_b200._lib import LIB

    rng = np.random.default_rng(2000 + world)
    ranks = Ranks(LIB, world)
    code = CODE[dtype]
    for n in (world * 300007 + 5, 2 * world + 1, world - 1):
        host = rng.standard_normal(n).astype(dtype)
        parts = _parts(n, world)
        x = torch.from_numpy(host).cuda()
        partials = torch.zeros(world, dtype=torch.float64, device="cuda")
        for r, (s, e) in enumerate(parts):
            if e == s:
                continue  # a rank without elements contributes 0
            shape, strides = _i64([e - s]), _i64([1])
            part = x[s:e]
            need = LIB.mpb_reduce_scratch_bytes(SUM, 1, shape, strides, part.data_ptr(), code, 1, code)
            scratch = torch.empty(max(1, need), dtype=torch.uint8, device="cuda")
            rc = LIB.mpb_reduce(SUM, 1, shape, strides, part.data_ptr(), code, 1, partials[r].data_ptr(), F64, code,
                                1, scratch.data_ptr(), need, torch.cuda.current_stream().cuda_stream)
            assert rc == 0, LIB.mpb_last_error()
        tdt = torch.float32 if dtype == np.float32 else torch.float64
        s_out = torch.full((world,), 9.0, dtype=tdt, device="cuda")
        m_out = torch.full((world,), 9.0, dtype=tdt, device="cuda")
        rc = LIB.mpb_peer_sum_finalize_emulated(partials.data_ptr(), ranks.ptrs, world, ranks.next(), float(n), code,
                                                s_out.data_ptr(), m_out.data_ptr(), ranks.status.data_ptr(),
                                                _stream())
        assert rc == 0, LIB.mpb_last_error()
        torch.cuda.synchronize()
        assert int(ranks.status.item()) == 0
        s_h, m_h = s_out.cpu().numpy(), m_out.cpu().numpy()
        # every rank holds the same bits
        assert (s_h.view(np.uint8).reshape(world, -1) == s_h.view(np.uint8).reshape(world, -1)[0]).all()
        assert (m_h.view(np.uint8).reshape(world, -1) == m_h.view(np.uint8).reshape(world, -1)[0]).all()
        # and the rank-order sum of the partials, rounded once, is the value
        want_sum = np.float64(0.0)
        for r in range(world):
            want_sum += np.float64(partials[r].item())
        assert s_h[0] == want_sum.astype(dtype)
        assert m_h[0] == np.float64(want_sum / n).astype(dtype)
        # against the oracle: within rtol * sum|x| (or closer to the f64 truth)
        from tests.helpers import assert_sum_close

        absx = np.abs(host.astype(np.float64)).sum()
        truth = host.astype(np.float64).sum()
        rtol = 1e-5 if dtype == np.float32 else 1e-12
        assert_sum_close(s_h[0], oracle.reduce("sum", host, None), absx, rtol, "sharded sum", truth=truth)
        if n:
            assert_sum_close(m_h[0], oracle.reduce("mean", host, None), absx / n, rtol, "sharded mean",
                             truth=truth / n)
