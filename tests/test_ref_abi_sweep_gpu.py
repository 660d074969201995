"""Every symbol of musapy's kernel C-ABI reproduced in
include/musapy_kernels_v2.h, called once through ctypes with a small strided
input and checked against the oracle.

The symbol list comes from the header itself, so a wrapper added there is
tested here; each name is dispatched on its musapy naming pattern (binary,
compare, unary, clamp, cast, naive / small-axis / partial / final / mid
reductions, cumsum_v3, fill, arange, linspace, eye, copy, copy_transpose2d).
"""
import ctypes
import os
import re

import numpy as np
import pytest
import torch

from tests.helpers import assert_bits_equal, assert_sum_close, assert_ulp

pytestmark = pytest.mark.gpu

SZ, SS = ctypes.c_size_t, ctypes.c_ssize_t
HEADER = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "include", "musapy_kernels_v2.h")
NP = {"f32": np.float32, "f64": np.float64, "i64": np.int64, "i32": np.int32, "i16": np.int16, "i8": np.int8,
      "u64": np.uint64, "u32": np.uint32, "u16": np.uint16, "u8": np.uint8, "c64": np.complex64,
      "c128": np.complex128, "bool": np.bool_}
CT = {"f32": ctypes.c_float, "f64": ctypes.c_double, "i64": ctypes.c_int64, "i32": ctypes.c_int32,
      "i16": ctypes.c_int16, "i8": ctypes.c_int8, "u64": ctypes.c_uint64, "u32": ctypes.c_uint32,
      "u16": ctypes.c_uint16, "u8": ctypes.c_uint8}
DT = "|".join(sorted(NP, key=len, reverse=True))


def symbols():
    return re.findall(r"void (musapy_[a-z0-9_]+)\(", open(HEADER).read())


def lib():
    from musapy_b200._lib import LIB

    return LIB


def sz(v):
    return (SZ * max(1, len(v)))(*v)


def ss(v):
    return (SS * max(1, len(v)))(*v)


def stream():
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


def P(t):
    return ctypes.c_void_p(t.data_ptr())


def rand(dt, shape, rng, positive=False):
    d = np.dtype(NP[dt])
    if d.kind == "f":
        x = rng.standard_normal(shape).astype(d)
        return np.abs(x) + d.type(0.25) if positive else x
    if d.kind == "c":
        return (rng.standard_normal(shape) + 1j * rng.standard_normal(shape)).astype(d)
    if d.kind == "b":
        return rng.random(shape) < 0.5
    info = np.iinfo(d)
    lo, hi = (1, 50) if positive else (max(info.min, -50), min(info.max, 50))
    return rng.integers(lo, hi, shape).astype(d)


def strided(x):
    """A (rows, cols) operand as a transposed device view: strides (1, rows)."""
    t = torch.from_numpy(np.ascontiguousarray(x.T)).cuda()
    return t, [1, x.shape[0]]


def out_np(t, dt):
    return t.cpu().numpy().view(NP[dt]) if NP[dt] != np.bool_ else t.cpu().numpy().astype(bool)


def check_float(got, want, what, ulp=None):
    if ulp is None:
        assert_bits_equal(got, want, what)
    else:
        assert_ulp(got, want, ulp, what)


BIN = re.compile(rf"musapy_(add|sub|mul|div|pow)_({DT})_v2$")
CMP = re.compile(rf"musapy_(eq|ne|lt|gt|le|ge)_({DT})_v2$")
UN = re.compile(rf"musapy_(sin|cos|exp|log|abs|sign|neg)_({DT})_v2$")
CLAMP = re.compile(rf"musapy_clamp_({DT})_v2$")
CAST = re.compile(rf"musapy_cast_({DT})_({DT})_v2$")
RED = re.compile(rf"musapy_(sum|prod|max|min|mean|argmax|argmin)_({DT})_v2$")
SMALL = re.compile(rf"musapy_(sum|prod|max|min|mean)_small_axis_({DT})_v2$")
PART = re.compile(rf"musapy_(sum|prod|max|min|mean)_partial_({DT})_v2$")
APART = re.compile(rf"musapy_(argmax|argmin)_partial_({DT})_v2$")
CUMSUM = re.compile(rf"musapy_cumsum_({DT})_v3$")
FILL = re.compile(rf"musapy_fill_({DT})$")
ARANGE = re.compile(rf"musapy_arange_({DT})$")
LINSPACE = re.compile(rf"musapy_linspace_({DT})$")
EYE = re.compile(rf"musapy_eye_({DT})$")
COPY = re.compile(rf"musapy_copy_({DT})$")
COPYT = re.compile(rf"musapy_copy_transpose2d_({DT})$")
# stages tested together with their partial stage
FOLLOWERS = re.compile(rf"musapy_(sum|prod|max|min|mean|argmax|argmin)_(final|mid)_({DT})_v2$")


def test_every_header_symbol_is_covered():
    names = symbols()
    assert len(names) >= 200
    pats = [BIN, CMP, UN, CLAMP, CAST, RED, SMALL, PART, APART, CUMSUM, FILL, ARANGE, LINSPACE, EYE, COPY, COPYT,
            FOLLOWERS]
    missing = [n for n in names if not any(p.match(n) for p in pats)]
    assert not missing, missing


def _reduce_check(op, got, x, axis, oracle, what):
    want = oracle.reduce(op, x, axis)
    if np.dtype(x.dtype).kind == "c":
        base = np.abs(x).astype(np.float64).sum(axis) / (x.shape[axis] if op == "mean" else 1)
        np.testing.assert_allclose(got, want, rtol=1e-5, atol=0 if op == "prod" else 1e-5 * base.max(), err_msg=what)
        return
    if op in ("max", "min", "argmax", "argmin") or np.dtype(x.dtype).kind in "iub":
        assert_bits_equal(got, want.astype(got.dtype) if op not in ("argmax", "argmin") else want, what)
    else:
        base = np.abs(x).astype(np.float64).sum(axis) / (x.shape[axis] if op == "mean" else 1)
        if op == "prod":
            # every one of the n-1 roundings of a product scales the result,
            # whatever the order, so the forward bound is (n-1)u relative
            # (Higham, Accuracy and Stability, 2nd ed., sec. 3.1). The CPU
            # multiplies sequentially and the GPU as a tree; factors
            # straddling 1.0 give the tree a one-sided tie-rounding bias that
            # the sequential product, drifting away from 1.0, avoids - so
            # either being within the bound, or no worse than the CPU, passes.
            # The truth is taken in extended precision.
            n = x.shape[axis]
            u = 2.0**-53 if x.dtype == np.float64 else 2.0**-24
            truth = np.prod(x.astype(np.longdouble), axis=axis)
            err_gpu = np.abs(got.astype(np.longdouble) - truth)
            err_cpu = np.abs(want.astype(np.longdouble) - truth)
            bound = (n - 1) * u * 1.01 * np.abs(truth)
            assert (err_gpu <= np.maximum(err_cpu * 1.0001, bound)).all(), (what, err_gpu.max(), bound.min())
        else:
            assert_sum_close(got, want.astype(got.dtype), base, 1e-5, what)


@pytest.mark.parametrize("name", symbols())
def test_symbol(oracle, name):
    rng = np.random.default_rng(sum(map(ord, name)))
    L = lib()
    fn = getattr(L, name)
    if FOLLOWERS.match(name):
        pytest.skip("called by the test of its partial stage")
    m = BIN.match(name) or CMP.match(name)
    if m:
        op, dt = m.groups()
        x, y = rand(dt, (37, 29), rng, positive=(op in ("pow", "div"))), rand(dt, (29,), rng, positive=True)
        xd, xst = strided(x)
        yd = torch.from_numpy(y).cuda()
        is_cmp = CMP.match(name) is not None
        c = torch.empty((37, 29), dtype=torch.uint8 if is_cmp else torch.from_numpy(x[:1]).dtype, device="cuda")
        fn(P(xd), P(yd), P(c), 2, sz([37, 29]), ss(xst), ss([0, 1]), stream())
        got = out_np(c, "bool") if is_cmp else c.cpu().numpy()
        if is_cmp:
            assert_bits_equal(got, oracle.compare(op, x, y), name)
        else:
            check_float(got, oracle.binary(op, x, y), name, ulp=2 if op == "pow" else None)
        return
    m = UN.match(name)
    if m:
        op, dt = m.groups()
        x = rand(dt, (41, 23), rng, positive=(op == "log"))
        xd, xst = strided(x)
        want = oracle.unary(op, np.ascontiguousarray(x))
        c = torch.empty((41, 23), dtype=torch.from_numpy(want[:1]).dtype, device="cuda")
        fn(P(xd), P(c), 2, sz([41, 23]), ss(xst), stream())
        check_float(c.cpu().numpy(), want, name, ulp=2 if op in ("sin", "cos", "exp", "log") else None)
        return
    m = CLAMP.match(name)
    if m:
        (dt,) = m.groups()
        x = rand(dt, (100,), rng)
        xd = torch.from_numpy(x).cuda()
        c = torch.empty_like(xd)
        fn.argtypes = [ctypes.c_void_p, ctypes.c_void_p, CT[dt], CT[dt], ctypes.c_int32, ctypes.c_void_p,
                       ctypes.c_void_p, ctypes.c_void_p]
        fn(P(xd), P(c), -0.5, 0.5, 1, sz([100]), ss([1]), stream())
        assert_bits_equal(c.cpu().numpy(), oracle.clamp(x, -0.5, 0.5), name)
        return
    m = CAST.match(name)
    if m:
        src, dst = m.groups()
        x = rand(src, (31, 17), rng) * (1 if np.dtype(NP[src]).kind not in "f" else 40)
        x = x.astype(NP[src])
        xd, xst = strided(x)
        c = torch.empty((31, 17), dtype=torch.from_numpy(np.zeros(1, NP[dst])).dtype, device="cuda")
        fn(P(xd), P(c), 2, sz([31, 17]), ss(xst), stream())
        assert_bits_equal(c.cpu().numpy(), oracle.cast(np.ascontiguousarray(x), oracle.code_of(np.dtype(NP[dst]))),
                          name)
        return
    m = RED.match(name) or SMALL.match(name)
    if m:
        op, dt = m.groups()
        x = rand(dt, (19, 53), rng, positive=(op == "prod"))
        if op == "prod" and np.dtype(NP[dt]).kind in "f":
            x = (np.float64(0.9) + rng.random((19, 53)) * 0.2).astype(NP[dt])
        if op == "prod" and np.dtype(NP[dt]).kind == "c":
            x = (np.exp(1j * rng.random((19, 53)))).astype(NP[dt])
        if op == "prod" and np.dtype(NP[dt]).kind == "i":
            x = rng.integers(1, 3, (19, 53)).astype(NP[dt])
        xd, xst = strided(x)
        for axis in (0, 1):
            L_, M_ = x.shape[axis], x.shape[1 - axis]
            out_dt = torch.int64 if op in ("argmax", "argmin") else torch.from_numpy(x[:1, :1]).dtype
            c = torch.empty(M_, dtype=out_dt, device="cuda")
            args = [P(xd), P(c), 2, sz(list(x.shape)), ss(xst), axis, SZ(L_), SZ(M_)]
            if SMALL.match(name):
                args.append(ctypes.c_int32(16))
            fn(*args, stream())
            _reduce_check(op, c.cpu().numpy(), np.ascontiguousarray(x), axis, oracle, f"{name} axis {axis}")
        return
    m = PART.match(name)
    if m:
        op, dt = m.groups()
        Lr, M_, tiles = 3000, 5, 3
        x = rand(dt, (M_, Lr), rng)
        if op == "prod":
            x = (np.exp(1j * rng.random((M_, Lr)) * 0.001) if np.dtype(NP[dt]).kind == "c"
                 else (np.float64(0.9999) + rng.random((M_, Lr)) * 0.0002) if np.dtype(NP[dt]).kind == "f"
                 else np.ones((M_, Lr))).astype(NP[dt])
        xd = torch.from_numpy(x).cuda()
        part = torch.empty(M_ * tiles, dtype=xd.dtype, device="cuda")
        fn(P(xd), P(part), 2, sz([M_, Lr]), ss([Lr, 1]), 1, SZ(Lr), SZ(M_), SZ(tiles), stream())
        c = torch.empty(M_, dtype=xd.dtype, device="cuda")
        fin = getattr(L, name.replace("_partial_", "_final_"))
        if op == "mean" or dt in ("c64", "c128"):  # these finals also take axis_len
            fin(P(part), P(c), SZ(tiles), SZ(M_), SZ(Lr), stream())
        else:
            fin(P(part), P(c), SZ(tiles), SZ(M_), stream())
        _reduce_check(op, c.cpu().numpy(), x, 1, oracle, name + " + final")
        return
    m = APART.match(name)
    if m:
        op, dt = m.groups()
        Lr, M_ = 5000, 3
        tiles = (Lr + 1023) // 1024
        x = rand(dt, (M_, Lr), rng)
        x[1, 123] = x[1, 4000] = x.max() + 1 if op == "argmax" else x.min() - 1
        xd = torch.from_numpy(x).cuda()
        pv = torch.empty(M_ * tiles, dtype=xd.dtype, device="cuda")
        pi = torch.empty(M_ * tiles, dtype=torch.int64, device="cuda")
        fn(P(xd), P(pv), P(pi), 2, sz([M_, Lr]), ss([Lr, 1]), 1, SZ(Lr), SZ(M_), SZ(tiles), stream())
        groups = (tiles + 1023) // 1024
        ov = torch.empty(M_ * groups, dtype=xd.dtype, device="cuda")
        oi = torch.empty(M_ * groups, dtype=torch.int64, device="cuda")
        getattr(L, name.replace("_partial_", "_mid_"))(P(pv), P(pi), P(ov), P(oi), SZ(M_), SZ(tiles), SZ(Lr),
                                                        stream())
        c = torch.empty(M_, dtype=torch.int64, device="cuda")
        getattr(L, name.replace("_partial_", "_final_"))(P(ov), P(oi), P(c), SZ(groups), SZ(M_), stream())
        assert_bits_equal(c.cpu().numpy(), oracle.reduce(op, x, 1), name + " + mid + final")
        return
    m = CUMSUM.match(name)
    if m:
        (dt,) = m.groups()
        Lr = 3000
        x = rand(dt, (3, Lr), rng)
        xd = torch.from_numpy(x).cuda()
        bpr = (Lr + 255) // 256
        tmp = torch.empty(3 * bpr, dtype=xd.dtype, device="cuda")
        c = torch.empty_like(xd)
        fn(P(xd), P(c), P(tmp), 2, sz([3, Lr]), ss([Lr, 1]), 1, SZ(Lr), SZ(3 * Lr), stream())
        want = oracle.cumsum(x, 1)
        if np.dtype(NP[dt]).kind == "i":
            assert_bits_equal(c.cpu().numpy(), want, name)
        else:
            assert_sum_close(c.cpu().numpy(), want, oracle.cumsum(np.abs(x).astype(np.float64), 1), 1e-5, name)
        return
    m = FILL.match(name)
    if m:
        (dt,) = m.groups()
        c = torch.zeros(1001, dtype=torch.from_numpy(np.zeros(1, NP[dt])).dtype, device="cuda")
        fn.argtypes = [ctypes.c_void_p, CT[dt], SZ, ctypes.c_void_p]
        fn(P(c), 7, 1001, stream())
        assert (c.cpu().numpy() == 7).all(), name
        return
    m = ARANGE.match(name)
    if m:
        (dt,) = m.groups()
        c = torch.empty(1003, dtype=torch.from_numpy(np.zeros(1, NP[dt])).dtype, device="cuda")
        fn.argtypes = [ctypes.c_void_p, CT[dt], CT[dt], SZ, ctypes.c_void_p]
        start, step = (0.5, 0.25) if dt in ("f32", "f64") else (-5, 3)
        fn(P(c), start, step, 1003, stream())
        T = NP[dt]
        want = (T(start) + np.arange(1003).astype(T) * T(step)).astype(T)
        assert_bits_equal(c.cpu().numpy(), want, name)
        return
    m = LINSPACE.match(name)
    if m:
        (dt,) = m.groups()
        T = NP[dt]
        c = torch.empty(101, dtype=torch.from_numpy(np.zeros(1, T)).dtype, device="cuda")
        fn.argtypes = [ctypes.c_void_p, CT[dt], CT[dt], SZ, ctypes.c_void_p]
        fn(P(c), -1.0, 3.0, 101, stream())
        step = (T(3.0) - T(-1.0)) / T(100)
        assert_bits_equal(c.cpu().numpy(), (T(-1.0) + np.arange(101).astype(T) * step).astype(T), name)
        return
    m = EYE.match(name)
    if m:
        (dt,) = m.groups()
        c = torch.empty((5, 7), dtype=torch.from_numpy(np.zeros(1, NP[dt])).dtype, device="cuda")
        fn(P(c), SZ(5), SZ(7), ctypes.c_int32(-1), stream())
        assert_bits_equal(c.cpu().numpy(), np.eye(5, 7, -1, dtype=NP[dt]), name)
        return
    m = COPYT.match(name)
    if m:
        (dt,) = m.groups()
        x = rand(dt, (70, 130), rng)  # src is (cols, rows)
        xd = torch.from_numpy(x).cuda()
        dst = torch.empty((130, 70), dtype=xd.dtype, device="cuda")
        fn(P(xd), P(dst), SZ(130), SZ(70), stream())
        assert_bits_equal(dst.cpu().numpy(), np.ascontiguousarray(x.T), name)
        return
    m = COPY.match(name)
    if m:
        (dt,) = m.groups()
        x = rand(dt, (40, 60), rng)
        xd, xst = strided(x)
        c = torch.empty((40, 60), dtype=xd.dtype, device="cuda")
        fn(P(xd), P(c), 2, sz([40, 60]), ss(xst), stream())
        assert_bits_equal(c.cpu().numpy(), x, name)
        return
    pytest.fail(f"no dispatch for {name}")
