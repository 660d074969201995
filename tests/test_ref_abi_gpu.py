"""musapy's kernel C-ABI (include/musapy_kernels_v2.h), called through
ctypes the way musapy's operator layer calls it (size_t shapes, ssize_t
strides, caller-owned partial buffers and cumsum tmp), checked against the
oracle."""
import ctypes

import numpy as np
import pytest
import torch

from tests.helpers import assert_bits_equal, assert_sum_close

pytestmark = pytest.mark.gpu

SZ = ctypes.c_size_t
SS = ctypes.c_ssize_t


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


def dev(x):
    return torch.from_numpy(np.ascontiguousarray(x)).cuda()


def test_binary_broadcast_f32(oracle):
    rng = np.random.default_rng(0)
    a = rng.random((4096, 1), dtype=np.float32)
    b = rng.random(4096, dtype=np.float32)
    c = torch.empty((4096, 4096), dtype=torch.float32, device="cuda")
    ad, bd = dev(a), dev(b)  # keep the device buffers alive across the launch
    lib().musapy_add_f32_v2(P(ad), P(bd), P(c), 2, sz([4096, 4096]), ss([1, 0]), ss([0, 1]), stream())
    assert_bits_equal(c.cpu().numpy(), oracle.binary("add", a, b), "musapy_add_f32_v2")


def test_cast_i64_f64_transposed(oracle):
    A = np.random.default_rng(2).integers(-1000, 1001, (300, 200)).astype(np.int64)
    c = torch.empty((200, 300), dtype=torch.float64, device="cuda")
    Ad = dev(A)
    lib().musapy_cast_i64_f64_v2(P(Ad), P(c), 2, sz([200, 300]), ss([1, 200]), stream())
    assert_bits_equal(c.cpu().numpy(), A.T.astype(np.float64), "musapy_cast_i64_f64_v2")


def test_compare_and_clamp(oracle):
    rng = np.random.default_rng(3)
    a, b = rng.standard_normal(1000).astype(np.float32), rng.standard_normal(1000).astype(np.float32)
    c = torch.empty(1000, dtype=torch.uint8, device="cuda")
    ad, bd = dev(a), dev(b)
    lib().musapy_lt_f32_v2(P(ad), P(bd), P(c), 1, sz([1000]), ss([1]), ss([1]), stream())
    assert_bits_equal(c.cpu().numpy().view(np.bool_), oracle.compare("lt", a, b), "musapy_lt_f32_v2")
    out = torch.empty(1000, dtype=torch.float32, device="cuda")
    f = lib().musapy_clamp_f32_v2
    f.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_float, ctypes.c_float, ctypes.c_int32,
                  ctypes.POINTER(SZ), ctypes.POINTER(SS), ctypes.c_void_p]
    f(P(ad), P(out), -0.5, 0.5, 1, sz([1000]), ss([1]), stream())
    assert_bits_equal(out.cpu().numpy(), oracle.clamp(a, -0.5, 0.5), "musapy_clamp_f32_v2")


def test_reduce_one_launch_and_small_axis(oracle):
    x = np.random.default_rng(4).standard_normal((64, 300)).astype(np.float32)
    xd = dev(x)
    for name, op, od in [("sum", "sum", torch.float32), ("max", "max", torch.float32),
                         ("argmax", "argmax", torch.int64), ("mean", "mean", torch.float32)]:
        c = torch.empty(64, dtype=od, device="cuda")
        getattr(lib(), f"musapy_{name}_f32_v2")(P(xd), P(c), 2, sz([64, 300]), ss([300, 1]), 1, SZ(300), SZ(64),
                                                 stream())
        got, want = c.cpu().numpy(), oracle.reduce(op, x, 1)
        if op in ("sum", "mean"):
            assert_sum_close(got, want, np.abs(x).sum(1) / (300 if op == "mean" else 1), 1e-5, name)
        else:
            assert_bits_equal(got, want, name)
    c = torch.empty(300, dtype=torch.float32, device="cuda")
    lib().musapy_min_small_axis_f32_v2(P(xd), P(c), 2, sz([64, 300]), ss([300, 1]), 0, SZ(64), SZ(300),
                                       ctypes.c_int32(64), stream())
    assert_bits_equal(c.cpu().numpy(), oracle.reduce("min", x, 0), "min_small_axis")


def test_partial_mid_final_pipeline(oracle):
    """musapy's multi-stage path (op_builder.rs:2519-3023): partial with
    tiles = ceil(L/1024) per output, optional mid stages, then final."""
    L, M = 40_000, 3
    x = np.random.default_rng(5).standard_normal((M, L)).astype(np.float32)
    x[1, 777] = 50.0
    x[1, 39_000] = 50.0
    xd = dev(x)
    tiles = (L + 1023) // 1024
    shape, st = sz([M, L]), ss([L, 1])
    for name in ["sum", "max", "mean"]:
        part = torch.empty(M * tiles, dtype=torch.float32, device="cuda")
        getattr(lib(), f"musapy_{name}_partial_f32_v2")(P(xd), P(part), 2, shape, st, 1, SZ(L), SZ(M), SZ(tiles),
                                                         stream())
        c = torch.empty(M, dtype=torch.float32, device="cuda")
        if name == "mean":
            lib().musapy_mean_final_f32_v2(P(part), P(c), SZ(tiles), SZ(M), SZ(L), stream())
        else:
            getattr(lib(), f"musapy_{name}_final_f32_v2")(P(part), P(c), SZ(tiles), SZ(M), stream())
        got, want = c.cpu().numpy(), oracle.reduce(name, x, 1)
        if name == "max":
            assert_bits_equal(got, want, name)
        else:
            assert_sum_close(got, want, np.abs(x).sum(1) / (L if name == "mean" else 1), 1e-5, name,
                             truth=oracle.reduce(name, x.astype(np.float64), 1))
    pv = torch.empty(M * tiles, dtype=torch.float32, device="cuda")
    pi = torch.empty(M * tiles, dtype=torch.int64, device="cuda")
    lib().musapy_argmax_partial_f32_v2(P(xd), P(pv), P(pi), 2, shape, st, 1, SZ(L), SZ(M), SZ(tiles), stream())
    groups = (tiles + 1023) // 1024
    ov = torch.empty(M * groups, dtype=torch.float32, device="cuda")
    oi = torch.empty(M * groups, dtype=torch.int64, device="cuda")
    lib().musapy_argmax_mid_f32_v2(P(pv), P(pi), P(ov), P(oi), SZ(M), SZ(tiles), SZ(L), stream())
    c = torch.empty(M, dtype=torch.int64, device="cuda")
    lib().musapy_argmax_final_f32_v2(P(ov), P(oi), P(c), SZ(groups), SZ(M), stream())
    assert_bits_equal(c.cpu().numpy(), oracle.reduce("argmax", x, 1), "argmax pipeline")


@pytest.mark.parametrize("L", [1000, 70_000])
def test_cumsum_v3_with_musapy_tmp(oracle, L):
    x = np.random.default_rng(6).random((3, L)).astype(np.float32)
    bpr = (L + 255) // 256
    elems = 3 * (bpr + (bpr + 255) // 256) if bpr > 256 else 3 * bpr
    tmp = torch.empty(max(1, elems), dtype=torch.float32, device="cuda")
    c = torch.empty((3, L), dtype=torch.float32, device="cuda")
    xd = dev(x)
    lib().musapy_cumsum_f32_v3(P(xd), P(c), P(tmp) if bpr > 1 else None, 2, sz([3, L]), ss([L, 1]), 1, SZ(L),
                               SZ(3 * L), stream())
    want = oracle.cumsum(x, 1)
    assert_sum_close(c.cpu().numpy(), want, oracle.cumsum(np.abs(x).astype(np.float64), 1), 1e-5, "cumsum_v3",
                     truth=oracle.cumsum(x.astype(np.float64), 1))


def test_copy_and_creation():
    x = np.random.default_rng(7).standard_normal((300, 500)).astype(np.float32)  # src is (cols, rows)
    dst = torch.empty((500, 300), dtype=torch.float32, device="cuda")
    xd = dev(x)
    lib().musapy_copy_transpose2d_f32(P(xd), P(dst), SZ(500), SZ(300), stream())
    assert_bits_equal(dst.cpu().numpy(), np.ascontiguousarray(x.T), "copy_transpose2d")
    out = torch.empty(1000, dtype=torch.float32, device="cuda")
    f = lib().musapy_arange_f32
    f.argtypes = [ctypes.c_void_p, ctypes.c_float, ctypes.c_float, SZ, ctypes.c_void_p]
    f(P(out), 0.5, 0.25, 1000, stream())
    want = np.float32(0.5) + np.arange(1000, dtype=np.float32) * np.float32(0.25)
    assert_bits_equal(out.cpu().numpy(), want, "arange")
    g = lib().musapy_linspace_f64
    g.argtypes = [ctypes.c_void_p, ctypes.c_double, ctypes.c_double, SZ, ctypes.c_void_p]
    out64 = torch.empty(11, dtype=torch.float64, device="cuda")
    g(P(out64), 0.0, 1.0, 11, stream())
    assert_bits_equal(out64.cpu().numpy(), 0.0 + np.arange(11) * ((1.0 - 0.0) / 10), "linspace")
    e = torch.empty((4, 6), dtype=torch.int32, device="cuda")
    lib().musapy_eye_i32(P(e), SZ(4), SZ(6), ctypes.c_int32(1), stream())
    assert_bits_equal(e.cpu().numpy(), np.eye(4, 6, 1, dtype=np.int32), "eye")
    h = lib().musapy_fill_f64
    h.argtypes = [ctypes.c_void_p, ctypes.c_double, SZ, ctypes.c_void_p]
    h(P(out64), 2.5, 11, stream())
    assert out64.cpu().numpy().tolist() == [2.5] * 11
