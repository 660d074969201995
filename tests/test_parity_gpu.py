"""GPU parity: the CUDA engine against the oracle (the reference CPU path
restated in oracle/oracle.c) on the same seeded inputs.

Bars (the north-star parity contract):
  * bit-exact: integer / bool / comparison / argmax / argmin / cast / max /
    min / IEEE add-sub-mul-div / complex arithmetic;
  * <= 2 ulp: sin / cos / exp / log / pow;
  * sums, means, cumsums: |gpu - cpu| <= rtol * sum|x| with rtol 1e-5 (f32)
    or 1e-12 (f64).
"""
import zlib

import numpy as np
import pytest

from tests.helpers import assert_bits_equal, assert_sum_close, assert_ulp

pytestmark = pytest.mark.gpu

RTOL = {np.dtype(np.float32): 1e-5, np.dtype(np.float64): 1e-12}


def dev(ms, x):
    return ms.from_numpy(np.asarray(x), device="cuda:0")


def rand(rng, shape, dtype):
    dtype = np.dtype(dtype)
    if dtype.kind == "f":
        return rng.standard_normal(shape).astype(dtype)
    if dtype.kind == "c":
        return (rng.standard_normal(shape) + 1j * rng.standard_normal(shape)).astype(dtype)
    if dtype == np.bool_:
        return rng.random(shape) < 0.5
    info = np.iinfo(dtype)
    return rng.integers(max(info.min, -1000), min(info.max, 1000), size=shape).astype(dtype)


# ------------------------------------------------------------- config 1
def test_config1_broadcast_add_and_row_sum(ms, oracle):
    """The CPU-runnable broadcast case: f32 (4096,1) + (4096,) drawn uniform[-1,1)
    from numpy PCG64 seed 0, then sum(axis=1)."""
    rng = np.random.default_rng(0)
    a = rng.random((4096, 1), dtype=np.float32) * 2 - 1
    b = rng.random(4096, dtype=np.float32) * 2 - 1
    c = ms.add(dev(ms, a), dev(ms, b))
    want = oracle.binary("add", a, b)
    assert_bits_equal(c.numpy(), want, "config1 add")
    s = ms.sum(c, axis=1).numpy()
    assert_sum_close(s, oracle.reduce("sum", want, axis=1), np.abs(want).sum(axis=1), 1e-5, "config1 sum")


# ------------------------------------------------------ binary arithmetic
VIEWS = ["contig", "bcast_row", "bcast_col", "scalar", "transposed", "flipped", "offset_slice", "strided"]


def make_operands(rng, view, dtype):
    if view == "contig":
        return rand(rng, (37, 129), dtype), rand(rng, (37, 129), dtype)
    if view == "bcast_row":
        return rand(rng, (64, 256), dtype), rand(rng, (256,), dtype)
    if view == "bcast_col":
        return rand(rng, (64, 1), dtype), rand(rng, (64, 256), dtype)
    if view == "scalar":
        return rand(rng, (), dtype), rand(rng, (5, 7, 9), dtype)
    if view == "transposed":
        return rand(rng, (96, 80), dtype).T, rand(rng, (80, 96), dtype)
    if view == "flipped":
        return rand(rng, (33, 65), dtype)[::-1, ::-1], rand(rng, (33, 65), dtype)
    if view == "offset_slice":
        return rand(rng, (1001,), dtype)[1:1001], rand(rng, (1000,), dtype)
    return rand(rng, (40, 60, 8), dtype)[::2, 1::3, :], rand(rng, (20, 20, 8), dtype)[:, ::-1]


def to_dev_view(ms, x):
    """Device array with the same strides/offset as a numpy view."""
    base = x
    while base.base is not None and isinstance(base.base, np.ndarray):
        base = base.base
    if x.size == 0 or x.flags.c_contiguous:
        return dev(ms, x)
    # rebuild through the device: copy the base, then take an equivalent view
    bd = dev(ms, base)
    off = (x.__array_interface__["data"][0] - base.__array_interface__["data"][0]) // x.itemsize
    from musapy_b200.array import _view

    return _view(bd, x.shape, [s // x.itemsize for s in x.strides], off)


@pytest.mark.parametrize("dtype", [np.float32, np.float64])
@pytest.mark.parametrize("op", ["add", "sub", "mul", "div"])
@pytest.mark.parametrize("view", VIEWS)
def test_binary_bit_exact(ms, oracle, dtype, op, view):
    rng = np.random.default_rng(zlib.crc32(f"{op}/{view}".encode()))
    a, b = make_operands(rng, view, dtype)
    got = getattr(ms, op)(to_dev_view(ms, a), to_dev_view(ms, b)).numpy()
    assert_bits_equal(got, oracle.binary(op, a, b), f"{op} {view}")


@pytest.mark.parametrize("dtype", [np.float32, np.float64])
def test_pow_ulp(ms, oracle, dtype):
    rng = np.random.default_rng(3)
    a = (0.1 + 3.9 * rng.random(100_000)).astype(dtype)
    b = (-2 + 4 * rng.random(100_000)).astype(dtype)
    got = ms.pow(dev(ms, a), dev(ms, b)).numpy()
    assert_ulp(got, oracle.binary("pow", a, b), 2, "pow")


def test_binary_special_values(ms, oracle):
    v = np.array([0.0, -0.0, 1.0, -1.0, np.inf, -np.inf, np.nan, 1e-45, 3.4e38, -3.4e38], np.float32)
    a, b = np.meshgrid(v, v)
    for op in ["add", "sub", "mul", "div"]:
        got = getattr(ms, op)(dev(ms, a), dev(ms, b)).numpy()
        assert_bits_equal(got, oracle.binary(op, a, b), op)
    assert_ulp(ms.pow(dev(ms, np.abs(a)), dev(ms, b)).numpy(), oracle.binary("pow", np.abs(a), b), 2, "pow special")


def test_mixed_dtype_transposed_promotion(ms, oracle):
    """Config 2 (small): int64 A^T + float64 row -> float64 (fused cast)."""
    rng = np.random.default_rng(2)
    A = rng.integers(-1000, 1001, (512, 384)).astype(np.int64)
    row = rng.standard_normal(512)
    got = ms.add(ms.transpose(dev(ms, A)), dev(ms, row))
    assert got.dtype == ms.float64
    assert_bits_equal(got.numpy(), oracle.binary("add", A.T, row), "i64^T + f64")


def test_gpu_narrow_promotion(ms, oracle):
    """On the device musapy promotes f32+f64 to the narrower f32 (dtype.rs:302-338)."""
    rng = np.random.default_rng(4)
    a = rng.standard_normal(1000).astype(np.float32)
    b = rng.standard_normal(1000)
    got = ms.add(dev(ms, a), dev(ms, b))
    assert got.dtype == ms.float32
    assert_bits_equal(got.numpy(), oracle.binary("add", a, b, all_gpu=True), "f32 + f64 on device")


# --------------------------------------------------------------- complex
@pytest.mark.parametrize("dtype", [np.complex64, np.complex128])
@pytest.mark.parametrize("op", ["add", "sub", "mul", "div"])
def test_complex_bit_exact(ms, oracle, dtype, op):
    rng = np.random.default_rng(5)
    a, b = rand(rng, (3000,), dtype), rand(rng, (3000,), dtype)
    got = getattr(ms, op)(dev(ms, a), dev(ms, b)).numpy()
    assert_bits_equal(got, oracle.binary(op, a, b), f"{op} {dtype}")


@pytest.mark.parametrize("dtype", [np.complex64, np.complex128])
def test_complex_unary_and_compare(ms, oracle, dtype):
    rng = np.random.default_rng(6)
    a = rand(rng, (2000,), dtype)
    b = a.copy()
    b[::3] += 1
    assert_bits_equal(ms.neg(dev(ms, a)).numpy(), oracle.unary("neg", a), "neg")
    assert_bits_equal(ms.abs(dev(ms, a)).numpy(), oracle.unary("abs", a), "abs")
    assert_bits_equal(ms.eq(dev(ms, a), dev(ms, b)).numpy(), oracle.compare("eq", a, b), "eq")
    assert_bits_equal(ms.ne(dev(ms, a), dev(ms, b)).numpy(), oracle.compare("ne", a, b), "ne")


# ----------------------------------------------------------------- unary
@pytest.mark.parametrize("dtype", [np.float32, np.float64])
@pytest.mark.parametrize("op", ["sin", "cos", "exp", "log"])
def test_transcendental_ulp(ms, oracle, dtype, op):
    rng = np.random.default_rng(7)
    x = rng.standard_normal(200_000).astype(dtype) * 10
    if op == "log":
        x = np.abs(x) + np.asarray(1e-30, dtype)
    if op == "exp":
        x = x * 8
    got = getattr(ms, op)(dev(ms, x)).numpy()
    assert_ulp(got, oracle.unary(op, x), 2, op)


@pytest.mark.parametrize("dtype", [np.float32, np.float64])
@pytest.mark.parametrize("op", ["abs", "sign", "neg"])
def test_simple_unary_exact(ms, oracle, dtype, op):
    x = np.array([0.0, -0.0, 1.5, -2.5, np.inf, -np.inf, np.nan, 1e-300 if dtype == np.float64 else 1e-40], dtype)
    x = np.concatenate([x, np.random.default_rng(8).standard_normal(1000).astype(dtype)])
    assert_bits_equal(getattr(ms, op)(dev(ms, x)).numpy(), oracle.unary(op, x), op)


@pytest.mark.parametrize("dtype", [np.float32, np.float64])
def test_clamp_exact(ms, oracle, dtype):
    x = np.concatenate([np.array([np.nan, -np.inf, np.inf, -0.0, 0.5, -0.5], dtype),
                        np.random.default_rng(9).standard_normal(5000).astype(dtype)])
    got = ms.clamp(dev(ms, x), -0.5, 0.5).numpy()
    assert_bits_equal(got, oracle.clamp(x, -0.5, 0.5), "clamp")


def test_config2_chain_small(ms, oracle):
    """Config 2 chain exp(sin(x)) -> clamp(-0.5, 0.5) on N(0,1) f32, per call."""
    x = np.random.default_rng(2).standard_normal(1 << 18, dtype=np.float32)
    s = ms.sin(dev(ms, x))
    s_want = oracle.unary("sin", x)
    assert_ulp(s.numpy(), s_want, 2, "sin")
    e = ms.exp(s)
    e_want = oracle.unary("exp", s.numpy())
    assert_ulp(e.numpy(), e_want, 2, "exp")
    c = ms.clamp(e, -0.5, 0.5)
    assert_bits_equal(c.numpy(), oracle.clamp(e.numpy(), -0.5, 0.5), "clamp")


# ----------------------------------------------------------- comparisons
@pytest.mark.parametrize("dtype", [np.float32, np.float64, np.float16, np.int64, np.int32])
@pytest.mark.parametrize("op", ["eq", "ne", "lt", "gt", "le", "ge"])
def test_compare_exact(ms, oracle, dtype, op):
    rng = np.random.default_rng(10)
    a = rand(rng, (300, 20), dtype)
    b = a.copy()
    b[::2] = rand(rng, b[::2].shape, dtype)
    if np.dtype(dtype).kind == "f":
        a[0, :4] = [np.nan, 0.0, -0.0, np.inf]
        b[0, :4] = [np.nan, -0.0, 0.0, np.inf]
    got = getattr(ms, op)(dev(ms, a), dev(ms, b))
    assert got.dtype == ms.bool_
    assert_bits_equal(got.numpy(), oracle.compare(op, a, b), op)
    # broadcast against a row
    got = getattr(ms, op)(dev(ms, a), dev(ms, b[0])).numpy()
    assert_bits_equal(got, oracle.compare(op, a, b[0]), op + " bcast")


# ------------------------------------------------------------------ casts
CASTS = [("float32", "bfloat16"), ("bfloat16", "float32"), ("float32", "float16"), ("float16", "float32"),
         ("float64", "float32"), ("float32", "float64"), ("int64", "float64"), ("int64", "float32"),
         ("float64", "int64"), ("float32", "int64"), ("int32", "float32"), ("uint64", "float32"),
         ("float64", "float16"), ("float64", "bfloat16"), ("int8", "float64"), ("float32", "int8"),
         ("float32", "uint8"), ("float32", "bool"), ("complex64", "complex128"), ("float32", "complex64"),
         ("float64", "complex128"), ("uint8", "int64"), ("int64", "int16")]


@pytest.mark.parametrize("src,dst", CASTS)
def test_cast_exact(ms, oracle, src, dst):
    rng = np.random.default_rng(11)
    sd = oracle.np_of(oracle.NAMES.index(src))
    if sd.kind == "f" or src == "bfloat16":
        x = (rng.standard_normal(20000) * np.exp(rng.uniform(-20, 20, 20000)))
        x = np.concatenate([x, [0.0, -0.0, np.inf, -np.inf, np.nan, 1e30, -1e30, 127.9, -128.9, 255.5, 3e9]])
        x = oracle.cast(x.astype(np.float64), oracle.NAMES.index(src))
    elif sd.kind == "c":
        x = rand(rng, (5000,), sd)
    else:
        info = np.iinfo(sd)
        x = rng.integers(info.min, info.max, size=20000, dtype=sd, endpoint=True)
    d = ms.from_numpy(x, device="cuda:0")
    got = d.astype(dst).numpy()
    want = oracle.cast(x, oracle.NAMES.index(dst))
    assert_bits_equal(got, want, f"{src}->{dst}")


@pytest.mark.parametrize("dtype", [np.uint8, np.float16, np.float32, np.float64, np.complex128])
@pytest.mark.parametrize("shape", [(64, 64), (1, 200), (130, 67), (3, 100, 129), (257, 33, 5)])
def test_tiled_transposed_copies(ms, dtype, shape):
    """contiguous() of views whose unit stride is on an outer dim (the tiled
    shared-memory path): interior and edge tiles, batch dims, every element
    size (16-byte elements use 32-wide tiles), bit-exact."""
    rng = np.random.default_rng(40)
    x = rng.standard_normal(shape)
    if np.dtype(dtype).kind == "c":
        x = x + 1j * rng.standard_normal(shape)
    x = x.astype(dtype) if np.dtype(dtype).kind != "u" else rng.integers(0, 256, shape).astype(dtype)
    xd = dev(ms, x)
    axes = tuple(reversed(range(x.ndim)))
    got = ms.contiguous(ms.transpose(xd)).numpy()
    assert_bits_equal(got, np.ascontiguousarray(np.transpose(x, axes)), f"transpose {shape}")
    if x.ndim == 3:
        perm = (0, 2, 1)
        got = ms.contiguous(ms.transpose(xd, perm)).numpy()
        assert_bits_equal(got, np.ascontiguousarray(np.transpose(x, perm)), f"permute {perm} {shape}")


def test_tiled_binary_both_operand_orders(ms, oracle):
    """Tiled path with the transposed operand first or second and the other
    operand a broadcast row, a broadcast column or a full array."""
    rng = np.random.default_rng(41)
    a = rng.standard_normal((190, 131)).astype(np.float32)
    at = dev(ms, a).T if hasattr(dev(ms, a), "T") else ms.transpose(dev(ms, a))
    ah = np.ascontiguousarray(a.T)
    for other in (rng.standard_normal(190).astype(np.float32), rng.standard_normal((131, 1)).astype(np.float32),
                  rng.standard_normal((131, 190)).astype(np.float32)):
        od = dev(ms, other)
        assert_bits_equal(ms.sub(at, od).numpy(), oracle.binary("sub", ah, other), "T - other")
        assert_bits_equal(ms.sub(od, at).numpy(), oracle.binary("sub", other, ah), "other - T")


def test_cast_strided_transposed(ms, oracle):
    x = np.random.default_rng(12).standard_normal((300, 500)).astype(np.float32)
    got = ms.transpose(dev(ms, x)).astype("bf16").numpy()
    want = oracle.cast(np.ascontiguousarray(x.T), oracle.BF16)
    assert_bits_equal(got, want, "transposed cast")
    assert_bits_equal(ms.contiguous(ms.transpose(dev(ms, x))).numpy(), np.ascontiguousarray(x.T), "contiguous")


# ------------------------------------------------------------ reductions
RED_SHAPES = [((256, 256), 0), ((256, 256), 1), ((100, 17), 1), ((1025, 5), 0), ((1025, 5), 1),
              ((7, 1024), 1), ((5000, 3), 0), ((3, 70000), 1), ((1_000_000,), None), ((2, 3, 4), (0, 2)),
              ((6, 50, 40), (1, 2)), ((6, 50, 40), (0, 1)), ((16, 33, 65), -1), ((4, 5, 6, 7), (0, 3))]


@pytest.mark.parametrize("shape,axis", RED_SHAPES)
@pytest.mark.parametrize("dtype", [np.float32, np.float64])
def test_reduce_float(ms, oracle, shape, axis, dtype):
    rng = np.random.default_rng(13)
    x = rng.standard_normal(shape).astype(dtype)
    xd = dev(ms, x)
    ax_abs = oracle.reduce("sum", np.abs(x).astype(np.float64), axis)
    for op in ["sum", "mean"]:
        got = getattr(ms, op)(xd, axis=axis).numpy()
        want = oracle.reduce(op, x, axis)
        truth = oracle.reduce(op, x.astype(np.float64), axis)
        L = x.size // max(1, want.size)
        bound = ax_abs / (L if op == "mean" else 1)
        assert_sum_close(got, want, bound, RTOL[np.dtype(dtype)], op, truth=truth)
    for op in ["max", "min", "argmax", "argmin"]:
        got = getattr(ms, op)(xd, axis=axis).numpy()
        assert_bits_equal(got, oracle.reduce(op, x, axis), f"{op} {shape} {axis}")


def test_reduce_prod_and_keepdims(ms, oracle):
    rng = np.random.default_rng(14)
    x = (0.5 + rng.random((64, 48))).astype(np.float32)
    # products of <= 64 factors stay well inside the f32 range
    for axis, v in [(0, x), (1, x), (None, x[:4, :10])]:
        got = ms.prod(dev(ms, v), axis=axis).numpy()
        want = oracle.reduce("prod", v, axis)
        np.testing.assert_allclose(got, want, rtol=1e-5)
    for op in ["sum", "max", "argmax", "mean"]:
        for axis in [0, 1, (0, 1)]:
            got = getattr(ms, op)(dev(ms, x), axis=axis, keepdims=True)
            want = oracle.reduce(op, x, axis, keepdims=True)
            assert got.shape == want.shape, (op, axis)


@pytest.mark.parametrize("keepdims", [False, True])
def test_reduce_multi_axis_into_out(ms, oracle, keepdims):
    """Reductions over several axes written into a caller's out= array: the
    one-pass kernels (sum, mean, argmax over merged axes) and the per-axis
    passes of float max/min (the last pass writes into out), with a NaN at
    the start of an inner run and signed zeros so the pass order shows."""
    rng = np.random.default_rng(16)
    x = rng.standard_normal((6, 40, 33)).astype(np.float32)
    x[2, 0, 0] = np.nan
    x[4, :, 5] = 0.0
    x[4, 3, 5] = -0.0
    xd = dev(ms, x)
    for op in ["sum", "mean", "max", "min", "argmax", "argmin"]:
        for axis in [(0, 2), (1, 2), (0, 1, 2)]:
            want = oracle.reduce(op, x, axis, keepdims=keepdims)
            dt = "i64" if op.startswith("arg") else "f32"
            out = ms.empty(want.shape, dt)
            got = getattr(ms, op)(xd, axis=axis, keepdims=keepdims, out=out)
            assert got is out
            if op in ("sum", "mean"):
                assert_sum_close(out.numpy(), want, oracle.reduce("sum", np.abs(x).astype(np.float64), axis,
                                                                  keepdims=keepdims), 1e-5, f"{op} {axis}")
            else:
                assert_bits_equal(out.numpy(), want, f"{op} {axis} keepdims={keepdims}")
    with pytest.raises(ms.ShapeError):
        ms.max(xd, axis=(0, 2), out=ms.empty((41,), "f32"))


def test_reduce_nan_ties_signed_zero(ms, oracle):
    """First occurrence on ties, NaN only when it is the first element,
    +0/-0 resolved by position - bit-identical to the sequential CPU loop."""
    cases = [
        [np.nan, 1.0, 5.0, 5.0],
        [1.0, np.nan, 5.0, 5.0, 2.0],
        [-0.0, 0.0, -1.0],
        [0.0, -0.0, -1.0],
        [np.nan, np.nan],
        [-np.inf, -np.inf],
        [3.0, 3.0, 3.0],
    ]
    for c in cases:
        for dtype in (np.float32, np.float64):
            x = np.array(c, dtype)
            for op in ["max", "min", "argmax", "argmin"]:
                assert_bits_equal(getattr(ms, op)(dev(ms, x)).numpy(), oracle.reduce(op, x, None), f"{op} {c}")
    # long rows (split / block kernels) with a NaN first and ties spread out
    x = np.zeros(1 << 20, np.float32)
    x[[5, 70000, 900000]] = 7.0
    for op in ["max", "argmax", "argmin", "min"]:
        assert_bits_equal(getattr(ms, op)(dev(ms, x)).numpy(), oracle.reduce(op, x, None), op + " long")
    x[0] = np.nan
    for op in ["max", "argmax"]:
        assert_bits_equal(getattr(ms, op)(dev(ms, x)).numpy(), oracle.reduce(op, x, None), op + " nan-first")
    m = np.random.default_rng(15).standard_normal((300, 700)).astype(np.float32)
    m[:, 0] = np.nan
    m[5, 3] = np.nan
    for axis in (0, 1):
        for op in ["max", "argmax", "min", "argmin"]:
            assert_bits_equal(getattr(ms, op)(dev(ms, m), axis=axis).numpy(), oracle.reduce(op, m, axis), f"{op} {axis}")


@pytest.mark.parametrize("shape,axis", RED_SHAPES)
@pytest.mark.parametrize("dtype", [np.float32, np.float64, np.float16])
def test_reduce_zero_extremum_sign(ms, oracle, shape, axis, dtype):
    """max over non-positive data (min over non-negative data) whose zeros are
    a random mix of +0 and -0: the result carries the sign of the first zero in
    index order, through every kernel kind (row, block, split, column, gather)."""
    rng = np.random.default_rng(16)
    x = -np.abs(rng.standard_normal(shape)).astype(dtype)
    z = rng.random(shape) < 0.02
    x[z] = np.where(rng.random(int(z.sum())) < 0.5, -0.0, 0.0).astype(dtype)
    for op, v in (("max", x), ("min", -x)):
        got = getattr(ms, op)(dev(ms, v), axis=axis).numpy()
        # the CPU path returns f32 for f16 input; the extremum is an input value
        want = oracle.reduce(op, v, axis).astype(got.dtype)
        assert_bits_equal(got, want, f"{op} {shape} {axis}")


@pytest.mark.parametrize("axis", [(0, 2), (1, 2), (0, 1), (0, 1, 2)])
def test_reduce_multi_axis_nan_runs(ms, oracle, axis):
    """max/min over several axes reduce one axis at a time (reduction.rs:118-223):
    a NaN at the start of an inner run hides that run from the next pass."""
    rng = np.random.default_rng(17)
    x = rng.standard_normal((6, 7, 9)).astype(np.float32)
    x[0, :, 3] = np.nan
    x[2, 4, 0] = np.nan
    x[:, 0, 5] = np.nan
    x[1, 1, 1] = 50.0
    x[0, 2, 0] = -0.0
    for op in ("max", "min"):
        got = getattr(ms, op)(dev(ms, x), axis=axis).numpy()
        assert_bits_equal(got, oracle.reduce(op, x, axis), f"{op} {axis}")
        got = getattr(ms, op)(dev(ms, x), axis=axis, keepdims=True).numpy()
        assert_bits_equal(got, oracle.reduce(op, x, axis, keepdims=True), f"{op} {axis} keepdims")


@pytest.mark.parametrize("dtype", [np.int64, np.int32, np.int8, np.uint8, np.bool_])
def test_reduce_int_exact(ms, oracle, dtype):
    rng = np.random.default_rng(16)
    x = rand(rng, (256, 256), dtype)
    for op in ["sum", "prod", "max", "min", "argmax", "argmin"]:
        for axis in [None, 0, 1]:
            got = getattr(ms, op)(dev(ms, x), axis=axis).numpy()
            assert_bits_equal(got, oracle.reduce(op, x, axis), f"{op} {axis}")
    got = ms.mean(dev(ms, x), axis=1)
    assert got.dtype == ms.float64
    assert_sum_close(got.numpy(), oracle.reduce("mean", x, 1), np.abs(x.astype(np.float64)).sum(1) / 256, 1e-12)


@pytest.mark.parametrize("dtype", [np.complex64, np.complex128])
def test_reduce_complex(ms, oracle, dtype):
    rng = np.random.default_rng(17)
    x = rand(rng, (30, 40), dtype)
    for op in ["sum", "mean", "prod"]:
        for axis in [None, 0, 1]:
            got = getattr(ms, op)(dev(ms, x), axis=axis).numpy()
            want = oracle.reduce(op, x, axis)
            np.testing.assert_allclose(got, want, rtol=1e-4 if dtype == np.complex64 else 1e-10)


def test_reduce_strided_views(ms, oracle):
    rng = np.random.default_rng(12)
    base = rng.random((64, 64), dtype=np.float32)
    v = base[:, ::-1]
    d = ms.flip(dev(ms, base), axis=1)
    t = ms.transpose(dev(ms, base))
    for op in ["max", "min", "argmax", "argmin"]:
        for axis in (0, 1, None):
            assert_bits_equal(getattr(ms, op)(d, axis=axis).numpy(), oracle.reduce(op, v, axis), f"flip {op}")
            assert_bits_equal(getattr(ms, op)(t, axis=axis).numpy(), oracle.reduce(op, base.T, axis), f"T {op}")
    for axis in (0, 1, None):
        assert_sum_close(ms.sum(d, axis=axis).numpy(), oracle.reduce("sum", v, axis),
                         oracle.reduce("sum", np.abs(v).astype(np.float64), axis), 1e-5)


def _col_plan(ms, a, axis, op="sum"):
    """(kind, splits, outputs per thread) the planner picks for reduction `op`
    of array `a` over `axis`."""
    import ctypes

    from musapy_b200._lib import LIB

    n = a.ndim
    M, L, S = ctypes.c_int64(), ctypes.c_int64(), ctypes.c_int64()
    v = ctypes.c_int()
    code = {"sum": 0, "max": 2, "argmax": 5, "argmin": 6}[op]
    kind = LIB.mpb_reduce_plan_at(code, n, (ctypes.c_int64 * n)(*a.shape), (ctypes.c_int64 * n)(*a.strides),
                                  ctypes.c_void_p(a.data_ptr), a.dtype.code, 1 << axis, ctypes.byref(M),
                                  ctypes.byref(L), ctypes.byref(S), ctypes.byref(v))
    return kind, S.value, v.value


# (dtype, shape, axis, view): views slice the kept inner dim so the base
# moves by one element (narrower loads or one output per thread) or flip the
# reduced axis (negative reduced stride)
COL_V_CASES = [
    (np.float32, (301, 256), 0, None), (np.float32, (301, 256), 0, "shift1"), (np.float32, (301, 256), 0, "shift2"),
    (np.float32, (301, 256), 0, "flip"), (np.float32, (9, 333, 64), 1, None), (np.float32, (20000, 64), 0, None),
    (np.float64, (301, 256), 0, None), (np.float64, (301, 256), 0, "shift1"), (np.float16, (301, 256), 0, None),
    (np.float16, (301, 256), 0, "shift2"), (np.int64, (301, 256), 0, None),
]


@pytest.mark.parametrize("dtype,shape,axis,view", COL_V_CASES)
def test_reduce_columns_several_outputs_per_thread(ms, oracle, dtype, shape, axis, view):
    """Column reductions whose threads take 2, 4 or 8 adjacent outputs with
    one 8- or 16-byte load per reduced step (and the one-per-thread kernel
    where a view's alignment rules that out), split and unsplit, against the
    oracle: max/min/argmax/argmin bit-exact (NaN first in a column, NaN
    later, signed zeros, ties), sums and means within 1e-5 * sum|x| (1e-3 for
    f16 results; bit-exact where the column is not split: the CPU path's
    order)."""
    rng = np.random.default_rng(41)
    x = rand(rng, shape, dtype)
    if np.dtype(dtype).kind == "f":
        idx = (slice(None),) * axis
        x[idx + (0, 3)] = np.nan            # NaN first in column 3
        x[idx + (5, 4)] = np.nan            # NaN later in column 4
        x[idx + (slice(None), 6)] = 0.0
        x[idx + (7, 6)] = -0.0              # zero extremum: sign of the first zero
        x[idx + (slice(None), 9)] = 2.0     # ties: the first index wins
    def viewed(a):
        """(device view, host array) of `a` under this case's view."""
        d = dev(ms, a)
        if view == "shift1":
            return d[..., 1:253], a[..., 1:253]
        if view == "shift2":
            return d[..., 2:254], a[..., 2:254]
        if view == "flip":
            return ms.flip(d, axis=axis), np.flip(a, axis=axis)
        return d, a

    xd, ref = viewed(x)
    size = np.dtype(dtype).itemsize
    kind, splits, per_thread = _col_plan(ms, xd, axis)
    kind_arg, _, per_thread_arg = _col_plan(ms, xd, axis, "argmax")
    assert kind in (4, 5) and kind_arg in (4, 5)
    if view is None:
        assert per_thread == 16 // size
        assert per_thread_arg == (8 if size <= 4 else 16) // size
    for op in ("max", "min", "argmax", "argmin"):
        if np.dtype(dtype) == np.float16 and op in ("max", "min"):
            want = oracle.reduce(op, ref, axis).astype(np.float16)
        else:
            want = oracle.reduce(op, ref, axis)
        assert_bits_equal(getattr(ms, op)(xd, axis=axis).numpy(), want,
                          f"{op} {view} {per_thread_arg if op.startswith('arg') else per_thread}/thread")
    half = np.dtype(dtype) == np.float16
    cd, clean = viewed(np.nan_to_num(x))
    for op in ("sum", "mean"):
        got = getattr(ms, op)(cd, axis=axis).numpy()
        # f16 sums accumulate in f32 on both sides and round once to f16
        want = oracle.reduce(op, clean, axis)
        want = want.astype(np.float16) if half else want
        if (np.dtype(dtype).kind == "i" and op == "sum") or (np.dtype(dtype).kind == "f" and splits == 1):
            assert_bits_equal(got, want, f"{op} {view} unsplit")
        else:
            L = clean.shape[axis]
            bound = oracle.reduce("sum", np.abs(clean).astype(np.float64), axis) / (L if op == "mean" else 1)
            assert_sum_close(got.astype(np.float64) if half else got, want.astype(np.float64) if half else want,
                             bound, 1e-3 if half else 1e-5, f"{op} {view}")


def test_reduce_columns_split_with_several_outputs_per_thread(ms, oracle):
    """Few columns and a long reduced dim: the planner splits the column
    kernel (4 outputs per thread, 2 for arg reductions), and the merge keeps
    the first occurrence across splits."""
    rng = np.random.default_rng(42)
    x = rng.standard_normal((100000, 1024)).astype(np.float32)
    x[99990, 7] = 50.0
    x[10, 7] = 50.0                          # tie across splits: index 10 wins
    x[0, 11] = np.nan
    xd = dev(ms, x)
    kind, splits, per_thread = _col_plan(ms, xd, 0)
    assert (kind, per_thread) == (5, 4) and splits > 1
    kind, splits, per_thread = _col_plan(ms, xd, 0, "argmax")
    assert (kind, per_thread) == (5, 2) and splits > 1
    for op in ("max", "min", "argmax", "argmin"):
        assert_bits_equal(getattr(ms, op)(xd, axis=0).numpy(), oracle.reduce(op, x, 0), op)
    y = np.nan_to_num(x)
    got = ms.sum(dev(ms, y), axis=0).numpy()
    assert_sum_close(got, oracle.reduce("sum", y, 0), oracle.reduce("sum", np.abs(y).astype(np.float64), 0), 1e-5)


# ---------------------------------------------------------------- cumsum
CUMSUM_CASES = [((4,), 0), ((2, 2), None), ((2, 2), 0), ((2, 2), 1), ((3, 70000), 1), ((1300,), 0), ((1537,), 0),
                ((100_000,), 0), ((262, 4096), 1), ((64, 33, 5), 1), ((5000, 7), 0), ((1 << 21,), None),
                ((400, 4097), -1), (((1 << 24) + 5,), None), ((5, 3_000_001), 1)]


@pytest.mark.parametrize("shape,axis", CUMSUM_CASES)
@pytest.mark.parametrize("dtype", [np.float32, np.float64, np.int64, np.int32])
def test_cumsum(ms, oracle, shape, axis, dtype):
    rng = np.random.default_rng(18)
    x = rand(rng, shape, dtype) if np.dtype(dtype).kind == "i" else rng.random(shape).astype(dtype)
    ms.ops.set_scan_status_check(True)
    got = ms.cumsum(dev(ms, x), axis=axis).numpy()
    ms.ops.set_scan_status_check(False)
    want = oracle.cumsum(x, axis)
    if np.dtype(dtype).kind == "i":
        assert_bits_equal(got, want, "cumsum int")
    else:
        absx = oracle.cumsum(np.abs(x).astype(np.float64), axis)
        truth = oracle.cumsum(x.astype(np.float64), axis)
        assert_sum_close(got, want, absx, RTOL[np.dtype(dtype)], "cumsum", truth=truth)


def test_cumsum_ones_boundaries(ms, oracle):
    """test_reduction.py:321-351: 65,536 / 65,537 / 1M ones in int64."""
    for n in (65536, 65537, 1_000_000):
        r = ms.cumsum(ms.ones(n, dtype="i64", device="cuda:0"), axis=0)
        assert ms.sum(r).item() == n * (n + 1) // 2
        assert r.numpy()[-1] == n


# ------------------------------------------------------------ edge cases
def test_empty_and_scalar(ms, oracle):
    e = dev(ms, np.zeros((0, 5), np.float32))
    assert ms.add(e, e).shape == (0, 5)
    assert ms.sum(e, axis=0).numpy().tolist() == [0.0] * 5
    assert ms.sum(e, axis=1).shape == (0,)
    s = dev(ms, np.array(3.0, np.float32))
    assert ms.add(s, s).item() == 6.0
    assert ms.cumsum(e).shape == (0,)


@pytest.mark.parametrize("op", ["sin", "cos", "exp", "log"])
def test_transcendental_special_values_f32(ms, oracle, op):
    """Edges of the float sin/cos/exp/log evaluation: signed zeros, inf, NaN,
    subnormals, arguments past the 2^20 reduction limit, exp's overflow and
    underflow thresholds, log near 1."""
    v = [0.0, -0.0, np.inf, -np.inf, np.nan, 1e-45, -1e-45, 1e-38, 3.4e38, -3.4e38, 1048575.9, 1048576.0,
         -1048577.0, 1e7, 12345678.0, 88.72, 88.73, 89.0, -87.3, -103.97, -103.98, -104.0, -150.0,
         1.0, 1.0000001, 0.99999994, 2.0, 0.5, np.pi / 2, np.pi, 3 * np.pi / 2, 1e-20, 710.0]
    x = np.array(v, np.float32)
    x = np.concatenate([x, np.random.default_rng(30).standard_normal(4096).astype(np.float32) * 1e5])
    got = getattr(ms, op)(dev(ms, x)).numpy()
    want = oracle.unary(op, x)
    assert_ulp(got, want, 2, op + " specials")
    zero = want == 0
    assert np.array_equal(np.signbit(got[zero]), np.signbit(want[zero])), op + ": signed zero"
    # the same inputs through the two-element (packed) path: contiguous, even length
    x2 = np.ascontiguousarray(np.repeat(x, 2))
    got2 = getattr(ms, op)(dev(ms, x2)).numpy()
    assert_bits_equal(got2[0::2], got, op + " paired vs single")


def test_f16_pow_special_values(ms, oracle):
    v = np.array([0.0, -0.0, 1.0, -1.0, 2.0, -2.0, 0.5, 65504.0, 6e-8, np.inf, -np.inf, np.nan, 3.0, -3.0],
                 np.float16)
    a, b = np.meshgrid(v, v)
    got = ms.pow(dev(ms, a), dev(ms, b)).numpy()
    assert_ulp(got, oracle.binary("pow", a, b), 2, "f16 pow specials")


@pytest.mark.parametrize("dtype,scalar", [(np.float32, 2.5), (np.float64, -1.0 / 3.0), (np.float16, 0.1),
                                          (np.int64, 2.5), (np.int32, -0.5), (np.float64, (1 << 60) + 3),
                                          (np.complex64, 1 + 2j), (np.float32, 3), (np.float32, 1e-46)])
def test_python_scalar_operands(ms, oracle, dtype, scalar):
    """Python scalars take the array operand's dtype (complex / float scalars
    widen integer arrays), are written on the device, and give the same bits as
    the oracle with the scalar as a 0-d array of that dtype."""
    rng = np.random.default_rng(50)
    x = rng.standard_normal(1000) * 10
    x = (x + 1j * rng.standard_normal(1000)).astype(dtype) if np.dtype(dtype).kind == "c" else \
        (x.astype(dtype) if np.dtype(dtype).kind == "f" else np.abs(x).astype(dtype))
    xd = dev(ms, x)
    got = ms.mul(xd, scalar)
    d = got.dtype
    want = oracle.binary("mul", x, np.array(scalar, dtype=ms.dtypes.to_numpy(d)), all_gpu=True)
    assert_bits_equal(got.numpy(), want, f"{dtype} * {scalar!r}")
    got_r = ms.sub(scalar, xd).numpy()
    want_r = oracle.binary("sub", np.array(scalar, dtype=ms.dtypes.to_numpy(d)), x, all_gpu=True)
    assert_bits_equal(got_r, want_r, f"{scalar!r} - {dtype}")


@pytest.fixture
def tma_switch():
    from musapy_b200._lib import LIB

    prev = LIB.mpb_ew_set_tma(-1)
    yield LIB
    LIB.mpb_ew_set_tma(prev)


@pytest.mark.parametrize("tma", [True, False])
@pytest.mark.parametrize("dtype", [np.float16, np.float32, np.float64, np.int64, np.uint16])
@pytest.mark.parametrize("shape", [(40, 104), (64, 256), (8, 4096), (1000, 8), (3, 40, 96), (2, 1000, 24),
                                   (37, 100)])
def test_tiled_tma_copies(ms, tma_switch, tma, dtype, shape):
    """contiguous() of transposed views through the TMA tile kernel and the
    shared-memory tile kernel: partial boxes along p and q, a batch dim,
    2-, 4- and 8-byte elements, and a view whose strides rule TMA out."""
    import ctypes

    LIB = tma_switch
    LIB.mpb_ew_set_tma(1 if tma else 0)
    rng = np.random.default_rng(42)
    x = rng.standard_normal(shape) * 1000
    x = x.astype(dtype) if np.dtype(dtype).kind == "f" else rng.integers(-30000, 30000, shape).astype(dtype)
    xd = dev(ms, x)
    perm = tuple(range(x.ndim - 2)) + (x.ndim - 1, x.ndim - 2)
    n0 = LIB.mpb_ew_tma_launches()
    got = ms.contiguous(ms.transpose(xd, perm)).numpy()
    assert_bits_equal(got, np.ascontiguousarray(np.transpose(x, perm)), f"transpose {shape}")
    isz = np.dtype(dtype).itemsize
    # the TMA kernel serves 2- and 8-byte elements (4-byte ones measured
    # faster on the shared-memory tile kernel)
    eligible = isz != 4 and (shape[-1] * isz) % 16 == 0 and shape[-2] % (16 // isz) == 0
    assert (LIB.mpb_ew_tma_launches() > n0) == (tma and eligible), "TMA path taken iff enabled and eligible"
    flag = ctypes.c_int(-1)
    assert LIB.mpb_ew_wait_status(ctypes.byref(flag)) == 0 and flag.value == 0


@pytest.mark.parametrize("tma", [True, False])
def test_tiled_tma_binary(ms, oracle, tma_switch, tma):
    """Binary ops with a transposed operand on both kernels: the other
    operand a row (constant along p), a column or a full array, in both
    operand orders, and musapy's int64-transposed + float64-row promotion."""
    LIB = tma_switch
    LIB.mpb_ew_set_tma(1 if tma else 0)
    rng = np.random.default_rng(43)
    a = rng.standard_normal((200, 136)).astype(np.float32)
    at = ms.transpose(dev(ms, a))
    ah = np.ascontiguousarray(a.T)
    for other in (rng.standard_normal(200).astype(np.float32), rng.standard_normal((136, 1)).astype(np.float32),
                  rng.standard_normal((136, 200)).astype(np.float32)):
        od = dev(ms, other)
        assert_bits_equal(ms.sub(at, od).numpy(), oracle.binary("sub", ah, other), "T - other")
        assert_bits_equal(ms.div(od, at).numpy(), oracle.binary("div", other, ah), "other / T")
    A = rng.integers(-1000, 1001, (96, 160), dtype=np.int64)
    row = rng.standard_normal(96)
    got = ms.add(ms.transpose(dev(ms, A)), dev(ms, row)).numpy()
    want = oracle.binary("add", np.ascontiguousarray(A.T), row)
    assert_bits_equal(got, want, "int64^T + float64 row")
    got = ms.add(dev(ms, row), ms.transpose(dev(ms, A))).numpy()
    assert_bits_equal(got, oracle.binary("add", row, np.ascontiguousarray(A.T)), "float64 row + int64^T")
    # the row operand carried in the TMA stages, with a last tile row of 4
    # values (100 = 3 * 32 + 4) and of 10 (202 = 6 * 32 + 10)
    n0 = LIB.mpb_ew_tma_launches()
    A = rng.integers(-1000, 1001, (100, 160), dtype=np.int64)
    row = rng.standard_normal(100)
    got = ms.add(ms.transpose(dev(ms, A)), dev(ms, row)).numpy()
    assert_bits_equal(got, oracle.binary("add", np.ascontiguousarray(A.T), row), "int64^T (100 cols) + f64 row")
    d = rng.standard_normal((202, 136))
    r = rng.standard_normal(202)
    got = ms.sub(ms.transpose(dev(ms, d)), dev(ms, r)).numpy()
    assert_bits_equal(got, oracle.binary("sub", np.ascontiguousarray(d.T), r), "f64^T (202 cols) - f64 row")
    assert (LIB.mpb_ew_tma_launches() - n0 == 2) == tma


@pytest.mark.parametrize("tma", [True, False])
@pytest.mark.parametrize("dtype", [np.float16, np.float64])
def test_tiled_tma_sliced_views(ms, tma_switch, tma, dtype):
    """Transposed slices: a 16-byte aligned window (TMA box loads from an
    offset base, extents smaller than the row pitch) and an unaligned one
    (the shared-memory tile kernel), bit-exact either way."""
    LIB = tma_switch
    LIB.mpb_ew_set_tma(1 if tma else 0)
    rng = np.random.default_rng(44)
    x = (rng.standard_normal((96, 160)) * 100).astype(dtype)
    xd = dev(ms, x)
    e = 16 // np.dtype(dtype).itemsize
    for r0, c0, r1, c1 in ((8, 2 * e, 88, 160 - e), (1, 1, 95, 150)):
        view = ms.transpose(xd[r0:r1, c0:c1])
        want = np.ascontiguousarray(x[r0:r1, c0:c1].T)
        assert_bits_equal(ms.contiguous(view).numpy(), want, f"slice {(r0, c0, r1, c1)}")
        assert_bits_equal(ms.add(view, view).numpy(), (want.astype(np.float64) * 2).astype(dtype), "view + view")


@pytest.mark.parametrize("shape", [(0,), (0, 5), (5, 0), (3, 0, 4)])
@pytest.mark.parametrize("dtype", [np.float32, np.float64, np.int64, np.float16])
def test_zero_size_every_family(ms, oracle, shape, dtype):
    """Zero-size operands through every op family: results keep the
    broadcast shape, empty reductions give the identity (sum 0, prod 1, mean
    NaN as the CPU path divides 0 by a count of 0) or raise for max/min/
    argmax/argmin, and cumsum, casts and transposed views stay empty."""
    x = np.zeros(shape, dtype)
    xd = dev(ms, x)
    is_f = np.dtype(dtype).kind == "f"
    if is_f:  # musapy's arithmetic whitelist is floating point
        for name in ("add", "sub", "mul", "div", "pow"):
            assert getattr(ms, name)(xd, xd).shape == shape, name
            assert getattr(ms, name)(xd, dev(ms, np.ones(shape[-1:], dtype))).shape == shape, name + " broadcast"
    for name in ("eq", "lt"):
        r = getattr(ms, name)(xd, xd)
        assert r.shape == shape and r.dtype == ms.bool_, name
    if is_f:
        for name in ("sin", "exp", "abs", "neg"):
            assert getattr(ms, name)(xd).shape == shape, name
        assert ms.clamp(xd, -1.0, 1.0).shape == shape
    assert xd.astype("f64").shape == shape
    assert ms.contiguous(ms.transpose(xd)).shape == tuple(reversed(shape))
    if dtype == np.float16:  # musapy's cumsum takes integers, f32 and f64
        with pytest.raises(ms.DtypeError):
            ms.cumsum(xd)
    else:
        assert ms.cumsum(xd).shape == (0,)
    for axis in range(len(shape)):
        out_shape = shape[:axis] + shape[axis + 1:]
        for name in ("sum", "prod", "mean"):
            got = getattr(ms, name)(xd, axis=axis).numpy()
            assert got.shape == out_shape, (name, axis)
            if got.size and shape[axis] == 0:
                want = {"sum": 0.0, "prod": 1.0, "mean": np.nan}[name]
                np.testing.assert_array_equal(got.astype(np.float64), np.full(out_shape, want), err_msg=name)
        for name in ("max", "argmax"):
            if shape[axis] == 0:
                with pytest.raises(ms.ShapeError):
                    getattr(ms, name)(xd, axis=axis)
            else:
                assert getattr(ms, name)(xd, axis=axis).shape == out_shape
    for name in ("max", "argmin"):
        with pytest.raises(ms.ShapeError):
            getattr(ms, name)(xd)
    assert float(ms.sum(xd).numpy()) == 0.0 and float(ms.prod(xd).numpy()) == 1.0
