"""The reference's own known answers (tests/golden/reference_kats.py) through
the ms.* API on the GPU, plus creation-op parity against the oracle.

The reference tests run on musapy's CPU device; on the GPU the result dtype
of a mixed-precision binary op follows the GPU promotion rule (dtype.rs
`all_gpu`), so dtypes are checked against that rule and values against the
reference's expected numbers with the reference test's tolerance.
"""
import ctypes

import numpy as np
import pytest

from tests.golden import reference_kats as K
from tests.golden_util import check_values, host, long_name
from tests.helpers import assert_bits_equal

pytestmark = pytest.mark.gpu


def dev(ms, x):
    return ms.from_numpy(np.asarray(x), device="cuda:0")


@pytest.mark.parametrize("case", K.BINARY, ids=lambda c: c[0] + c[1])
def test_binary(ms, oracle, case):
    src, op, a, b, exp, kw = case
    x, y = host(a, kw.get("a_dtype", "f32"), oracle), host(b, kw.get("b_dtype", "f32"), oracle)
    got = getattr(ms, op)(dev(ms, x), dev(ms, y)).numpy()
    want_dt = oracle.promote(oracle.code_of(x.dtype), oracle.code_of(y.dtype), True)
    assert oracle.code_of(got.dtype) == want_dt, src
    check_values(got, exp, kw.get("tol"), src)


@pytest.mark.parametrize("case", K.UNARY, ids=lambda c: c[0] + c[1])
def test_unary(ms, oracle, case):
    src, op, a, exp, kw = case
    got = getattr(ms, op)(dev(ms, host(a, kw.get("dtype", "f32"), oracle))).numpy()
    check_values(got, exp, kw.get("tol"), src)


@pytest.mark.parametrize("case", K.CLAMP, ids=lambda c: c[0])
def test_clamp(ms, oracle, case):
    src, a, lo, hi, exp, kw = case
    got = ms.clamp(dev(ms, host(a, kw.get("dtype", "f32"), oracle)), lo, hi).numpy()
    check_values(got, exp, None, src)


@pytest.mark.parametrize("case", K.COMPARE, ids=lambda c: c[0] + c[1])
def test_compare(ms, oracle, case):
    src, op, a, b, exp, kw = case
    x, y = host(a, kw.get("a_dtype", "f32"), oracle), host(b, kw.get("b_dtype", "f32"), oracle)
    got = getattr(ms, op)(dev(ms, x), dev(ms, y)).numpy()
    assert got.tolist() == exp, src


@pytest.mark.parametrize("case", K.CAST, ids=lambda c: c[0])
def test_cast(ms, oracle, case):
    src, a, sd, dd, exp = case
    got = dev(ms, host(a, sd, oracle)).astype(dd).numpy()
    assert oracle.NAMES[oracle.code_of(got.dtype)] == long_name(dd), src
    check_values(got, exp, None, src)


@pytest.mark.parametrize("case", K.REDUCE, ids=lambda c: c[0] + c[1])
def test_reduce(ms, oracle, case):
    src, op, a, axis, keep, exp, kw = case
    got = getattr(ms, op)(dev(ms, host(a, kw.get("dtype", "f32"), oracle)), axis=axis, keepdims=keep).numpy()
    if "out_dtype" in kw:
        assert oracle.NAMES[oracle.code_of(got.dtype)] == long_name(kw["out_dtype"]), src
    check_values(np.asarray(got), exp, kw.get("tol"), src)


@pytest.mark.parametrize("case", K.CUMSUM, ids=lambda c: c[0])
def test_cumsum(ms, oracle, case):
    src, a, axis, exp, kw = case
    got = ms.cumsum(dev(ms, host(a, kw.get("dtype", "f32"), oracle)), axis=axis).numpy()
    check_values(got, exp, kw.get("tol"), src)


# ---------------------------------------------------------------- creation
@pytest.mark.parametrize("case", K.CREATION, ids=lambda c: c[0])
def test_creation_kat(ms, oracle, case):
    src, kind, args, kw, exp, dt, tol = case
    got = getattr(ms, kind)(*args, **kw).numpy()
    assert oracle.NAMES[oracle.code_of(got.dtype)] == long_name(dt), src
    check_values(got, exp, tol, src)


@pytest.mark.parametrize("case", K.CREATION_ERRORS, ids=lambda c: c[0])
def test_creation_errors(ms, case):
    src, kind, args = case
    with pytest.raises(ms.ShapeError):
        getattr(ms, kind)(*args)


CREATE_DTYPES = ["f32", "f64", "i64", "i32", "i16", "u8", "f16", "bf16", "bool", "c64"]


@pytest.mark.parametrize("dt", CREATE_DTYPES)
def test_arange_linspace_parity(ms, oracle, dt):
    """Bit-exact against the CPU restatement over lengths that exercise the
    16-byte packs and the scalar tail, negative and fractional steps, values
    past the integer types' range (saturation) and past f32's 2^24."""
    code = oracle.NAMES.index(long_name(dt))
    for args in [(0, 1), (0, 7), (3, 4099, 1), (-2.5, 1e5, 0.37), (1e9, -1e9, -123456.789), (0, 1 << 20, 3),
                 (16777215, 16777300)]:
        got = ms.arange(*args, dtype=dt).numpy()
        want = oracle.arange(*args, dtype=code)
        assert_bits_equal(got, want, f"arange{args} {dt}")
    for start, stop, num in [(0.0, 1.0, 50), (1.0, -1.0, 3), (-3e5, 7e6, (1 << 20) + 3), (2.0, 8.0, 1), (0, 1, 0)]:
        got = ms.linspace(start, stop, num, dtype=dt).numpy()
        assert_bits_equal(got, oracle.linspace(start, stop, num, dtype=code), f"linspace {start},{stop},{num} {dt}")


@pytest.mark.parametrize("dt", CREATE_DTYPES)
def test_eye_parity(ms, oracle, dt):
    code = oracle.NAMES.index(long_name(dt))
    for n, m, k in [(1, None, 0), (3, 5, 2), (5, 3, -2), (4, 4, 9), (4, 4, -9), (257, 130, 0), (100, 1000, -37),
                    (2048, 2048, 1)]:
        got = ms.eye(n, m, k, dtype=dt).numpy()
        assert_bits_equal(got, oracle.eye(n, m, k, dtype=code), f"eye {n},{m},{k} {dt}")


def test_arange_unaligned_output(ms, oracle):
    """Through the C-ABI into a buffer that starts 4 bytes past a 16-byte
    boundary: the scalar path, same values."""
    import torch

    from musapy_b200._lib import LIB

    buf = torch.zeros(1001, dtype=torch.float32, device="cuda")
    view = buf[1:]
    rc = LIB.mpb_arange(ctypes.c_void_p(view.data_ptr()), oracle.F32, 1000, -3.0, 0.1,
                        ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert rc == 0
    got = view.cpu().numpy()
    assert_bits_equal(got, oracle.arange(-3.0, -3.0 + 1000 * 0.1 - 0.05, 0.1, dtype=oracle.F32)[:1000], "unaligned")
    assert buf[0].item() == 0.0
