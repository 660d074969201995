"""The parity oracle (and the C++ host logic) against the reference's own
known answers (tests/golden/reference_kats.py). CPU only."""
import numpy as np
import pytest

from tests.golden import reference_kats as K
from tests.golden_util import check_values, host, long_name


@pytest.mark.parametrize("case", K.BINARY, ids=lambda c: c[0])
def test_binary(oracle, case):
    src, op, a, b, exp, kw = case
    ad, bd = kw.get("a_dtype", "f32"), kw.get("b_dtype", "f32")
    x, y = host(a, ad, oracle), host(b, bd, oracle)
    # The reference tests run on the CPU device: JAX promotion (all_gpu=False).
    got = oracle.binary(op, x, y)
    if "out_dtype" in kw:
        assert oracle.NAMES[oracle.code_of(got.dtype)] == long_name(kw["out_dtype"]), src
    check_values(got, exp, kw.get("tol"), src)


@pytest.mark.parametrize("case", K.UNARY, ids=lambda c: c[0] + c[1])
def test_unary(oracle, case):
    src, op, a, exp, kw = case
    got = oracle.unary(op, host(a, kw.get("dtype", "f32"), oracle))
    check_values(got, exp, kw.get("tol"), src)


@pytest.mark.parametrize("case", K.CLAMP, ids=lambda c: c[0])
def test_clamp(oracle, case):
    src, a, lo, hi, exp, kw = case
    check_values(oracle.clamp(host(a, kw.get("dtype", "f32"), oracle), lo, hi), exp, None, src)


@pytest.mark.parametrize("case", K.COMPARE, ids=lambda c: c[0] + c[1])
def test_compare(oracle, case):
    src, op, a, b, exp, kw = case
    got = oracle.compare(op, host(a, kw.get("a_dtype", "f32"), oracle), host(b, kw.get("b_dtype", "f32"), oracle))
    assert got.tolist() == exp, src


@pytest.mark.parametrize("case", K.CAST, ids=lambda c: c[0])
def test_cast(oracle, case):
    src, a, sd, dd, exp = case
    got = oracle.cast(host(a, sd, oracle), oracle.NAMES.index(long_name(dd)))
    check_values(got, exp, None, src)


@pytest.mark.parametrize("case", K.REDUCE, ids=lambda c: c[0] + c[1])
def test_reduce(oracle, case):
    src, op, a, axis, keep, exp, kw = case
    got = oracle.reduce(op, host(a, kw.get("dtype", "f32"), oracle), axis, keep)
    if "out_dtype" in kw:
        assert oracle.NAMES[oracle.code_of(got.dtype)] == long_name(kw["out_dtype"]), src
    check_values(np.asarray(got), exp, kw.get("tol"), src)


@pytest.mark.parametrize("case", K.CUMSUM, ids=lambda c: c[0])
def test_cumsum(oracle, case):
    src, a, axis, exp, kw = case
    got = oracle.cumsum(host(a, kw.get("dtype", "f32"), oracle), axis)
    check_values(got, exp, kw.get("tol"), src)


@pytest.mark.parametrize("case", K.PROMOTE, ids=lambda c: f"{c[0]}+{c[1]}:{c[2]}")
def test_promote_oracle_and_library(oracle, case):
    a, b, gpu, want, line = case
    ca, cb = oracle.NAMES.index(a), oracle.NAMES.index(b)
    assert oracle.NAMES[oracle.promote(ca, cb, gpu)] == want, f"{K.PROMOTE_SRC}:{line}"
    from musapy_b200._lib import LIB

    assert oracle.NAMES[LIB.mpb_promote(ca, cb, 1 if gpu else 0)] == want, f"{K.PROMOTE_SRC}:{line}"


def test_promote_exhaustive_agreement(oracle):
    """The C++ restatement and the oracle's agree on all 15x15x2 pairs."""
    from musapy_b200._lib import LIB

    for a in range(15):
        for b in range(15):
            for g in (0, 1):
                assert LIB.mpb_promote(a, b, g) == oracle.promote(a, b, bool(g)), (a, b, g)


@pytest.mark.parametrize("case", K.BROADCAST_SHAPE, ids=lambda c: str(c[3]))
def test_broadcast_shape(case):
    from musapy_b200._lib import LIB, i64arr

    a, b, want, line = case
    out = i64arr([0] * 8)
    n = LIB.mpb_broadcast_shape(len(a), i64arr(a), len(b), i64arr(b), out)
    if want is None:
        assert n < 0, f"{K.BROADCAST_SRC}:{line}"
    else:
        assert list(out[:n]) == want, f"{K.BROADCAST_SRC}:{line}"


@pytest.mark.parametrize("case", K.BROADCAST_STRIDES, ids=lambda c: str(c[4]))
def test_broadcast_strides(case):
    from musapy_b200._lib import LIB, i64arr

    shape, strides, target, want, line = case
    out = i64arr([0] * max(1, len(target)))
    LIB.mpb_broadcast_strides(len(shape), i64arr(shape), i64arr(strides), len(target), i64arr(target), out)
    assert list(out[: len(target)]) == want, f"{K.BROADCAST_SRC}:{line}"


def _oracle_creation(oracle, kind, args, kw):
    kw = dict(kw)
    if "dtype" in kw:
        kw["dtype"] = oracle.NAMES.index(long_name(kw["dtype"]))
    return getattr(oracle, kind)(*args, **kw)


@pytest.mark.parametrize("case", K.CREATION, ids=lambda c: c[0])
def test_creation(oracle, case):
    src, kind, args, kw, exp, dt, tol = case
    got = _oracle_creation(oracle, kind, args, kw)
    assert oracle.NAMES[oracle.code_of(got.dtype)] == long_name(dt), src
    check_values(got, exp, tol, src)


@pytest.mark.parametrize("case", K.CREATION_ERRORS, ids=lambda c: c[0])
def test_creation_errors(oracle, case):
    src, kind, args = case
    with pytest.raises(ValueError):
        getattr(oracle, kind)(*args)


def _cpu_view(shape, strides):
    import sys

    import torch

    A = sys.modules["musapy_b200.array"].Array
    from musapy_b200 import float32

    return A(torch.empty(16, dtype=torch.uint8), tuple(shape), tuple(strides), 0, float32, 0)


def test_python_broadcast_helpers_match_library():
    """ops.py's per-op broadcast shape/strides against the library's
    restatement (which the reference's broadcast.rs vectors pin), on those
    vectors and on random shapes."""
    import random

    from musapy_b200 import errors, ops
    from musapy_b200._lib import LIB, i64arr

    cases = [(a, b) for a, b, _, _ in K.BROADCAST_SHAPE]
    rnd = random.Random(7)
    for _ in range(400):
        na, nb = rnd.randint(0, 5), rnd.randint(0, 5)
        a = [rnd.choice([1, 1, 2, 3, 5]) for _ in range(na)]
        b = [rnd.choice([1, 1, 2, 3, 5]) for _ in range(nb)]
        cases.append((a, b))
    for a, b in cases:
        out = i64arr([0] * max(len(a), len(b), 1))
        n = LIB.mpb_broadcast_shape(len(a), i64arr(a), len(b), i64arr(b), out)
        va, vb = _cpu_view(a, [3 + i for i in range(len(a))]), _cpu_view(b, [7 * i - 2 for i in range(len(b))])
        if n < 0:
            with pytest.raises(errors.ShapeError):
                ops._broadcast_shape(va, vb)
            continue
        shape = tuple(out[:n])
        assert ops._broadcast_shape(va, vb) == shape, (a, b)
        for v in (va, vb):
            st = i64arr([0] * max(1, len(shape)))
            LIB.mpb_broadcast_strides(v.ndim, i64arr(v.shape), i64arr(v.strides), len(shape), i64arr(shape), st)
            assert list(ops._bstrides(v, shape)) == list(st[: len(shape)]), (v.shape, shape)


@pytest.mark.parametrize("dtype", [np.float32, np.float64, np.int64])
@pytest.mark.parametrize("op", ["max", "min", "argmax", "argmin"])
def test_one_output_extremum_is_thread_count_independent(oracle, dtype, op):
    """The oracle's chunked one-output extremum (several threads) gives the
    sequential loop's exact result: first occurrence on ties, a NaN first
    element decides, later NaNs are skipped, -0.0 and 0.0 compare equal."""
    rng = np.random.default_rng(7)
    n = 1 << 18
    cases = []
    if np.dtype(dtype).kind == "f":
        x = rng.standard_normal(n).astype(dtype)
        x[[5000, 90000, 200000]] = x.max() + 1  # ties across chunks
        x[[7, 100000]] = np.nan
        cases.append(x)
        y = x.copy()
        y[0] = np.nan
        cases.append(y)
        z = np.zeros(n, dtype)
        z[:1000] = -0.0
        z[150000] = 0.0
        cases.append(z)
        cases.append(np.full(n, np.nan, dtype))
    else:
        x = rng.integers(-50, 50, n).astype(dtype)
        x[[3, 70000, 260000]] = 99
        x[[4, 80000]] = -99
        cases.append(x)
    for x in cases:
        for view in (x, x[::-1], x[1::3]):
            try:
                oracle.set_threads(1)
                want = oracle.reduce(op, view, None)
                oracle.set_threads(8)
                got = oracle.reduce(op, view, None)
            finally:
                oracle.set_threads(1)
            assert np.asarray(got).tobytes() == np.asarray(want).tobytes(), (op, dtype)
