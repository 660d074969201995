"""Comparison helpers for parity tests (bit-exact, ulp, condition-aware)."""
import numpy as np


def bits(x: np.ndarray) -> np.ndarray:
    x = np.ascontiguousarray(x)
    return x.view({1: np.uint8, 2: np.uint16, 4: np.uint32, 8: np.uint64, 16: np.uint64}[x.itemsize])


def _is_float_like(d: np.dtype) -> bool:
    return d.kind in "fc" or d.name == "bfloat16"


def assert_bits_equal(got: np.ndarray, want: np.ndarray, what: str = "") -> None:
    """Bit-exact equality; every NaN compares equal to every NaN (NaN
    payloads are not compared)."""
    got, want = np.asarray(got), np.asarray(want)
    assert got.shape == want.shape, f"{what}: shape {got.shape} != {want.shape}"
    assert got.dtype == want.dtype, f"{what}: dtype {got.dtype} != {want.dtype}"
    if _is_float_like(got.dtype):
        g, w = got.reshape(-1), want.reshape(-1)
        if got.dtype.kind == "c":
            g = g.view(got.real.dtype)
            w = w.view(want.real.dtype)
        both_nan = np.isnan(g.astype(np.float64)) & np.isnan(w.astype(np.float64))
        diff = (bits(g) != bits(w)) & ~both_nan
    else:
        diff = (got != want).reshape(-1)
    n = int(diff.sum())
    if n:
        i = int(np.flatnonzero(diff)[0])
        raise AssertionError(f"{what}: {n} of {diff.size} elements differ; first at {i}: "
                             f"got {got.reshape(-1)[i if got.dtype.kind != 'c' else i // 2]!r} "
                             f"want {want.reshape(-1)[i if want.dtype.kind != 'c' else i // 2]!r}")


def ulp_diff(got: np.ndarray, want: np.ndarray) -> np.ndarray:
    """|difference| in units in the last place of the float type (NaN==NaN,
    inf==inf count as 0)."""
    got, want = np.asarray(got), np.asarray(want)
    if got.dtype == np.float32:
        it, sign = np.int64, np.int64(1) << 31
        gi = got.view(np.int32).astype(np.int64)
        wi = want.view(np.int32).astype(np.int64)
    elif got.dtype == np.float64:
        gi = got.view(np.int64).astype(object)
        wi = want.view(np.int64).astype(object)
        sign = 1 << 63
        it = object
    else:  # 16-bit: float16 or bfloat16 bit patterns
        gi = got.view(np.int16).astype(np.int64)
        wi = want.view(np.int16).astype(np.int64)
        sign = 1 << 15
        it = np.int64

    def ordered(v):
        # map sign-magnitude to a monotone integer line
        if it is object:
            return np.array([(-(int(x) & ((1 << 63) - 1))) if int(x) < 0 else int(x) for x in v.reshape(-1)],
                            dtype=object).reshape(v.shape)
        neg = v < 0
        out = v.copy()
        out[neg] = -(v[neg] & (sign - 1))
        return out

    d = np.abs(ordered(gi) - ordered(wi))
    g64 = got.astype(np.float64) if got.dtype.itemsize != 2 else got.astype(np.float32).astype(np.float64)
    w64 = want.astype(np.float64) if want.dtype.itemsize != 2 else want.astype(np.float32).astype(np.float64)
    same = (np.isnan(g64) & np.isnan(w64)) | (g64 == w64)
    d = np.where(same, 0, d)
    return d.astype(np.float64)


def assert_ulp(got, want, max_ulp: float, what: str = "") -> None:
    d = ulp_diff(np.asarray(got), np.asarray(want))
    m = float(d.max()) if d.size else 0.0
    assert m <= max_ulp, f"{what}: max ulp difference {m} > {max_ulp}"


def assert_sum_close(got, want, absx_sum, rtol: float, what: str = "", truth=None) -> None:
    """Condition-aware check for sums: |got - want| <= rtol * sum|x|.

    The reference CPU path accumulates sequentially in the input float type,
    which drifts from the exact sum on long inputs. When `truth` (an f64
    evaluation) is given, a value is also accepted if it is at least as close
    to the truth as the CPU value is (plus the same bound)."""
    got = np.asarray(got, dtype=np.float64)
    want = np.asarray(want, dtype=np.float64)
    bound = rtol * np.asarray(absx_sum, dtype=np.float64) + 1e-300
    err = np.abs(got - want)
    ok = (err <= bound) | (np.isnan(got) & np.isnan(want)) | (got == want)
    if truth is not None:
        truth = np.asarray(truth, dtype=np.float64)
        ok |= np.abs(got - truth) <= np.abs(want - truth) + bound
    bad = ~ok
    if bad.any():
        i = np.flatnonzero(bad.reshape(-1))[0]
        raise AssertionError(f"{what}: {int(bad.sum())} values outside rtol={rtol}*sum|x|; "
                             f"first: got {got.reshape(-1)[i]!r} want {want.reshape(-1)[i]!r} "
                             f"bound {np.broadcast_to(bound, got.shape).reshape(-1)[i]!r}")


def bit_mismatches(got: np.ndarray, want: np.ndarray, chunk: int = 1 << 24) -> int:
    """Number of elements whose bits differ between two same-shaped arrays of
    one dtype, counted in chunks so that multi-GiB outputs need no large
    temporaries. Two NaNs compare equal whatever their payloads."""
    got, want = np.asarray(got), np.asarray(want)
    assert got.shape == want.shape and got.dtype == want.dtype, (got.shape, want.shape, got.dtype, want.dtype)
    g, w = got.reshape(-1), want.reshape(-1)
    if got.dtype.kind == "c":
        g, w = g.view(got.real.dtype), w.view(want.real.dtype)
    floaty = _is_float_like(g.dtype)
    bad = 0
    for i in range(0, g.size, chunk):
        gc, wc = g[i:i + chunk], w[i:i + chunk]
        if floaty:
            diff = bits(gc) != bits(wc)
            if diff.any():
                both_nan = np.isnan(gc.astype(np.float32)) & np.isnan(wc.astype(np.float32))
                bad += int((diff & ~both_nan).sum())
        else:
            bad += int((gc != wc).sum())
    return bad


def max_ulp_chunked(got: np.ndarray, want: np.ndarray, chunk: int = 1 << 22) -> float:
    """max ulp_diff over two large float arrays, chunk by chunk."""
    g, w = np.asarray(got).reshape(-1), np.asarray(want).reshape(-1)
    m = 0.0
    for i in range(0, g.size, chunk):
        d = ulp_diff(g[i:i + chunk], w[i:i + chunk])
        if d.size:
            m = max(m, float(d.max()))
    return m
