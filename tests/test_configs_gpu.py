"""The benchmark's full-size workloads on one GPU, every output element
compared with the oracle.

Workloads (seeded numpy PCG64 inputs, built by bench.config_inputs and
bench.gen_rows):
  * int64 (8192, 8192) read through its transpose + a float64 row, and the
    float32 chain exp(sin(x)) -> clamp(-0.5, 0.5) on 2^28 elements (seed 2);
  * float32 (64, 4096, 4096) reductions over axes 2, 0 and (0, 2), argmax
    over axis 1 and cumsum along the last axis (seed 1);
  * f32 <-> bf16 casts, f16 pow and comparisons on 2^30 elements, complex64
    mul on 2^27 (seed 4);
  * the float32 (65536, 32768) broadcast add and full reductions of the
    sharded workload, here on one GPU (seed 5).

Every output is copied back (in blocks where it is large) and compared with
the oracle run over the same inputs with all host threads: bit-exact for
integer, bool, cast, IEEE add/mul, clamp, max and argmax; within 2 ulp for
sin/exp/pow; sums, means and cumsums within rtol * sum|x| (1e-5 for f32) of
the oracle or at least as close to an f64 truth as the oracle is. Each test
reports the number of elements compared in the terminal summary.
"""
import numpy as np
import pytest

import bench
from tests.helpers import assert_sum_close, bit_mismatches, max_ulp_chunked

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module", autouse=True)
def oracle_all_threads(oracle):
    oracle.set_threads(oracle.max_threads())
    yield
    oracle.set_threads(1)


@pytest.fixture(scope="module")
def c2():
    return bench.config_inputs("C2")


@pytest.fixture(scope="module")
def c3():
    return bench.config_inputs("C3")["x"]


@pytest.fixture(scope="module")
def c4():
    return bench.config_inputs("C4")


def _exact(got, want, what, compared):
    n = bit_mismatches(got, want)
    assert n == 0, f"{what}: {n} of {np.asarray(want).size} elements differ from the oracle"
    compared(what, np.asarray(want).size)


def test_config2_transposed_int64_plus_f64_row(ms, oracle, c2, compared):
    A, row = c2["A"], c2["row"]
    out = ms.add(ms.transpose(ms.from_numpy(A)), ms.from_numpy(row))
    assert out.dtype == ms.float64 and out.shape == (8192, 8192)
    _exact(out.numpy(), oracle.binary("add", A.T, row), "int64^T + f64 row", compared)


def test_config2_chain(ms, oracle, c2, compared):
    x = c2["x"]
    xd = ms.from_numpy(x)
    s = ms.sin(xd)
    e = ms.exp(s)
    c = ms.clamp(e, -0.5, 0.5)
    sh = s.numpy()
    u = max_ulp_chunked(sh, oracle.unary("sin", x))
    assert u <= 2, f"sin: max {u} ulp from the oracle"
    compared(f"sin within 2 ulp (max {u:g})", x.size)
    eh = e.numpy()
    u = max_ulp_chunked(eh, oracle.unary("exp", sh))
    assert u <= 2, f"exp: max {u} ulp from the oracle"
    compared(f"exp within 2 ulp (max {u:g})", x.size)
    del sh
    _exact(c.numpy(), oracle.clamp(eh, -0.5, 0.5), "clamp", compared)


def _truths(xt, dims):
    """f64 sum and sum|x| over `dims` of a device tensor (torch, on the GPU):
    the exact-sum reference and the scale of the sum tolerance."""
    import torch

    s = torch.sum(xt, dim=dims, dtype=torch.float64).cpu().numpy()
    a = torch.sum(xt.abs(), dim=dims, dtype=torch.float64).cpu().numpy()
    return s, a


def test_config3_reductions_every_output(ms, oracle, c3, compared):
    x = c3
    xd = ms.from_numpy(x)
    xt = xd.torch()
    for axis, dims in ((2, (2,)), (0, (0,)), ((0, 2), (0, 2))):
        n = 1
        for d in dims:
            n *= x.shape[d]
        truth, absx = _truths(xt, dims)
        for op in ("sum", "mean", "max"):
            got = getattr(ms, op)(xd, axis=axis).numpy()
            want = oracle.reduce(op, x, axis)
            what = f"{op} axis={axis}"
            if op == "max" or axis == 0:
                # max in any order, and a single strided axis summed in the
                # CPU path's own order: bit-exact
                _exact(got, want, what, compared)
            else:
                scale = n if op == "mean" else 1
                assert_sum_close(got, want, absx / scale, 1e-5, what, truth=truth / scale)
                compared(what + " within 1e-5*sum|x|", want.size)
    am = ms.argmax(xd, axis=1).numpy()
    _exact(am, oracle.reduce("argmax", x, 1), "argmax axis=1", compared)


def test_config3_cumsum_last_axis_every_element(ms, oracle, c3, compared):
    x = c3
    cs = ms.cumsum(ms.from_numpy(x), axis=-1)
    got = cs.numpy()
    for p in range(x.shape[0]):
        plane = x[p]
        assert_sum_close(got[p], oracle.cumsum(plane, -1), oracle.cumsum(np.abs(plane).astype(np.float64), -1),
                         1e-5, f"cumsum plane {p}", truth=oracle.cumsum(plane.astype(np.float64), -1))
    compared("cumsum within 1e-5*cumsum|x|", got.size)


def test_config3_cumsum_flattened_every_element(ms, oracle, c3, compared):
    """cumsum with axis=None over all 2^30 elements: one decoupled look-back
    scan (262,144 tiles), against the oracle's sequential f32 running sum;
    the f64 truth and the sum|x| scale are running sums in float64."""
    x = c3.reshape(-1)
    ms.ops.set_scan_status_check(True)
    try:
        got = ms.cumsum(ms.from_numpy(c3)).numpy()
    finally:
        ms.ops.set_scan_status_check(False)
    want = oracle.cumsum(x, 0)
    carry, carry_abs = 0.0, 0.0
    step = 1 << 24
    for i in range(0, x.size, step):
        ch = x[i:i + step].astype(np.float64)
        truth = np.cumsum(ch) + carry
        absx = np.cumsum(np.abs(ch)) + carry_abs
        assert_sum_close(got[i:i + step], want[i:i + step], absx, 1e-5, f"cumsum(axis=None) at {i}", truth=truth)
        carry, carry_abs = truth[-1], absx[-1]
    compared("cumsum(axis=None) within 1e-5*cumsum|x|", x.size)


def test_config4_bf16_round_trip(ms, oracle, c4, compared):
    x = c4["x"]
    xd = ms.from_numpy(x)
    xb = xd.astype("bf16")
    back = xb.astype("f32")
    want_b = oracle.cast(x, oracle.BF16)
    _exact(xb.numpy(), want_b, "f32 -> bf16", compared)
    del xd
    _exact(back.numpy(), oracle.cast(want_b, oracle.F32), "bf16 -> f32", compared)
    # idempotence over the whole array: bf16 -> f32 -> bf16 is exact
    assert ms.sum(ms.ne(back.astype("bf16"), xb)).item() == 0


def test_config4_f16_pow_and_compare(ms, oracle, c4, compared):
    a, b = c4["a"], c4["b"]
    ad, bd = ms.from_numpy(a), ms.from_numpy(b)
    p = ms.pow(ad, bd)
    u = max_ulp_chunked(p.numpy(), oracle.binary("pow", a, b))
    assert u <= 2, f"f16 pow: max {u} ulp from the oracle"
    compared(f"f16 pow within 2 ulp (max {u:g})", a.size)
    del p
    lt, eq = ms.lt(ad, bd), ms.eq(ad, bd)
    _exact(lt.numpy(), oracle.compare("lt", a, b), "f16 lt", compared)
    _exact(eq.numpy(), oracle.compare("eq", a, b), "f16 eq", compared)


def test_config4_complex64_mul(ms, oracle, c4, compared):
    z1, z2 = c4["z1"], c4["z2"]
    z = ms.mul(ms.from_numpy(z1), ms.from_numpy(z2))
    _exact(z.numpy(), oracle.binary("mul", z1, z2), "c64 mul", compared)


# ------------------------------------------------------------ config 5
BLOCK = 2048  # rows per host block: 256 MiB of float32


@pytest.fixture(scope="module")
def c5(ms):
    """The sharded workload's whole matrix on one GPU (2^31 f32, 8 GiB),
    uploaded block by block, and its row vector."""
    import torch

    rows, cols = bench.ROWS, bench.COLS
    x = ms.empty((rows, cols), "f32")
    host = torch.empty((BLOCK, cols), dtype=torch.float32, pin_memory=True)
    xt = x.torch()
    for r0 in range(0, rows, BLOCK):
        bench.gen_rows(r0, r0 + BLOCK, cols, out=host.numpy())
        xt[r0:r0 + BLOCK].copy_(host)
    torch.cuda.synchronize()
    return x, bench.gen_row_vector(rows, cols)


def test_config5_broadcast_add_every_element(ms, oracle, c5, compared):
    """y = x + row over all 2^31 elements, copied back in 256 MiB row blocks
    and compared bit for bit with the oracle's add of the same rows."""
    import torch

    x, row = c5
    rows, cols = x.shape
    y = ms.add(x, ms.from_numpy(row))
    yt = y.torch()
    got = torch.empty((BLOCK, cols), dtype=torch.float32, pin_memory=True)
    host = np.empty((BLOCK, cols), np.float32)
    bad = 0
    for r0 in range(0, rows, BLOCK):
        got.copy_(yt[r0:r0 + BLOCK])
        bench.gen_rows(r0, r0 + BLOCK, cols, out=host)
        bad += bit_mismatches(got.numpy(), oracle.binary("add", host, row))
    assert bad == 0, f"broadcast add: {bad} elements differ from the oracle"
    compared("broadcast add (65536, 32768) + (32768,)", rows * cols)
    # and the row sums of y, every one
    rs = ms.sum(y, axis=1).numpy()
    yt64 = yt.double()
    want_truth = yt64.sum(dim=1).cpu().numpy()
    absy = yt64.abs_().sum(dim=1).cpu().numpy()
    del yt64
    for r0 in range(0, rows, BLOCK):
        got.copy_(yt[r0:r0 + BLOCK])
        assert_sum_close(rs[r0:r0 + BLOCK], oracle.reduce("sum", got.numpy(), 1), absy[r0:r0 + BLOCK], 1e-5,
                         "sum(axis=1)", truth=want_truth[r0:r0 + BLOCK])
    compared("sum(axis=1) within 1e-5*sum|y|", rows)


def test_config5_full_size_reductions(ms, oracle, c5):
    """Full argmax/argmin with the winner planted near the last index,
    2^31 - 12345 (no 32-bit wrap anywhere in the split kernels' index
    arithmetic), a later tie (the first occurrence wins), and the full
    sum/mean against the oracle's f64 truth (the oracle's own f32 mean stalls
    its divisor at 2^24, so the truth decides)."""
    import torch

    x, _ = c5
    rows, cols = x.shape
    t = x.torch()
    big = (1 << 31) - 12345
    r, c = divmod(big, cols)
    planted = [(r, c, 5.0), (r, c + 100, 5.0), (r - 7, 11, -5.0)]
    saved = [float(t[i, j]) for i, j, _ in planted]
    try:
        for i, j, v in planted:
            t[i, j] = v
        assert ms.argmax(x).item() == big
        assert ms.argmin(x).item() == (r - 7) * cols + 11
        s, m = ms.sum(x).item(), ms.mean(x).item()
        td = t.double()
        truth = td.sum().item()
        absum = td.abs_().sum().item()
        del td
        assert abs(s - truth) <= 1e-5 * absum
        assert abs(m - truth / t.numel()) <= 1e-5 * absum / t.numel()
    finally:
        for (i, j, _), v in zip(planted, saved):
            t[i, j] = v
        torch.cuda.synchronize()
