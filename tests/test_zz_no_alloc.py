"""mpb_reduce_noalloc against mpb_reduce and the oracle, called through the C-ABI.

mpb_reduce_noalloc serves callers that cannot allocate device memory (an
application that owns the whole device budget through its own pool, or a
latency-critical loop where cudaMalloc / cudaFree must not run because they
can synchronise the device): it takes no scratch argument and uses an array
built into the library instead. This file checks, on two calls in a row,
that its results are bit-identical to the scratch-taking entry point's when
both run the same plan, that they match the oracle (bit-exact for max and
argmax/argmin, within the sum tolerance of the other parity tests for sums and
means), that a reduction whose split would not fit in the built-in array still
runs, and that repeated calls leave the device's free memory unchanged.
pytest collects this file last, so a run that stops at the first failure has
already run every other test; it also passes on its own in a fresh process.
"""
import ctypes

import numpy as np
import pytest
import torch

from tests.helpers import assert_bits_equal, assert_sum_close

pytestmark = pytest.mark.gpu

F32, F64, I64 = 10, 11, 4
SUM, MAX, MEAN, ARGMAX, ARGMIN = 0, 2, 4, 5, 6
NAMES = {SUM: "sum", MAX: "max", MEAN: "mean", ARGMAX: "argmax", ARGMIN: "argmin"}
SPLIT_KINDS = (3, 5)  # row_split, col_split
SCRATCH_LIMIT = 256 * 1024


def _lib():
    from musapy_b200._lib import LIB, c_i64p, c_vp

    f = LIB.mpb_reduce_noalloc
    f.restype = ctypes.c_int
    f.argtypes = [ctypes.c_int, ctypes.c_int, c_i64p, c_i64p, c_vp, ctypes.c_int, ctypes.c_uint64,
                  c_vp, ctypes.c_int, ctypes.c_int, ctypes.c_int, c_vp]
    return LIB


def _i64(v):
    return (ctypes.c_int64 * max(1, len(v)))(*v)


def _plan_kind(lib, x: torch.Tensor, dt: int, mask: int) -> int:
    m, n, s = ctypes.c_int64(), ctypes.c_int64(), ctypes.c_int64()
    kind = lib.mpb_reduce_plan(x.dim(), _i64(list(x.shape)), _i64(list(x.stride())), dt, mask,
                               ctypes.byref(m), ctypes.byref(n), ctypes.byref(s))
    assert kind >= 0, lib.mpb_last_error()
    return int(kind)


def _out_dtype(op: int, dt: int) -> int:
    return I64 if op in (ARGMAX, ARGMIN) else dt


def _torch_dtype(code: int):
    return {F32: torch.float32, F64: torch.float64, I64: torch.int64}[code]


def _noalloc_twice(lib, x: torch.Tensor, dt: int, op: int, mask: int, out_shape):
    """Two calls in a row of mpb_reduce_noalloc on the same input (each into
    an output pre-filled with garbage); returns both results on the host."""
    shape, strides = _i64(list(x.shape)), _i64(list(x.stride()))
    stream = torch.cuda.current_stream().cuda_stream
    od = _out_dtype(op, dt)
    outs = []
    for _ in range(2):
        o = torch.full(out_shape, -7, dtype=_torch_dtype(od), device=x.device)
        rc = lib.mpb_reduce_noalloc(op, x.dim(), shape, strides, x.data_ptr(), dt, mask, o.data_ptr(), od, dt, 1,
                                    stream)
        assert rc == 0, lib.mpb_last_error()
        outs.append(o)
    torch.cuda.synchronize()
    return [o.cpu().numpy() for o in outs]


def _scratch_entry_point(lib, x: torch.Tensor, dt: int, op: int, mask: int, out_shape):
    """One call of mpb_reduce with torch-allocated scratch (the regular path)."""
    shape, strides = _i64(list(x.shape)), _i64(list(x.stride()))
    od = _out_dtype(op, dt)
    need = lib.mpb_reduce_scratch_bytes(op, x.dim(), shape, strides, x.data_ptr(), dt, mask, dt)
    scratch = torch.empty(max(1, need), dtype=torch.uint8, device=x.device)
    ref = torch.empty(out_shape, dtype=_torch_dtype(od), device=x.device)
    rc = lib.mpb_reduce(op, x.dim(), shape, strides, x.data_ptr(), dt, mask, ref.data_ptr(), od, dt, 1,
                        scratch.data_ptr(), need, torch.cuda.current_stream().cuda_stream)
    assert rc == 0, lib.mpb_last_error()
    torch.cuda.synchronize()
    return ref.cpu().numpy(), need


def _check_against_oracle(oracle, host: np.ndarray, axis, op: int, got: np.ndarray, what: str) -> None:
    want = oracle.reduce(NAMES[op], host, axis)
    if op in (SUM, MEAN):
        absx = np.abs(host.astype(np.float64))
        absx_sum = absx.sum() if axis is None else absx.sum(axis=axis)
        n = host.size if axis is None else host.shape[axis]
        truth = oracle.reduce(NAMES[op], host.astype(np.float64), axis)
        assert_sum_close(got, want, absx_sum / (n if op == MEAN else 1), 1e-5 if host.dtype == np.float32 else 1e-12,
                         what, truth=truth)
    else:
        assert_bits_equal(np.asarray(got), np.asarray(want), what)


CASES = [
    # (shape, dtype, mask, out_shape, ops)
    (((1 << 24) + 3,), np.float32, 1, (), (SUM, MEAN, MAX, ARGMAX)),        # full reduction: row split
    ((1024, 100), np.float32, 1, (100,), (SUM, MEAN, MAX, ARGMAX)),         # long axis, few columns: column split
    (((1 << 22) + 5,), np.float64, 1, (), (ARGMIN, SUM)),                   # f64 argmin: 16-byte partials
    ((4096, 300), np.float32, 1, (300,), (SUM, MAX, ARGMIN)),               # split capped to fit the array
]


@pytest.mark.parametrize("shape,dtype,mask,out_shape,ops", CASES)
def test_noalloc_matches_scratch_entry_point_and_oracle_twice(oracle, shape, dtype, mask, out_shape, ops):
    lib = _lib()
    rng = np.random.default_rng(99)
    host = rng.standard_normal(shape).astype(dtype)
    dt = F32 if dtype == np.float32 else F64
    x = torch.from_numpy(host).cuda()
    assert _plan_kind(lib, x, dt, mask) in SPLIT_KINDS, "the case must use a split plan (the one that needs scratch)"
    axis = None if len(shape) == 1 else 0
    for op in ops:
        ref, need = _scratch_entry_point(lib, x, dt, op, mask, out_shape)
        first, second = _noalloc_twice(lib, x, dt, op, mask, out_shape)
        for k, got in enumerate((first, second)):
            what = f"{NAMES[op]} {shape} {np.dtype(dtype).name} call {k + 1}"
            if need <= SCRATCH_LIMIT:  # same plan as mpb_reduce: the same bits
                assert_bits_equal(np.asarray(got), np.asarray(ref), what + " vs mpb_reduce")
            _check_against_oracle(oracle, host, axis, op, got, what + " vs oracle")


def test_noalloc_runs_reductions_too_wide_to_split_in_its_array(oracle):
    """More than 16384 outputs: no split fits in the built-in array, so the
    reduction runs unsplit (one thread walks each column in index order, the
    CPU path's summation order: bit-exact for the sum too)."""
    lib = _lib()
    rng = np.random.default_rng(7)
    host = rng.standard_normal((512, 20000)).astype(np.float32)
    x = torch.from_numpy(host).cuda()
    for op in (SUM, MAX, ARGMAX):
        first, second = _noalloc_twice(lib, x, F32, op, 1, (20000,))
        for got in (first, second):
            assert_bits_equal(got, oracle.reduce(NAMES[op], host, 0), f"{NAMES[op]} (512, 20000) axis 0")


def test_noalloc_leaves_free_device_memory_unchanged():
    """Fifty calls on the split path after a first one (which loads the
    library's module on the device) change the device's free memory by
    nothing: the entry point allocates nothing."""
    lib = _lib()
    x = torch.randn((1 << 24) + 3, device="cuda")
    out = torch.empty((), dtype=torch.int64, device="cuda")
    shape, strides = _i64([x.numel()]), _i64([1])
    stream = torch.cuda.current_stream().cuda_stream

    def call():
        rc = lib.mpb_reduce_noalloc(ARGMAX, 1, shape, strides, x.data_ptr(), F32, 1, out.data_ptr(), I64, F32, 1,
                                    stream)
        assert rc == 0, lib.mpb_last_error()

    call()
    torch.cuda.synchronize()
    free0, _ = torch.cuda.mem_get_info()
    for _ in range(50):
        call()
    torch.cuda.synchronize()
    free1, _ = torch.cuda.mem_get_info()
    assert free1 == free0
    assert int(out.item()) == int(torch.argmax(x).item())
