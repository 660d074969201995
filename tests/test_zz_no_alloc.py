"""mpb_reduce_noalloc against mpb_reduce, called through the C-ABI.

mpb_reduce_noalloc serves callers that cannot allocate device memory (an
application that owns the whole device budget through its own pool, or a
latency-critical loop where cudaMalloc / cudaFree must not run because they
can synchronise the device): it takes no scratch argument and uses an
array built into the library instead. This file checks, on two calls in a
row, that its results match the scratch-taking entry point within the
tolerances the other parity tests use, and that oversized requests are
refused. pytest collects this file last, so a run that stops at the first
failure has already run every other test; it also passes on its own in a
fresh process.
"""
import ctypes

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

F32, F64, I64 = 10, 11, 4
SUM, MAX, MEAN, ARGMAX = 0, 2, 4, 5
MPB_ERR_SCRATCH = 4


def _lib():
    from musapy_b200._lib import LIB, c_i64p, c_vp

    f = LIB.mpb_reduce_noalloc
    f.restype = ctypes.c_int
    f.argtypes = [ctypes.c_int, ctypes.c_int, c_i64p, c_i64p, c_vp, ctypes.c_int, ctypes.c_uint64,
                  c_vp, ctypes.c_int, ctypes.c_int, ctypes.c_int, c_vp]
    return LIB


def _i64(v):
    return (ctypes.c_int64 * max(1, len(v)))(*v)


def _reduce_both(lib, x: torch.Tensor, op: int, mask: int, out_dtype: int, out_shape):
    """One call of mpb_reduce (torch-allocated scratch) and two calls in a row
    of mpb_reduce_noalloc on the same input; returns the three outputs."""
    shape, strides = _i64(list(x.shape)), _i64(list(x.stride()))
    stream = torch.cuda.current_stream().cuda_stream
    td = {F32: torch.float32, F64: torch.float64, I64: torch.int64}[out_dtype]
    need = lib.mpb_reduce_scratch_bytes(op, x.dim(), shape, strides, x.data_ptr(), F32, mask, F32)
    assert need > 0, "the case must use the split plan (the one that needs scratch)"
    scratch = torch.empty(need, dtype=torch.uint8, device=x.device)
    ref = torch.empty(out_shape, dtype=td, device=x.device)
    rc = lib.mpb_reduce(op, x.dim(), shape, strides, x.data_ptr(), F32, mask, ref.data_ptr(), out_dtype, F32, 1,
                        scratch.data_ptr(), need, stream)
    assert rc == 0, lib.mpb_last_error()
    outs = []
    for _ in range(2):
        o = torch.full(out_shape, -7, dtype=td, device=x.device)
        rc = lib.mpb_reduce_noalloc(op, x.dim(), shape, strides, x.data_ptr(), F32, mask, o.data_ptr(), out_dtype,
                                    F32, 1, stream)
        assert rc == 0, lib.mpb_last_error()
        outs.append(o)
    torch.cuda.synchronize()
    return ref.cpu().numpy(), [o.cpu().numpy() for o in outs]


@pytest.mark.parametrize("shape,mask,out_shape", [
    ((1 << 24) + 3, 1, ()),      # full reduction: row split across CTAs
    ((1024, 100), 1, (100,)),    # few columns, long axis: column split
])
def test_noalloc_matches_scratch_entry_point_twice(shape, mask, out_shape):
    lib = _lib()
    rng = np.random.default_rng(99)
    host = rng.standard_normal(shape).astype(np.float32)
    x = torch.from_numpy(host).cuda()
    absx = np.abs(host.astype(np.float64))
    absx_sum = absx.sum() if mask == 1 and host.ndim == 1 else absx.sum(axis=0)
    for op, out_dtype in [(SUM, F32), (MEAN, F32), (MAX, F32), (ARGMAX, I64)]:
        ref, (first, second) = _reduce_both(lib, x, op, mask, out_dtype, out_shape)
        for got in (first, second):
            if op in (SUM, MEAN):
                bound = 1e-5 * (absx_sum / (host.shape[0] if op == MEAN else 1))
                assert np.all(np.abs(got.astype(np.float64) - ref.astype(np.float64)) <= bound), (op, got, ref)
            else:
                assert np.array_equal(got, ref), (op, got, ref)


def test_noalloc_rejects_requests_beyond_its_scratch():
    lib = _lib()
    # a column reduction split so widely that its partials exceed the built-in array
    x = torch.zeros((4096, 300), dtype=torch.float32, device="cuda")
    shape, strides = _i64([4096, 300]), _i64([300, 1])
    need = lib.mpb_reduce_scratch_bytes(SUM, 2, shape, strides, x.data_ptr(), F32, 1, F32)
    assert need > 256 * 1024
    out = torch.empty(300, dtype=torch.float32, device="cuda")
    rc = lib.mpb_reduce_noalloc(SUM, 2, shape, strides, x.data_ptr(), F32, 1, out.data_ptr(), F32, F32, 1,
                                torch.cuda.current_stream().cuda_stream)
    assert rc == MPB_ERR_SCRATCH
    assert b"built-in scratch" in lib.mpb_last_error()
