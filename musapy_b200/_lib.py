"""ctypes binding of libmusapy_b200.so (the C-ABI declared in include/musapy_b200.h).

torch is imported first so that the library's dynamic CUDA-runtime dependency
resolves to the runtime torch already loaded: one runtime, one error state and
one set of streams in the process. There is no fallback: when the shared
library is missing, importing this module raises.
"""
from __future__ import annotations

import ctypes
import os

import torch  # noqa: F401  (loads the CUDA runtime the library links against)

from . import errors

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "_lib", "libmusapy_b200.so")

c_i64p = ctypes.POINTER(ctypes.c_int64)
c_vp = ctypes.c_void_p

# status codes (csrc/mpb_types.h)
MPB_OK = 0
MPB_ERR_INVALID = 1
MPB_ERR_DTYPE = 2
MPB_ERR_SHAPE = 3
MPB_ERR_SCRATCH = 4
MPB_ERR_CUDA = 5
MPB_ERR_TIMEOUT = 6
MPB_ERR_UNSUPPORTED = 7

# elementwise ops
OPS = {
    "add": 0, "sub": 1, "mul": 2, "div": 3, "pow": 4,
    "eq": 10, "ne": 11, "lt": 12, "gt": 13, "le": 14, "ge": 15,
    "sin": 20, "cos": 21, "exp": 22, "log": 23, "abs": 24, "sign": 25, "neg": 26,
    "clamp": 30, "cast": 31, "fill": 32,
}
# reductions
RED_OPS = {"sum": 0, "prod": 1, "max": 2, "min": 3, "mean": 4, "argmax": 5, "argmin": 6,
           "argmax_rec": 7, "argmin_rec": 8}

# reduction planner kinds (csrc/reduce.h RedKind)
RED_KINDS = {0: "empty", 1: "row_warp", 2: "row_block", 3: "row_split", 4: "col", 5: "col_split", 6: "gen"}


def _load() -> ctypes.CDLL:
    if not os.path.exists(LIB_PATH):
        raise ImportError(
            f"{LIB_PATH} is missing: build it with `python musapy_b200/build.py` "
            "(musapy_b200 has no CPU fallback)"
        )
    L = ctypes.CDLL(LIB_PATH)
    L.mpb_last_error.restype = ctypes.c_char_p
    L.mpb_last_error.argtypes = []
    L.mpb_version.restype = ctypes.c_int
    L.mpb_num_sms.restype = ctypes.c_int
    L.mpb_promote.restype = ctypes.c_int
    L.mpb_promote.argtypes = [ctypes.c_int, ctypes.c_int, ctypes.c_int]
    L.mpb_broadcast_shape.restype = ctypes.c_int
    L.mpb_broadcast_shape.argtypes = [ctypes.c_int, c_i64p, ctypes.c_int, c_i64p, c_i64p]
    L.mpb_broadcast_strides.restype = None
    L.mpb_broadcast_strides.argtypes = [ctypes.c_int, c_i64p, c_i64p, ctypes.c_int, c_i64p, c_i64p]
    L.mpb_collapse.restype = ctypes.c_int
    L.mpb_collapse.argtypes = [ctypes.c_int, c_i64p, ctypes.c_int, c_i64p, c_i64p, c_i64p]
    L.mpb_reduce_plan.restype = ctypes.c_int
    L.mpb_reduce_plan.argtypes = [ctypes.c_int, c_i64p, c_i64p, ctypes.c_int, ctypes.c_uint64, c_i64p, c_i64p, c_i64p]
    L.mpb_reduce_plan_at.restype = ctypes.c_int
    L.mpb_reduce_plan_at.argtypes = [ctypes.c_int, ctypes.c_int, c_i64p, c_i64p, ctypes.c_void_p, ctypes.c_int,
                                     ctypes.c_uint64, c_i64p, c_i64p, c_i64p, ctypes.POINTER(ctypes.c_int)]
    L.mpb_elementwise.restype = ctypes.c_int
    L.mpb_elementwise.argtypes = [
        ctypes.c_int, ctypes.c_int, c_i64p,
        c_vp, ctypes.c_int, c_i64p,
        c_vp, ctypes.c_int, c_i64p,
        c_vp, ctypes.c_int, ctypes.c_int,
        ctypes.c_double, ctypes.c_double, c_vp,
    ]
    L.mpb_reduce_scratch_bytes.restype = ctypes.c_size_t
    L.mpb_reduce_scratch_bytes.argtypes = [
        ctypes.c_int, ctypes.c_int, c_i64p, c_i64p, c_vp, ctypes.c_int, ctypes.c_uint64, ctypes.c_int,
    ]
    L.mpb_reduce.restype = ctypes.c_int
    L.mpb_reduce.argtypes = [
        ctypes.c_int, ctypes.c_int, c_i64p, c_i64p, c_vp, ctypes.c_int, ctypes.c_uint64,
        c_vp, ctypes.c_int, ctypes.c_int, ctypes.c_int, c_vp, ctypes.c_size_t, c_vp,
    ]
    L.mpb_cumsum_scratch_bytes.restype = ctypes.c_size_t
    L.mpb_cumsum_scratch_bytes.argtypes = [
        ctypes.c_int, c_i64p, c_i64p, c_vp, ctypes.c_int, ctypes.c_int, c_vp, ctypes.c_int,
    ]
    L.mpb_cumsum.restype = ctypes.c_int
    L.mpb_cumsum.argtypes = [
        ctypes.c_int, c_i64p, c_i64p, c_vp, ctypes.c_int, ctypes.c_int, c_vp, ctypes.c_int,
        c_vp, ctypes.c_size_t, c_vp,
    ]
    L.mpb_cumsum_status.restype = ctypes.c_int
    L.mpb_cumsum_status.argtypes = [c_vp, c_vp]
    L.mpb_launch_count.restype = ctypes.c_ulonglong
    L.mpb_launch_count.argtypes = []
    L.mpb_shard_arg_combine.restype = ctypes.c_int
    L.mpb_shard_arg_combine.argtypes = [c_vp, ctypes.c_int, c_i64p, ctypes.c_int, ctypes.c_int, c_vp, c_vp, c_vp]
    L.mpb_shard_sum_finalize.restype = ctypes.c_int
    L.mpb_shard_sum_finalize.argtypes = [c_vp, ctypes.c_double, ctypes.c_int, c_vp, c_vp, c_vp]
    L.mpb_arange.restype = ctypes.c_int
    L.mpb_arange.argtypes = [c_vp, ctypes.c_int, ctypes.c_int64, ctypes.c_double, ctypes.c_double, c_vp]
    L.mpb_linspace.restype = ctypes.c_int
    L.mpb_linspace.argtypes = [c_vp, ctypes.c_int, ctypes.c_int64, ctypes.c_double, ctypes.c_double, c_vp]
    L.mpb_eye.restype = ctypes.c_int
    L.mpb_eye.argtypes = [c_vp, ctypes.c_int, ctypes.c_int64, ctypes.c_int64, ctypes.c_int64, c_vp]
    L.mpb_copy_h2d.restype = ctypes.c_int
    L.mpb_copy_h2d.argtypes = [c_vp, c_vp, ctypes.c_size_t, c_vp]
    L.mpb_copy_d2h.restype = ctypes.c_int
    L.mpb_copy_d2h.argtypes = [c_vp, c_vp, ctypes.c_size_t, c_vp]
    L.mpb_peer_buffer_bytes.restype = ctypes.c_size_t
    L.mpb_peer_handle_bytes.restype = ctypes.c_size_t
    L.mpb_peer_alloc.restype = ctypes.c_int
    L.mpb_peer_alloc.argtypes = [ctypes.POINTER(c_vp), c_vp]
    L.mpb_peer_open.restype = ctypes.c_int
    L.mpb_peer_open.argtypes = [c_vp, ctypes.POINTER(c_vp)]
    L.mpb_peer_close.restype = ctypes.c_int
    L.mpb_peer_close.argtypes = [c_vp]
    L.mpb_peer_free.restype = ctypes.c_int
    L.mpb_peer_free.argtypes = [c_vp]
    L.mpb_peer_allgather.restype = ctypes.c_int
    L.mpb_peer_allgather.argtypes = [c_vp, ctypes.c_int, ctypes.POINTER(c_vp), ctypes.c_int, ctypes.c_int,
                                     ctypes.c_uint64, c_vp, c_vp, c_vp]
    L.mpb_ew_set_tma.restype = ctypes.c_int
    L.mpb_ew_set_tma.argtypes = [ctypes.c_int]
    L.mpb_ew_tma_launches.restype = ctypes.c_uint64
    L.mpb_ew_wait_status.restype = ctypes.c_int
    L.mpb_ew_wait_status.argtypes = [ctypes.POINTER(ctypes.c_int)]
    L.mpb_peer_sum_finalize.restype = ctypes.c_int
    L.mpb_peer_sum_finalize.argtypes = [c_vp, ctypes.POINTER(c_vp), ctypes.c_int, ctypes.c_int, ctypes.c_uint64,
                                        ctypes.c_double, ctypes.c_int, c_vp, c_vp, c_vp, c_vp]
    L.mpb_peer_arg_combine.restype = ctypes.c_int
    L.mpb_peer_arg_combine.argtypes = [c_vp, ctypes.POINTER(c_vp), ctypes.c_int, ctypes.c_int, ctypes.c_uint64,
                                       c_i64p, ctypes.c_int, ctypes.c_int, c_vp, c_vp, c_vp, c_vp]
    L.mpb_peer_sum_finalize_emulated.restype = ctypes.c_int
    L.mpb_peer_sum_finalize_emulated.argtypes = [c_vp, ctypes.POINTER(c_vp), ctypes.c_int, ctypes.c_uint64,
                                                 ctypes.c_double, ctypes.c_int, c_vp, c_vp, c_vp, c_vp]
    L.mpb_peer_arg_combine_emulated.restype = ctypes.c_int
    L.mpb_peer_arg_combine_emulated.argtypes = [c_vp, ctypes.POINTER(c_vp), ctypes.c_int, ctypes.c_uint64, c_i64p,
                                                ctypes.c_int, ctypes.c_int, c_vp, c_vp, c_vp, c_vp]
    L.mpb_shard_sum_parts_finalize.restype = ctypes.c_int
    L.mpb_shard_sum_parts_finalize.argtypes = [c_vp, ctypes.c_int, ctypes.c_int, ctypes.c_double, ctypes.c_int,
                                               c_vp, c_vp, c_vp]
    return L


LIB = _load()


def _load_native():
    """The compiled per-op binding (csrc/native_module.cpp). It links
    against the library file loaded above, which the dynamic loader maps
    once: both routes share one library state."""
    import importlib.machinery
    import importlib.util
    import sysconfig

    path = os.path.join(_HERE, "_lib", "_native" + sysconfig.get_config_var("EXT_SUFFIX"))
    if not os.path.exists(path):
        raise ImportError(f"{path} is missing: build it with `python musapy_b200/build.py`")
    loader = importlib.machinery.ExtensionFileLoader("musapy_b200._native", path)
    spec = importlib.util.spec_from_file_location("musapy_b200._native", path, loader=loader)
    mod = importlib.util.module_from_spec(spec)
    loader.exec_module(mod)
    return mod


NATIVE = _load_native()


_I64_TYPES = [ctypes.c_int64 * max(1, n) for n in range(33)]


def i64arr(vals) -> ctypes.Array:
    n = len(vals)
    t = _I64_TYPES[n] if n <= 32 else ctypes.c_int64 * n
    return t(*vals)


def last_error() -> str:
    msg = LIB.mpb_last_error()
    return msg.decode() if msg else ""


def check(rc: int, what: str = "") -> None:
    """Raise the musapy exception matching a non-zero status code."""
    if rc == MPB_OK:
        return
    msg = f"{what}: {last_error()}" if what else last_error()
    if rc == MPB_ERR_DTYPE:
        raise errors.DtypeError(msg)
    if rc in (MPB_ERR_SHAPE,):
        raise errors.ShapeError(msg)
    if rc == MPB_ERR_SCRATCH:
        raise errors.MemoryError(msg)
    if rc == MPB_ERR_TIMEOUT:
        raise errors.KernelError(msg)
    if rc == MPB_ERR_CUDA:
        raise errors.KernelError(msg)
    raise errors.MusapyError(msg)


def launch_count() -> int:
    """Kernels launched by libmusapy_b200 in this process so far."""
    return int(LIB.mpb_launch_count())
