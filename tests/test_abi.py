"""The C-ABI library loads on a machine without a GPU and exports every
function the public headers declare (no compute calls here)."""
import ctypes
import os
import re

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADERS = [os.path.join(ROOT, "include", h) for h in sorted(os.listdir(os.path.join(ROOT, "include")))
           if h.endswith(".h")]


def declared_functions():
    names = set()
    for h in HEADERS:
        text = open(h).read()
        text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
        text = re.sub(r"//[^\n]*", "", text)
        for m in re.finditer(r"\b((?:mpb|musapy)_[a-z0-9_]+)\s*\(", text):
            names.add(m.group(1))
    return sorted(names)


def test_headers_declare_entry_points():
    names = declared_functions()
    assert "mpb_elementwise" in names and "mpb_reduce" in names and "mpb_cumsum" in names


def test_library_exports_every_declared_symbol():
    from musapy_b200._lib import LIB_PATH

    lib = ctypes.CDLL(LIB_PATH)
    missing = [n for n in declared_functions() if not hasattr(lib, n)]
    assert not missing, f"declared but not exported: {missing[:20]}"


def test_version_and_promote_without_gpu():
    from musapy_b200._lib import LIB

    assert LIB.mpb_version() >= 1
    assert LIB.mpb_promote(4, 11, 0) == 11  # int64 + float64 -> float64


def test_native_binding_shares_the_library_state():
    """The compiled per-op binding calls the same loaded library as the
    ctypes route: an error it raises is visible through mpb_last_error."""
    from musapy_b200._lib import NATIVE, last_error

    assert {"elementwise", "reduce", "reduce_scratch_bytes"} <= set(dir(NATIVE))
    rc = NATIVE.elementwise(999, (4, 4), 16, 0, (4, 1), 32, 0, (4, 1), 48, 0, 0, 0.0, 0.0, 0)
    assert rc != 0 and "unknown op 999" in last_error()


def test_native_binding_validates_arguments():
    from musapy_b200._lib import NATIVE

    with pytest.raises(TypeError):
        NATIVE.elementwise(0, (4,))
    with pytest.raises(ValueError):
        NATIVE.elementwise(0, (4, 4), 16, 0, (1,), 32, 0, (4, 1), 48, 0, 0, 0.0, 0.0, 0)
    with pytest.raises(ValueError):
        NATIVE.elementwise(0, (1,) * 33, 16, 0, None, None, 0, None, 48, 0, 0, 0.0, 0.0, 0)
    with pytest.raises(TypeError):
        NATIVE.reduce_scratch_bytes(0, (4,), (1,), 16, 0, "x", 0)


def test_native_broadcast_binding_validates_shapes():
    from musapy_b200._lib import NATIVE

    with pytest.raises(ValueError):  # (3,) does not broadcast to (4,)
        NATIVE.elementwise_bc(0, (4,), 16, 10, (3,), (1,), 32, 10, (4,), (1,), 48, 10, 10, 0.0, 0.0, 0)
    with pytest.raises(ValueError):  # more dims than the output
        NATIVE.elementwise_bc(0, (4,), 16, 10, (1, 4), (4, 1), 32, 10, (4,), (1,), 48, 10, 10, 0.0, 0.0, 0)
    with pytest.raises(ValueError):  # strides and shape differ
        NATIVE.elementwise_bc(0, (4,), 16, 10, (4,), (1, 1), 32, 10, (4,), (1,), 48, 10, 10, 0.0, 0.0, 0)


def _plan_at(op, shape, strides, addr, dt, mask):
    from musapy_b200._lib import LIB

    n = len(shape)
    M, L, S = ctypes.c_int64(), ctypes.c_int64(), ctypes.c_int64()
    v = ctypes.c_int()
    kind = LIB.mpb_reduce_plan_at(op, n, (ctypes.c_int64 * n)(*shape), (ctypes.c_int64 * n)(*strides),
                                  ctypes.c_void_p(addr), dt, mask, ctypes.byref(M), ctypes.byref(L),
                                  ctypes.byref(S), ctypes.byref(v))
    return kind, M.value, L.value, S.value, v.value


# dtype codes of mpb_types.h: i64 4, f16 9, f32 10, f64 11, bf16 12, c64 13, c128 14;
# ops: 0 sum, 2 max, 5 argmax, 6 argmin; kinds: 4 column, 5 column split
@pytest.mark.parametrize("op,shape,strides,addr,dt,mask,want", [
    # argmax over axis 1 of (64, 4096, 4096) f32: 2 outputs per thread (8-byte
    # loads for arg reductions), one partial wave, 16 MiB in flight - no split
    (5, (64, 4096, 4096), (1 << 24, 4096, 1), 1 << 20, 10, 0b010, (4, 262144, 4096, 1, 2)),
    (6, (64, 4096, 4096), (1 << 24, 4096, 1), (1 << 20) + 8, 10, 0b010, (4, 262144, 4096, 1, 2)),
    # half of it (32 planes): 8 MiB in flight would leave the grid
    # latency-bound, so it is split
    (5, (32, 4096, 4096), (1 << 24, 4096, 1), 1 << 20, 10, 0b010, (5, 131072, 4096, None, 2)),
    # aligned to 4 bytes only: one per thread, split against the tail wave
    (5, (64, 4096, 4096), (1 << 24, 4096, 1), (1 << 20) + 4, 10, 0b010, (5, 262144, 4096, None, 1)),
    # sum / max over axis 0 of (64, 4096, 4096): 16-byte loads, many waves, no split
    (0, (64, 4096, 4096), (1 << 24, 4096, 1), 1 << 20, 10, 0b001, (4, 1 << 24, 64, 1, 4)),
    (2, (64, 4096, 4096), (1 << 24, 4096, 1), 1 << 20, 10, 0b001, (4, 1 << 24, 64, 1, 4)),
    # the same input aligned to 8 bytes only: 2 per thread
    (0, (64, 4096, 4096), (1 << 24, 4096, 1), (1 << 20) + 8, 10, 0b001, (4, 1 << 24, 64, 1, 2)),
    (0, (256, 256), (256, 1), 0, 11, 0b01, (None, 256, 256, None, 2)),   # f64: 16-byte pairs
    (5, (256, 256), (256, 1), 0, 11, 0b01, (None, 256, 256, None, 2)),   # f64 argmax too
    (0, (256, 256), (256, 1), 0, 9, 0b01, (None, 256, 256, None, 8)),    # f16: 8 per 16-byte load
    (5, (256, 256), (256, 1), 0, 9, 0b01, (None, 256, 256, None, 4)),    # f16 argmax: 8-byte loads
    (0, (256, 256), (256, 1), 0, 12, 0b01, (None, 256, 256, None, 8)),   # bf16
    (0, (256, 256), (256, 1), 0, 13, 0b01, (None, 256, 256, None, 2)),   # c64
    (0, (256, 256), (256, 1), 0, 14, 0b01, (None, 256, 256, None, 1)),   # c128: one 16-byte element
    (0, (256, 256), (256, 1), 0, 4, 0b01, (None, 256, 256, None, 2)),    # int64
    (0, (1025, 5), (5, 1), 0, 10, 0b01, (None, 5, 1025, None, 1)),       # inner extent 5
    (0, (1025, 6), (6, 1), 0, 10, 0b01, (None, 6, 1025, None, 2)),       # inner extent 6
    (0, (256, 256), (-256, 1), 0, 10, 0b01, (None, 256, 256, None, 4)),  # flipped reduced axis
    # few outputs and a long reduced dim: little in flight, so split
    (0, (100000, 1024), (1024, 1), 0, 10, 0b01, (5, 1024, 100000, None, 4)),
    (5, (100000, 1024), (1024, 1), 0, 10, 0b01, (5, 1024, 100000, None, 2)),
])
def test_reduce_plan_column_vector_width(op, shape, strides, addr, dt, mask, want):
    """The column planner's outputs per thread (from the op, alignment and
    extents) and its split choice, on the host without a GPU."""
    got = _plan_at(op, shape, strides, addr, dt, mask)
    for g, w, name in zip(got, want, ("kind", "M", "L", "splits", "outputs per thread")):
        if w is not None:
            assert g == w, f"{name}: {got} vs {want}"
    if want[0] == 5:
        assert got[3] > 1
