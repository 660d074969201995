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
