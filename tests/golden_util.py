"""Helpers shared by the golden-KAT test files."""
import numpy as np

SHORT = {"f16": "float16", "f32": "float32", "f64": "float64", "bf16": "bfloat16", "c64": "complex64",
         "c128": "complex128", "i8": "int8", "i16": "int16", "i32": "int32", "i64": "int64", "u8": "uint8",
         "b1": "bool", "bool": "bool"}


def long_name(d: str) -> str:
    return SHORT.get(d, d)


def host(values, dtype: str, oracle):
    """Literal values as a numpy array of `dtype`, converted with the
    oracle's (musapy's) cast rules."""
    code = oracle.NAMES.index(long_name(dtype))
    nd = oracle.np_of(code)
    arr = np.asarray(values)
    if nd.kind == "c":
        return arr.astype(nd)
    if arr.dtype.kind == "c":
        raise TypeError("complex literal for a real dtype")
    if code in (oracle.F64, oracle.I64):
        return arr.astype(nd)
    src = np.asarray(arr, dtype=np.float64) if arr.dtype.kind == "f" else arr.astype(np.int64)
    return oracle.cast(src, code)


def check_values(got: np.ndarray, expect, tol, what: str) -> None:
    exp = np.asarray(expect)
    assert got.shape == exp.shape, f"{what}: shape {got.shape} != {exp.shape}"
    g = got.astype(np.complex128 if got.dtype.kind == "c" else np.float64)
    e = exp.astype(np.complex128 if exp.dtype.kind == "c" else np.float64)
    if tol is None:
        assert np.array_equal(g, e), f"{what}: got {got.tolist()} want {exp.tolist()}"
    else:
        assert np.allclose(g, e, rtol=0, atol=tol), f"{what}: got {got.tolist()} want {exp.tolist()} (tol {tol})"
