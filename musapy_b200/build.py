"""Build libmusapy_b200.so in-tree for sm_100a.

Every ``.cu`` under ``csrc/`` is compiled to an object by ``nvcc`` (in
parallel) and linked into ``musapy_b200/_lib/libmusapy_b200.so``; then
``csrc/native_module.cpp``, the CPython binding of the per-op calls, is
compiled by ``g++`` against it into ``musapy_b200/_lib/_native*.so``. Objects are
rebuilt only when a source or header is newer than the object, so repeated
calls are cheap. The CUDA runtime is linked dynamically, so the library
shares one runtime (and one error state) with the host process.

Usage:  python musapy_b200/build.py [--force] [--jobs N]

Run it as a script (it needs only the standard library): importing the
package loads the library, which may be missing or stale before a build.
"""
from __future__ import annotations

import argparse
import concurrent.futures as cf
import glob
import os
import shutil
import subprocess
import sys
import sysconfig

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
INCLUDE = os.path.join(os.path.dirname(HERE), "include")
BUILD = os.path.join(HERE, "_build")
LIBDIR = os.path.join(HERE, "_lib")
LIBNAME = "libmusapy_b200.so"
CUDA_HOME = os.environ.get("CUDA_HOME", "/usr/local/cuda")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ARCH + [
    "-O3",
    "-lineinfo",
    "-std=c++17",
    "--expt-relaxed-constexpr",
    "-Xcompiler",
    "-fPIC,-O2",
    "-cudart",
    "shared",
    "-I",
    CSRC,
    "-I",
    INCLUDE,
]


def nvcc() -> str:
    exe = shutil.which("nvcc") or os.path.join(CUDA_HOME, "bin", "nvcc")
    if not os.path.exists(exe):
        raise RuntimeError("nvcc not found (CUDA toolkit required to build musapy_b200)")
    return exe


def lib_path() -> str:
    return os.path.join(LIBDIR, LIBNAME)


def _headers() -> list[str]:
    return (glob.glob(os.path.join(CSRC, "*.h")) + glob.glob(os.path.join(CSRC, "*.cuh"))
            + glob.glob(os.path.join(INCLUDE, "*.h")))


def _stale(src: str, obj: str, newest_header: float) -> bool:
    if not os.path.exists(obj):
        return True
    t = os.path.getmtime(obj)
    return os.path.getmtime(src) > t or newest_header > t


def _compile(src: str, obj: str, extra: list[str]) -> tuple[str, int, str]:
    cmd = [nvcc()] + NVCC_FLAGS + extra + ["-c", src, "-o", obj]
    p = subprocess.run(cmd, capture_output=True, text=True)
    return src, p.returncode, p.stdout + p.stderr


def build(force: bool = False, jobs: int | None = None, extra: list[str] | None = None, verbose: bool = False) -> str:
    """Compile (when stale) and link the library; return its path."""
    os.makedirs(BUILD, exist_ok=True)
    os.makedirs(LIBDIR, exist_ok=True)
    extra = extra or []
    srcs = sorted(glob.glob(os.path.join(CSRC, "*.cu")))
    newest_header = max([os.path.getmtime(h) for h in _headers()] + [0.0])
    todo = []
    objs = []
    for s in srcs:
        o = os.path.join(BUILD, os.path.basename(s)[:-3] + ".o")
        objs.append(o)
        if force or _stale(s, o, newest_header):
            todo.append((s, o))
    if todo:
        jobs = jobs or min(len(todo), os.cpu_count() or 4)
        with cf.ThreadPoolExecutor(max_workers=jobs) as ex:
            futs = [ex.submit(_compile, s, o, extra) for s, o in todo]
            errors = []
            for f in cf.as_completed(futs):
                src, rc, out = f.result()
                if rc != 0:
                    errors.append(f"--- {os.path.basename(src)} ---\n{out}")
                elif verbose and out.strip():
                    print(out, file=sys.stderr)
            if errors:
                raise RuntimeError("nvcc failed:\n" + "\n".join(errors))
    lib = lib_path()
    if todo or not os.path.exists(lib) or any(os.path.getmtime(o) > os.path.getmtime(lib) for o in objs):
        cmd = [nvcc()] + ARCH + ["-shared", "-cudart", "shared", "-o", lib] + objs + [
            "-Xlinker",
            f"-rpath={CUDA_HOME}/lib64",
            "-Xlinker",
            f"-soname={LIBNAME}",
        ]
        p = subprocess.run(cmd, capture_output=True, text=True)
        if p.returncode != 0:
            raise RuntimeError("link failed:\n" + p.stdout + p.stderr)
    build_native(force=force)
    return lib


def native_path() -> str:
    return os.path.join(LIBDIR, "_native" + sysconfig.get_config_var("EXT_SUFFIX"))


def build_native(force: bool = False) -> str:
    """The CPython binding of the per-op entry points (csrc/native_module.cpp),
    linked against the library beside it."""
    src = os.path.join(CSRC, "native_module.cpp")
    out = native_path()
    deps = [src, lib_path(), os.path.join(INCLUDE, "musapy_b200.h")]
    if not force and os.path.exists(out) and all(os.path.getmtime(d) <= os.path.getmtime(out) for d in deps):
        return out
    cxx = shutil.which("g++") or shutil.which("c++")
    if cxx is None:
        raise RuntimeError("g++ not found (needed for the Python binding of musapy_b200)")
    cmd = [cxx, "-O2", "-std=c++17", "-shared", "-fPIC", "-fvisibility=hidden", "-I", sysconfig.get_paths()["include"],
           "-I", INCLUDE, src, "-o", out, "-L", LIBDIR, "-l:" + LIBNAME, "-Wl,-rpath,$ORIGIN"]
    p = subprocess.run(cmd, capture_output=True, text=True)
    if p.returncode != 0:
        raise RuntimeError("Python binding build failed:\n" + p.stdout + p.stderr)
    return out


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--jobs", type=int, default=None)
    ap.add_argument("--ptxas-v", action="store_true", help="print register/spill usage")
    args = ap.parse_args()
    extra = ["-Xptxas", "-v"] if args.ptxas_v else []
    print(build(force=args.force, jobs=args.jobs, extra=extra, verbose=args.ptxas_v))


if __name__ == "__main__":
    main()
