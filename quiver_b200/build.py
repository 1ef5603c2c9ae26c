"""Builds the in-tree libraries with nvcc and g++.

``quiver_b200/libquiver_b200.so``: every source under ``quiver_b200/csrc`` (CUDA and the host C++
of the C ABI, compiled as CUDA for sm_100a so they share headers) becomes one object.

``quiver_b200/libquiver.so``: the quiver C++ API (``include/quiver/*.h``) implemented in
``quiver_b200/cpp`` over the C ABI, linked against libquiver_b200.so (found next to it at run time).

Objects are rebuilt only when a source or header is newer. Run as ``python -m quiver_b200.build``
or call :func:`build`.
"""
from __future__ import annotations

import concurrent.futures as cf
import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
BUILD = os.path.join(HERE, "_build")
LIB = os.path.join(HERE, "libquiver_b200.so")
CPP = os.path.join(HERE, "cpp")
CPP_LIB = os.path.join(HERE, "libquiver.so")
CXX_FLAGS = ["-std=c++20", "-O2", "-fPIC", "-Wall", "-Wextra", "-I", os.path.join(ROOT, "include"),
             "-I", CPP]

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", "-Xcompiler", "-O3",
              "--expt-relaxed-constexpr", "-I", os.path.join(ROOT, "include"), "-I", CSRC]


def _nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found: the CUDA toolkit is required to build quiver_b200")


def _sources() -> list[str]:
    return sorted(os.path.join(CSRC, f) for f in os.listdir(CSRC)
                  if f.endswith((".cu", ".cc")))


def _headers() -> list[str]:
    hdrs = [os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith((".h", ".cuh"))]
    return hdrs + [os.path.join(ROOT, "include", "qv_gpu.h")]


def _cpp_headers() -> list[str]:
    hdrs = [os.path.join(CPP, f) for f in os.listdir(CPP) if f.endswith(".h")]
    inc = os.path.join(ROOT, "include")
    for dirpath, _, files in os.walk(inc):
        hdrs += [os.path.join(dirpath, f) for f in files if f.endswith(".h")]
    return hdrs


def _cxx() -> str:
    for cand in (os.environ.get("CXX"), shutil.which("g++"), "/usr/bin/g++"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("g++ not found: a C++20 compiler is required to build the quiver C++ API")


def _stale(target: str, deps: list[str]) -> bool:
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps)


def build(verbose: bool = False, jobs: int = 0) -> str:
    """Compiles stale objects and relinks the library; returns its path."""
    nvcc = _nvcc()
    os.makedirs(BUILD, exist_ok=True)
    headers = _headers()
    srcs = _sources()
    objs = []
    todo = []
    for src in srcs:
        obj = os.path.join(BUILD, os.path.basename(src) + ".o")
        objs.append(obj)
        if _stale(obj, [src] + headers):
            cmd = [nvcc, *ARCH, *NVCC_FLAGS, "-x", "cu", "-c", src, "-o", obj]
            todo.append(cmd)

    def run(cmd):
        if verbose:
            print(" ".join(cmd), flush=True)
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"nvcc failed for {cmd[-3]}:\n{r.stdout}\n{r.stderr}")
        if verbose and (r.stdout or r.stderr):
            print(r.stdout + r.stderr, flush=True)

    if todo:
        with cf.ThreadPoolExecutor(max_workers=jobs or min(len(todo), os.cpu_count() or 4)) as ex:
            list(ex.map(run, todo))
    if todo or _stale(LIB, objs):
        cmd = [nvcc, *ARCH, "-shared", "-o", LIB, *objs, "-lcudart", "-lpthread"]
        run(cmd)
    build_cpp(verbose)
    return LIB


def build_cpp(verbose: bool = False) -> str:
    """Compiles the quiver C++ API into libquiver.so (needs libquiver_b200.so built first)."""
    cxx = _cxx()
    srcs = sorted(os.path.join(CPP, f) for f in os.listdir(CPP) if f.endswith(".cc"))
    if not _stale(CPP_LIB, srcs + _cpp_headers() + [LIB]):
        return CPP_LIB
    cmd = [cxx, *CXX_FLAGS, "-shared", "-o", CPP_LIB, *srcs, "-L", HERE, "-lquiver_b200",
           "-Wl,-rpath,$ORIGIN", "-lpthread"]
    if verbose:
        print(" ".join(cmd), flush=True)
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"g++ failed for the C++ API:\n{r.stdout}\n{r.stderr}")
    return CPP_LIB


if __name__ == "__main__":
    print(build(verbose="-v" in sys.argv))
