"""In-tree build of libactcomp.so (sm_100a) with nvcc.

``python triton-kernel-test_b200/actcomp/build.py`` (this file run on its own:
importing the ``actcomp`` package loads the library it builds) compiles every
``csrc/*.cu`` into ``actcomp/libactcomp.so`` next to this file.  The library
links the CUDA runtime statically and takes the driver's tensor-map encoder
through ``cudaGetDriverEntryPoint``, so it loads on a machine without a GPU
(the CPU test suite checks its exported symbols) and needs no libcuda at link
time.
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys
import tempfile

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
CSRC = os.path.join(ROOT, "csrc")
LIB = os.path.join(PKG, "libactcomp.so")
# the bounds-checked build (-DACT_BOUNDS_CHECK): device-side index checks that
# record a bit in the device error word instead of trapping; tests only
LIB_BC = os.path.join(PKG, "libactcomp_bc.so")

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-lineinfo", "-std=c++17", "-rdc=true",
    "--fmad=false",               # keep every a*b+c a separately rounded mul and add (oracle parity)
    "-Xcompiler", "-fPIC",
    "--expt-relaxed-constexpr",
    "-Xptxas", "-warn-spills",
]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", shutil.which("nvcc")):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found: the CUDA toolkit is required to build libactcomp")


def sources() -> list[str]:
    return sorted(os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith(".cu"))


def _deps() -> list[str]:
    hdr = [os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith((".cuh", ".h"))]
    inc = os.path.join(os.path.dirname(ROOT), "include", "actcomp.h")
    return sources() + hdr + ([inc] if os.path.exists(inc) else [])


def stale(lib: str = LIB) -> bool:
    if not os.path.exists(lib):
        return True
    t = os.path.getmtime(lib)
    return any(os.path.getmtime(p) > t for p in _deps())


def build(force: bool = False, verbose: bool = False, jobs: int | None = None, bounds_check: bool = False) -> str:
    """Compile (if stale) and return the path of libactcomp.so (libactcomp_bc.so
    with bounds_check)."""
    lib = LIB_BC if bounds_check else LIB
    if not force and not stale(lib):
        return lib
    exe = nvcc()
    flags = NVCC_FLAGS + (["-DACT_BOUNDS_CHECK"] if bounds_check else [])
    tmp = tempfile.mkdtemp(prefix="actcomp_build_")
    try:
        objs = []
        procs = []
        for src in sources():
            obj = os.path.join(tmp, os.path.basename(src) + ".o")
            cmd = [exe, *flags, "-c", src, "-o", obj]
            if verbose:
                print(" ".join(cmd), flush=True)
            procs.append((src, subprocess.Popen(cmd, stdout=subprocess.PIPE, stderr=subprocess.STDOUT, text=True)))
            objs.append(obj)
        failed = []
        for src, p in procs:
            out, _ = p.communicate()
            if out.strip() and (verbose or p.returncode):
                print(out, file=sys.stderr)
            if p.returncode:
                failed.append(src)
        if failed:
            raise RuntimeError(f"nvcc failed for {failed}")
        out_tmp = lib + ".tmp"
        cmd = [exe, "-gencode", "arch=compute_100a,code=sm_100a", "-shared", "-Xcompiler", "-fPIC", "-o", out_tmp,
               *objs, "-cudart", "static"]
        subprocess.run(cmd, check=True)
        os.replace(out_tmp, lib)
    finally:
        shutil.rmtree(tmp, ignore_errors=True)
    return lib


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose="-v" in sys.argv, bounds_check="--bounds-check" in sys.argv))
