"""Compile the sm_100a CUDA sources into the in-tree shared library libhoa.so.

    python -m holonomyawareattention_b200._build [--force] [--verbose] [--debug-bounds]

--debug-bounds builds libhoa_debug.so instead: the same sources with
-DHOA_DEBUG_BOUNDS, in which every kernel of the core path checks the index
ranges of its global accesses and records HOA_ERR_BOUNDS (read through
hoa_debug_bounds) for a range outside its buffer, skipping that access.

The library exposes only the C ABI declared in include/hoa.h (no torch types),
so it can be bound from ctypes, cgo, JNI or C/C++ alike.
"""
from __future__ import annotations

import argparse
import os
import shutil
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
INCLUDE = os.path.join(ROOT, "include")
LIB = os.path.join(PKG, "libhoa.so")
BUILD_DIR = os.path.join(PKG, "_build")
LIB_DEBUG = os.path.join(PKG, "libhoa_debug.so")
BUILD_DIR_DEBUG = os.path.join(PKG, "_build", "debug_bounds")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", "--expt-relaxed-constexpr",
              "-Xptxas", "-warn-spills"]


def nvcc_path() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found: the CUDA toolkit is required to build libhoa.so")


def sources():
    return sorted(os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith(".cu"))


def _deps():
    deps = sources() + [os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith((".cuh", ".h"))]
    deps.append(os.path.join(INCLUDE, "hoa.h"))
    return deps


def up_to_date(lib: str = LIB) -> bool:
    if not os.path.exists(lib):
        return False
    t = os.path.getmtime(lib)
    return all(os.path.getmtime(p) <= t for p in _deps())


def build(force: bool = False, verbose: bool = False, extra_flags=(), debug_bounds: bool = False) -> str:
    lib = LIB_DEBUG if debug_bounds else LIB
    build_dir = BUILD_DIR_DEBUG if debug_bounds else BUILD_DIR
    if debug_bounds:
        extra_flags = (*extra_flags, "-DHOA_DEBUG_BOUNDS")
    if not force and up_to_date(lib):
        return lib
    nvcc = nvcc_path()
    os.makedirs(build_dir, exist_ok=True)
    objs = []

    def compile_one(src):
        obj = os.path.join(build_dir, os.path.basename(src)[:-3] + ".o")
        cmd = [nvcc, *NVCC_FLAGS, *ARCH, *extra_flags, "-I", INCLUDE, "-c", src, "-o", obj]
        if verbose:
            print(" ".join(cmd), flush=True)
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"nvcc failed on {src}:\n{r.stdout}\n{r.stderr}")
        if verbose and (r.stdout or r.stderr):
            print(r.stdout + r.stderr, flush=True)
        return obj

    with ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 1)) as ex:
        objs = list(ex.map(compile_one, sources()))
    tmp = lib + ".tmp"
    cuda_lib = os.path.join(os.path.dirname(os.path.dirname(nvcc)), "lib64")
    cmd = [nvcc, *ARCH, "-shared", "-o", tmp, *objs, "-lcudart", "-L", cuda_lib, "-lcublasLt",
           "-Xlinker", f"-rpath={cuda_lib}"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
    os.replace(tmp, lib)
    return lib


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose", action="store_true")
    ap.add_argument("--ptxas-v", action="store_true", help="print register/smem usage")
    ap.add_argument("--debug-bounds", action="store_true",
                    help="build libhoa_debug.so with the device-side index checks")
    a = ap.parse_args(argv)
    extra = ["-Xptxas", "-v"] if a.ptxas_v else []
    print(build(force=a.force or a.ptxas_v, verbose=a.verbose or a.ptxas_v, extra_flags=extra,
                debug_bounds=a.debug_bounds))


if __name__ == "__main__":
    sys.exit(main())
