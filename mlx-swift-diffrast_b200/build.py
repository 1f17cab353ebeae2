"""Build libdiffrast.so (the C-ABI library) for sm_100a with nvcc.

    python mlx-swift-diffrast_b200/build.py [--force] [--jobs N]

Objects go to mlx-swift-diffrast_b200/_build/, the shared library to
mlx-swift-diffrast_b200/diffrast/libdiffrast.so (in-tree, next to the Python
binding that loads it).  A file is recompiled when it or any header changed.
"""
from __future__ import annotations

import argparse
import concurrent.futures as cf
import glob
import os
import shutil
import subprocess
import sys

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
BUILD = os.path.join(PKG, "_build")
INCLUDE = os.path.join(ROOT, "include")
LIB = os.path.join(PKG, "diffrast", "libdiffrast.so")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
# -fmad=false keeps a kernel's float arithmetic identical to the CPU oracle's
# unfused operations (coverage-critical code also uses explicit _rn
# intrinsics, so it does not depend on this flag).  The translation units in
# FMA_SOURCES hold only gradient kernels, whose outputs are compared with the
# oracle within tolerances, not bit for bit: they are built with contraction.
NVCC_FLAGS = ARCH + [
    "-O3", "-lineinfo", "-std=c++17", "--expt-relaxed-constexpr",
    "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
    "-I" + INCLUDE, "-I" + CSRC,
]
FMA_SOURCES = {"raster_bwd.cu", "texture_bwd.cu"}


def fmad_flag(src: str) -> str:
    return "-fmad=true" if os.path.basename(src) in FMA_SOURCES else "-fmad=false"


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found")


def _headers():
    return glob.glob(os.path.join(CSRC, "*.cuh")) + glob.glob(os.path.join(INCLUDE, "*.h"))


def _stale(src: str, obj: str) -> bool:
    if not os.path.exists(obj):
        return True
    t = os.path.getmtime(obj)
    return any(os.path.getmtime(p) > t for p in [src, *_headers(), __file__])


def compile_one(src: str, force: bool, extra=()) -> str:
    obj = os.path.join(BUILD, os.path.basename(src).replace(".cu", ".o"))
    if force or _stale(src, obj):
        cmd = [nvcc(), *NVCC_FLAGS, fmad_flag(src), *extra, "-c", src, "-o", obj]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"nvcc failed for {src}:\n{r.stdout}\n{r.stderr}")
        if r.stderr.strip():
            sys.stderr.write(r.stderr)
    return obj


def build(force: bool = False, jobs: int = 0, verbose_ptxas: bool = False) -> str:
    os.makedirs(BUILD, exist_ok=True)
    srcs = sorted(glob.glob(os.path.join(CSRC, "*.cu")))
    extra = ["-Xptxas", "-v"] if verbose_ptxas else []
    with cf.ThreadPoolExecutor(max_workers=jobs or min(8, os.cpu_count() or 1)) as ex:
        objs = list(ex.map(lambda s: compile_one(s, force or verbose_ptxas, extra), srcs))
    if force or not os.path.exists(LIB) or any(os.path.getmtime(o) > os.path.getmtime(LIB) for o in objs):
        cmd = [nvcc(), *ARCH, "-shared", "-o", LIB, *objs]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
    return LIB


DRIVER_SRC = os.path.join(PKG, "cdriver", "dr_check.cpp")
DRIVER = os.path.join(PKG, "cdriver", "dr_check")


def build_driver(force: bool = False) -> str:
    """The C++ caller of the ABI (cdriver/dr_check.cpp): host compiler only,
    linked against libdiffrast.so and the CUDA runtime."""
    lib = build()
    if not force and os.path.exists(DRIVER) and os.path.getmtime(DRIVER) >= max(
            os.path.getmtime(DRIVER_SRC), os.path.getmtime(lib), *[os.path.getmtime(h) for h in _headers()]):
        return DRIVER
    cuda = os.path.dirname(os.path.dirname(nvcc()))
    cmd = [os.environ.get("CXX", "g++"), "-O2", "-std=c++17", "-I" + INCLUDE, "-I" + os.path.join(cuda, "include"),
           DRIVER_SRC, "-o", DRIVER, "-L" + os.path.dirname(lib), "-ldiffrast", "-L" + os.path.join(cuda, "lib64"),
           "-lcudart", "-Wl,-rpath," + os.path.dirname(lib), "-Wl,-rpath,$ORIGIN/../diffrast"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"driver build failed:\n{r.stdout}\n{r.stderr}")
    return DRIVER


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--jobs", type=int, default=0)
    ap.add_argument("--ptxas-v", action="store_true", help="print register/smem usage")
    a = ap.parse_args()
    print(build(a.force, a.jobs, a.ptxas_v))
    print(build_driver(a.force))
