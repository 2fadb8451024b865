"""Build recipe for the sm_100a library (libqvl_b200.so, in-tree).

Every .cu under csrc/ is compiled with nvcc for sm_100a only and linked into
one shared library with a pure C ABI (include/qvl_b200.h).  The CUDA runtime
is linked statically so the library has no runtime-version coupling with the
host process (PyTorch, or the reference's C++ host).
"""
from __future__ import annotations

import glob
import os
import shutil
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
LIBDIR = os.path.join(PKG, "lib")
OBJDIR = os.path.join(PKG, "_build")
LIB = os.path.join(LIBDIR, "libqvl_b200.so")
SHIM = os.path.join(LIBDIR, "libqvl_b200_linear_shim.so")
SHIM_SRC = os.path.join(PKG, "host", "linear_shim.cpp")

NVCC = os.environ.get("NVCC", shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc")
CUDA_HOME = os.path.dirname(os.path.dirname(os.path.realpath(NVCC)))
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC,-O2", "--expt-relaxed-constexpr",
         "-I" + os.path.join(ROOT, "include")]


def _stale(obj: str, deps: list[str]) -> bool:
    if not os.path.exists(obj):
        return True
    t = os.path.getmtime(obj)
    return any(os.path.getmtime(d) > t for d in deps)


def build(verbose: bool = False, ptxas_v: bool = False) -> str:
    os.makedirs(LIBDIR, exist_ok=True)
    os.makedirs(OBJDIR, exist_ok=True)
    srcs = sorted(glob.glob(os.path.join(CSRC, "*.cu")))
    headers = glob.glob(os.path.join(CSRC, "*.cuh")) + glob.glob(os.path.join(ROOT, "include", "*.h"))
    objs = []
    jobs = []
    for s in srcs:
        o = os.path.join(OBJDIR, os.path.basename(s) + ".o")
        objs.append(o)
        if _stale(o, [s] + headers):
            cmd = [NVCC, *ARCH, *FLAGS, "-c", s, "-o", o]
            if ptxas_v:
                cmd.insert(1, "-Xptxas=-v")
            jobs.append(cmd)

    def run(cmd):
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0 or verbose or ptxas_v:
            sys.stderr.write(" ".join(cmd) + "\n" + r.stdout + r.stderr)
        if r.returncode != 0:
            raise RuntimeError(f"nvcc failed for {cmd[-3]}")

    with ThreadPoolExecutor(max_workers=min(8, max(1, len(jobs)))) as ex:
        list(ex.map(run, jobs))
    if jobs or not os.path.exists(LIB):
        cmd = [NVCC, *ARCH, "-shared", "-o", LIB, *objs]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError("link failed:\n" + r.stdout + r.stderr)
    # C++ host shim with the reference's linear() signature (links the library)
    if not os.path.exists(SHIM) or os.path.getmtime(SHIM) < max(os.path.getmtime(SHIM_SRC), os.path.getmtime(LIB)):
        cmd = ["g++", "-std=c++17", "-O2", "-fPIC", "-shared", "-o", SHIM, SHIM_SRC,
               "-I" + os.path.join(ROOT, "include"), "-I" + os.path.join(CUDA_HOME, "include"),
               "-L" + LIBDIR, "-lqvl_b200", "-Wl,-rpath,$ORIGIN",
               "-L" + os.path.join(CUDA_HOME, "lib64"), "-lcudart"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError("shim build failed:\n" + r.stdout + r.stderr)
    return LIB


if __name__ == "__main__":
    print(build(verbose="-v" in sys.argv, ptxas_v="--ptxas" in sys.argv))
