"""Build the sampler's C-ABI shared library for sm_100a (in tree).

    python -m flashgen_b200.build          # -> flashgen_b200/lib/libflashgen_sampler.so

The library is plain nvcc output (``-shared``, static CUDA runtime) so that it
has no torch dependency and loads through ctypes, cgo, JNI or pybind11 alike.
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
LIBDIR = os.path.join(HERE, "lib")
LIBNAME = "libflashgen_sampler.so"
LIBPATH = os.path.join(LIBDIR, LIBNAME)
SOURCES = [os.path.join(CSRC, "fg_abi.cu")]
DEPS = SOURCES + [os.path.join(CSRC, f) for f in ("fg_common.cuh", "fg_sample_kernel.cuh", "fg_kernels.cuh")] + [
    os.path.join(ROOT, "include", "flashgen_sampler.h")]

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-lineinfo", "-O3", "-std=c++17",
    "-Xcompiler", "-fPIC", "-shared",
    "-Xptxas", "-v",
]


def nvcc_path() -> str:
    cuda = os.environ.get("CUDA_HOME", "/usr/local/cuda")
    p = os.path.join(cuda, "bin", "nvcc")
    return p if os.path.exists(p) else (shutil.which("nvcc") or "nvcc")


def up_to_date() -> bool:
    if not os.path.exists(LIBPATH):
        return False
    t = os.path.getmtime(LIBPATH)
    return all(os.path.getmtime(d) <= t for d in DEPS if os.path.exists(d))


def build(force: bool = False, verbose: bool = False) -> str:
    if not force and up_to_date():
        return LIBPATH
    os.makedirs(LIBDIR, exist_ok=True)
    tmp = LIBPATH + ".tmp"
    cmd = [nvcc_path(), *NVCC_FLAGS, "-o", tmp, *SOURCES]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError("nvcc failed:\n" + " ".join(cmd) + "\n" + res.stdout + res.stderr)
    if verbose:
        sys.stderr.write(res.stderr)
    os.replace(tmp, LIBPATH)
    return LIBPATH


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose=True))
