"""Build the sampler's C-ABI shared library for sm_100a (in tree).

    python -m flashgen_b200.build          # -> flashgen_b200/lib/libflashgen_sampler.so
                                           #    flashgen_b200/_C*.so (PyBind11 binding)

The library is plain nvcc output (``-shared``, static CUDA runtime) so that it
has no torch dependency and loads through ctypes, cgo, JNI or pybind11 alike.
Each kernel lives in its own translation unit; the units compile in parallel
to objects under ``flashgen_b200/lib/obj`` and link into the one library.
"""
from __future__ import annotations

import glob
import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
LIBDIR = os.path.join(HERE, "lib")
OBJDIR = os.path.join(LIBDIR, "obj")
LIBNAME = "libflashgen_sampler.so"
LIBPATH = os.path.join(LIBDIR, LIBNAME)
SOURCES = [os.path.join(CSRC, f) for f in ("fg_abi.cu", "fg_host.cu", "fg_cluster.cu", "fg_stream.cu")]
HEADERS = sorted(glob.glob(os.path.join(CSRC, "*.cuh")) + glob.glob(os.path.join(CSRC, "*.h"))) + [
    os.path.join(ROOT, "include", "flashgen_sampler.h")]
DEPS = SOURCES + HEADERS

BINDINGS = os.path.join(CSRC, "bindings", "fg_bindings.cpp")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ARCH + ["-lineinfo", "-O3", "-std=c++17", "-Xcompiler", "-fPIC", "-Xptxas", "-v"]


def nvcc_path() -> str:
    cuda = os.environ.get("CUDA_HOME", "/usr/local/cuda")
    p = os.path.join(cuda, "bin", "nvcc")
    return p if os.path.exists(p) else (shutil.which("nvcc") or "nvcc")


def up_to_date() -> bool:
    if not os.path.exists(LIBPATH):
        return False
    t = os.path.getmtime(LIBPATH)
    return all(os.path.getmtime(d) <= t for d in DEPS if os.path.exists(d))


def _includes(path: str, seen=None) -> set:
    """The file and every local header it includes, transitively."""
    seen = set() if seen is None else seen
    if path in seen or not os.path.exists(path):
        return seen
    seen.add(path)
    with open(path) as f:
        for line in f:
            line = line.strip()
            if line.startswith("#include \""):
                inc = line.split("\"")[1]
                _includes(os.path.normpath(os.path.join(os.path.dirname(path), inc)), seen)
    return seen


def _object_current(src: str, obj: str) -> bool:
    if not os.path.exists(obj):
        return False
    t = os.path.getmtime(obj)
    return all(os.path.getmtime(d) <= t for d in _includes(src) | {os.path.abspath(__file__)})


def build(force: bool = False, verbose: bool = False) -> str:
    if not force and up_to_date():
        return LIBPATH
    os.makedirs(OBJDIR, exist_ok=True)
    nvcc = nvcc_path()
    procs = []
    objs = []
    for src in SOURCES:
        obj = os.path.join(OBJDIR, os.path.basename(src).replace(".cu", ".o"))
        objs.append(obj)
        if not force and _object_current(src, obj):
            continue
        cmd = [nvcc, *NVCC_FLAGS, "-c", "-o", obj, src]
        procs.append((cmd, subprocess.Popen(cmd, stdout=subprocess.PIPE, stderr=subprocess.PIPE, text=True)))
    errors = []
    for cmd, p in procs:
        out, err = p.communicate()
        if p.returncode != 0:
            errors.append(" ".join(cmd) + "\n" + out + err)
        elif verbose:
            sys.stderr.write(err)
    if errors:
        raise RuntimeError("nvcc failed:\n" + "\n".join(errors))
    tmp = LIBPATH + ".tmp"
    link = [nvcc, *ARCH, "-shared", "-o", tmp, *objs]
    res = subprocess.run(link, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError("link failed:\n" + " ".join(link) + "\n" + res.stdout + res.stderr)
    os.replace(tmp, LIBPATH)
    return LIBPATH


def bindings_path() -> str:
    import sysconfig
    return os.path.join(HERE, "_C" + sysconfig.get_config_var("EXT_SUFFIX"))


def build_bindings(force: bool = False) -> str:
    """The PyBind11 module flashgen_b200._C, linked against the in-tree
    library (found through an $ORIGIN-relative rpath)."""
    import sysconfig
    import pybind11
    out = bindings_path()
    deps = [BINDINGS, os.path.join(ROOT, "include", "flashgen_sampler.h"), LIBPATH]
    if not force and os.path.exists(out) and all(os.path.getmtime(d) <= os.path.getmtime(out) for d in deps):
        return out
    cxx = shutil.which("g++") or "g++"
    cmd = [cxx, "-O2", "-shared", "-fPIC", "-std=c++17", "-fvisibility=hidden",
           "-I", pybind11.get_include(), "-I", sysconfig.get_paths()["include"],
           BINDINGS, "-o", out + ".tmp", "-L", LIBDIR, "-lflashgen_sampler", "-Wl,-rpath,$ORIGIN/lib"]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError("bindings build failed:\n" + " ".join(cmd) + "\n" + res.stdout + res.stderr)
    os.replace(out + ".tmp", out)
    return out


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose=True))
    print(build_bindings(force="--force" in sys.argv))
