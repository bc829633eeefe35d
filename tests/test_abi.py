"""The C-ABI library loads, exports every symbol include/flashgen_sampler.h
declares, and its argument struct has the same layout in C and in ctypes.
No GPU needed: only argument validation paths are called."""
import ctypes
import os
import re
import subprocess

import pytest

from flashgen_b200 import _lib

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "flashgen_sampler.h")


def declared_functions():
    src = open(HEADER).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"^\s*(?:const\s+)?\w+\**\s+\**(fg_\w+)\s*\(", src, flags=re.M)))


def test_symbols_exported():
    lib = _lib.load()
    names = declared_functions()
    assert set(names) == set(_lib.EXPORTED_SYMBOLS)
    for n in names:
        assert hasattr(lib, n), n
    out = subprocess.run(["nm", "-D", "--defined-only", _lib.lib_path()], capture_output=True, text=True).stdout
    for n in names:
        assert re.search(r"\bT " + n + r"\b", out), n


def test_struct_layout_matches_header(tmp_path):
    fields = [f[0] for f in _lib.FgSampleArgs._fields_]
    prog = '#include <stdio.h>\n#include <stddef.h>\n#include "flashgen_sampler.h"\nint main(void){\n'
    prog += 'printf("%zu\\n", sizeof(FgSampleArgs));\n'
    for f in fields:
        prog += f'printf("%zu\\n", offsetof(FgSampleArgs, {f}));\n'
    prog += "return 0;}\n"
    c = tmp_path / "probe.c"
    c.write_text(prog)
    exe = tmp_path / "probe"
    subprocess.check_call(["gcc", "-std=c99", "-I", os.path.dirname(HEADER), str(c), "-o", str(exe)])
    vals = [int(v) for v in subprocess.check_output([str(exe)]).split()]
    assert vals[0] == ctypes.sizeof(_lib.FgSampleArgs)
    for f, off in zip(fields, vals[1:]):
        assert getattr(_lib.FgSampleArgs, f).offset == off, f


def test_header_compiles_as_cxx(tmp_path):
    c = tmp_path / "probe.cc"
    c.write_text('#include "flashgen_sampler.h"\nint main(){ return fg_version() > 0 ? 0 : 1; }\n')
    subprocess.check_call(["g++", "-fsyntax-only", "-I", os.path.dirname(HEADER), str(c)])


def test_validation_without_gpu():
    lib = _lib.load()
    assert lib.fg_version() == 200
    assert lib.fg_sample(None, None) == _lib.FG_EINVAL
    a = _lib.FgSampleArgs()
    assert lib.fg_sample(ctypes.byref(a), None) == _lib.FG_EINVAL      # null logits
    a.logits, a.dtype, a.batch, a.vocab, a.row_stride = 16, 7, 1, 8, 8
    assert lib.fg_sample(ctypes.byref(a), None) == _lib.FG_EINVAL      # bad dtype
    a.dtype = _lib.FG_DTYPE_F32
    a.temperature = a.top_p = a.top_k = a.uniforms = a.out_ids = 16
    a.row_stride, a.batch = 8, 0
    assert lib.fg_sample(ctypes.byref(a), None) == _lib.FG_EINVAL      # no workspace
    a.workspace, a.batch = 256, 1
    a.workspace_bytes = _lib.FG_SAMPLE_WORKSPACE_MIN_BYTES - 1
    assert lib.fg_sample(ctypes.byref(a), None) == _lib.FG_EINVAL      # workspace below the counters
    a.workspace_bytes = _lib.FG_SAMPLE_WORKSPACE_MIN_BYTES
    a.row_stride = 4
    assert lib.fg_sample(ctypes.byref(a), None) == _lib.FG_EINVAL      # stride < vocab
    a.row_stride, a.batch = 8, 0
    assert lib.fg_sample(ctypes.byref(a), None) == _lib.FG_OK          # empty batch: nothing to do
    a.batch = (1 << 30) + 1
    assert lib.fg_sample(ctypes.byref(a), None) == _lib.FG_ENOTSUP     # row-queue counter bound
    a.batch, a.hist_ids = 1, 16
    assert lib.fg_sample(ctypes.byref(a), None) == _lib.FG_EINVAL      # ids without offsets
    assert lib.fg_argmax(None, 0, 1, 8, 8, None, None) == _lib.FG_EINVAL
    assert lib.fg_strerror(_lib.FG_ENOTSUP).decode().startswith("shape")


def test_noalloc_validation_without_gpu():
    lib = _lib.load()
    assert lib.fg_sample_noalloc(None, None) == _lib.FG_EINVAL
    a = _lib.FgSampleArgs()
    a.workspace = 256
    assert lib.fg_sample_noalloc(ctypes.byref(a), None) == _lib.FG_EINVAL   # takes no workspace
    a.workspace = None
    a.batch = (1 << 30) + 1
    assert lib.fg_sample_noalloc(ctypes.byref(a), None) == _lib.FG_ESCRATCH
    assert "scratch" in lib.fg_strerror(_lib.FG_ESCRATCH).decode()


def test_workspace_size_query_without_gpu():
    lib = _lib.load()
    # the batch path keeps a block per row; the size grows with batch and history
    small = _lib.workspace_size(1024, 128256, _lib.FG_DTYPE_BF16, 0)
    big = _lib.workspace_size(1024, 128256, _lib.FG_DTYPE_BF16, 1024)
    assert _lib.FG_SAMPLE_WORKSPACE_MIN_BYTES < small < big
    assert _lib.workspace_size(2048, 128256, _lib.FG_DTYPE_BF16, 1024) > big
    for B, V in ((1, 256000), (4, 128256), (37, 128256), (8, 50257), (1, 7)):
        for dt in (_lib.FG_DTYPE_F32, _lib.FG_DTYPE_F16, _lib.FG_DTYPE_BF16):
            assert _lib.workspace_size(B, V, dt, 512) >= _lib.FG_SAMPLE_WORKSPACE_MIN_BYTES
    assert lib.fg_sample_workspace_size(1, 8, 9, 0) == 0         # bad dtype
    assert lib.fg_sample_workspace_size(-1, 8, 0, 0) == 0        # bad batch
    assert lib.fg_sample_workspace_size(1, 8, 0, -1) == 0        # bad history bound


def test_split_mode_validation_without_gpu():
    lib = _lib.load()
    for bad in (-1, 3, 100):
        assert lib.fg_sample_set_split(bad) == _lib.FG_EINVAL
    for mode in (0, 2, 1):   # ends on the default (automatic)
        assert lib.fg_sample_set_split(mode) == _lib.FG_OK
