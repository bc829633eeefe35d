"""ctypes binding of include/flashgen_sampler.h.

The shared library is built in tree by ``flashgen_b200.build``. Loading fails
loudly when it is missing: there is no CPU or PyTorch fallback for sampling.
"""
from __future__ import annotations

import ctypes
import os
import threading

from . import build as _build

FG_OK, FG_EINVAL, FG_ELAUNCH, FG_ENOTSUP, FG_EDEVICE, FG_ESCRATCH = 0, 1, 2, 3, 4, 5
FG_DTYPE_F32, FG_DTYPE_F16, FG_DTYPE_BF16 = 0, 1, 2

FG_ROW_NAN = 0x0001
FG_ROW_POS_INF = 0x0002
FG_ROW_ALL_MASKED = 0x0004
FG_ROW_BAD_HISTORY = 0x0008
FG_ROW_BAD_PARAM = 0x0010
FG_ROW_BAD_UNIFORM = 0x0020
FG_ROW_TIMEOUT = 0x0040
FG_ROW_CAND_TRUNC = 0x0080
FG_ROW_ERROR_MASK = 0x00FF
FG_ROW_GENERAL_PATH = 0x0100
FG_ROW_GREEDY = 0x0200

EXPORTED_SYMBOLS = ("fg_sample", "fg_sample_workspace_size", "fg_sample_candidates", "fg_sample_noalloc",
                    "fg_sample_set_split",
                    "fg_apply_repetition_penalty", "fg_argmax", "fg_strerror", "fg_version")


class FgSampleArgs(ctypes.Structure):
    """Mirror of ``FgSampleArgs`` (field order and types must match the header)."""

    _fields_ = [
        ("logits", ctypes.c_void_p),
        ("dtype", ctypes.c_int32),
        ("batch", ctypes.c_int32),
        ("vocab", ctypes.c_int32),
        ("hist_max_len", ctypes.c_int32),
        ("row_stride", ctypes.c_int64),
        ("vocab_offset", ctypes.c_int64),
        ("vocab_total", ctypes.c_int64),
        ("hist_ids", ctypes.c_void_p),
        ("hist_offsets", ctypes.c_void_p),
        ("temperature", ctypes.c_void_p),
        ("top_p", ctypes.c_void_p),
        ("top_k", ctypes.c_void_p),
        ("repetition_penalty", ctypes.c_void_p),
        ("presence_penalty", ctypes.c_void_p),
        ("frequency_penalty", ctypes.c_void_p),
        ("greedy", ctypes.c_void_p),
        ("uniforms", ctypes.c_void_p),
        ("out_ids", ctypes.c_void_p),
        ("out_status", ctypes.c_void_p),
        ("out_probs", ctypes.c_void_p),
        ("workspace", ctypes.c_void_p),
        ("workspace_bytes", ctypes.c_size_t),
    ]


FG_SAMPLE_WORKSPACE_MIN_BYTES = 256


_lib = None
_lock = threading.Lock()


def lib_path() -> str:
    return _build.LIBPATH


def load(build_if_missing: bool = True) -> ctypes.CDLL:
    """Load (building first if needed) the sampler library."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is not None:
            return _lib
        path = _build.LIBPATH
        if not os.path.exists(path):
            if not build_if_missing:
                raise RuntimeError(f"flashgen_b200: {path} is missing; run `python -m flashgen_b200.build`")
            _build.build()
        lib = ctypes.CDLL(path)
        lib.fg_sample.argtypes = [ctypes.POINTER(FgSampleArgs), ctypes.c_void_p]
        lib.fg_sample.restype = ctypes.c_int
        lib.fg_sample_workspace_size.argtypes = [ctypes.c_int32, ctypes.c_int32, ctypes.c_int32, ctypes.c_int32]
        lib.fg_sample_workspace_size.restype = ctypes.c_size_t
        lib.fg_sample_candidates.argtypes = [ctypes.POINTER(FgSampleArgs), ctypes.c_void_p, ctypes.c_void_p,
                                             ctypes.c_void_p, ctypes.c_int32, ctypes.c_void_p]
        lib.fg_sample_candidates.restype = ctypes.c_int
        lib.fg_sample_noalloc.argtypes = [ctypes.POINTER(FgSampleArgs), ctypes.c_void_p]
        lib.fg_sample_noalloc.restype = ctypes.c_int
        lib.fg_sample_set_split.argtypes = [ctypes.c_int]
        lib.fg_sample_set_split.restype = ctypes.c_int
        lib.fg_apply_repetition_penalty.argtypes = [
            ctypes.c_void_p, ctypes.c_int32, ctypes.c_int32, ctypes.c_int32, ctypes.c_int64,
            ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p]
        lib.fg_apply_repetition_penalty.restype = ctypes.c_int
        lib.fg_argmax.argtypes = [ctypes.c_void_p, ctypes.c_int32, ctypes.c_int32, ctypes.c_int32,
                                  ctypes.c_int64, ctypes.c_void_p, ctypes.c_void_p]
        lib.fg_argmax.restype = ctypes.c_int
        lib.fg_strerror.argtypes = [ctypes.c_int]
        lib.fg_strerror.restype = ctypes.c_char_p
        lib.fg_version.argtypes = []
        lib.fg_version.restype = ctypes.c_int
        _lib = lib
        return lib


def set_workspace(a: FgSampleArgs, ws) -> None:
    """Point ``a`` at a device workspace tensor and record its size."""
    a.workspace = ws.data_ptr()
    a.workspace_bytes = ws.numel() * ws.element_size()


def workspace_size(batch: int, vocab: int, dtype: int, hist_max_len: int) -> int:
    """Workspace bytes of fg_sample's fastest path for this shape."""
    return int(load().fg_sample_workspace_size(batch, vocab, dtype, max(0, int(hist_max_len))))


def check(rc: int, what: str) -> None:
    if rc != FG_OK:
        msg = load().fg_strerror(rc).decode()
        raise RuntimeError(f"{what} failed: {msg} (code {rc})")
