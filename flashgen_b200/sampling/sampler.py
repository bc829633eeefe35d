"""Token sampler: drop-in for FlashGen's ``flashgen.sampling.sampler.Sampler``.

Same class, method names, argument meaning and return types as the
reference (``flashgen/sampling/sampler.py:46-169``); every method runs on the
GPU through the C ABI (``include/flashgen_sampler.h``) — one fused sm_100a
kernel per call — with no host copy of the logits.

Differences a caller can observe, all deliberate:

* The draw is an inverse CDF driven by one uniform per row (``uniforms=``,
  default ``torch.rand`` on the logits' device) instead of
  ``torch.multinomial``; the distribution is the same, the random stream is not.
* Ties at the top-p cut are kept in ascending token-id order (the reference's
  unstable ``sort`` leaves that order unspecified).
* Rows with ``temperature == 0`` are greedy (as in
  ``csrc/runtime/pipeline.cpp:284``); the reference's Python path would sample
  them at temperature 1.
* Penalties (repetition, presence, frequency) are applied inside ``sample``
  when ``token_histories`` is given; the reference only offers
  ``apply_repetition_penalty`` as a separate in-place helper (kept here too).
"""
from __future__ import annotations

from typing import List, Optional, Sequence, Tuple, Union

import numpy as np
import torch

from .. import _lib
from ..core.config import SamplingParams

_DTYPES = {torch.float32: _lib.FG_DTYPE_F32, torch.float16: _lib.FG_DTYPE_F16,
           torch.bfloat16: _lib.FG_DTYPE_BF16}

History = Union[None, Sequence[Sequence[int]], Tuple[torch.Tensor, torch.Tensor]]


def _ptr(t: Optional[torch.Tensor]) -> Optional[int]:
    return None if t is None else t.data_ptr()


def _row_logits(logits: torch.Tensor) -> torch.Tensor:
    if logits.dtype not in _DTYPES:
        logits = logits.float()
    if logits.stride(-1) != 1:
        logits = logits.contiguous()
    return logits


def histories_to_csr(histories: Sequence[Sequence[int]], device) -> Tuple[torch.Tensor, torch.Tensor, int]:
    """Pack per-row token lists into CSR (ids int32, offsets int64) on ``device``."""
    lens = np.fromiter((len(h) for h in histories), dtype=np.int64, count=len(histories))
    offs = np.zeros(len(histories) + 1, dtype=np.int64)
    np.cumsum(lens, out=offs[1:])
    if offs[-1] > 0:
        ids = np.concatenate([np.asarray(h, dtype=np.int32).reshape(-1) for h in histories])
    else:
        ids = np.zeros(0, dtype=np.int32)
    hmax = int(lens.max()) if len(lens) else 0
    return (torch.from_numpy(ids).to(device, non_blocking=True),
            torch.from_numpy(offs).to(device, non_blocking=True), hmax)


class PackedParams:
    """Per-row parameters as device structure-of-arrays."""

    def __init__(self, temperature, top_p, top_k, rep, presence, frequency, greedy, device):
        B = len(temperature)
        host = np.empty((5, B), dtype=np.float32)
        host[0], host[1], host[2], host[3], host[4] = temperature, top_p, rep, presence, frequency
        self.f32 = torch.from_numpy(host).to(device, non_blocking=True)
        self.top_k = torch.from_numpy(np.asarray(top_k, dtype=np.int32).copy()).to(device, non_blocking=True)
        self.greedy = torch.from_numpy(np.asarray(greedy, dtype=np.uint8).copy()).to(device, non_blocking=True)
        self.any_rep = bool(np.any(np.asarray(rep) != 1.0))
        self.any_presence = bool(np.any(np.asarray(presence) != 0.0))
        self.any_frequency = bool(np.any(np.asarray(frequency) != 0.0))
        self.all_greedy = bool(np.all(np.asarray(greedy) | (np.asarray(temperature) == 0.0)))

    @staticmethod
    def from_params(params: Sequence[SamplingParams], device) -> "PackedParams":
        return PackedParams([p.temperature for p in params], [p.top_p for p in params],
                            [p.top_k for p in params], [p.repetition_penalty for p in params],
                            [getattr(p, "presence_penalty", 0.0) for p in params],
                            [getattr(p, "frequency_penalty", 0.0) for p in params],
                            [bool(p.greedy) for p in params], device)


_WORKSPACES = {}


def workspace_for(device: torch.device, stream: torch.cuda.Stream, nbytes: int = 0) -> torch.Tensor:
    """The zero-initialised fg_sample workspace of (device, stream), at least
    `nbytes` long (it grows, zeroed, when a call needs more). Calls on one
    stream are serialised by the stream, so they can share it."""
    key = (device.index, stream.cuda_stream)
    ws = _WORKSPACES.get(key)
    need = max(int(nbytes), _lib.FG_SAMPLE_WORKSPACE_MIN_BYTES)
    if ws is None or ws.numel() * 4 < need:
        ws = torch.zeros((need + 3) // 4, dtype=torch.int32, device=device)
        _WORKSPACES[key] = ws
    return ws


def fused_sample(logits: torch.Tensor, packed: PackedParams, uniforms: torch.Tensor,
                 hist: Optional[Tuple[torch.Tensor, torch.Tensor, int]] = None,
                 out: Optional[torch.Tensor] = None, status: Optional[torch.Tensor] = None,
                 probs: Optional[torch.Tensor] = None, vocab_offset: int = 0, vocab_total: int = 0,
                 stream: Optional[torch.cuda.Stream] = None,
                 workspace: Optional[torch.Tensor] = None) -> torch.Tensor:
    """One fg_sample call on device tensors (no checks beyond the C ABI's)."""
    lib = _lib.load()
    B, V = logits.shape
    if out is None:
        out = torch.empty(B, dtype=torch.int64, device=logits.device)
    a = _lib.FgSampleArgs()
    a.logits = logits.data_ptr()
    a.dtype = _DTYPES[logits.dtype]
    a.batch, a.vocab = B, V
    a.row_stride = logits.stride(0) if B > 1 else V
    a.vocab_offset, a.vocab_total = vocab_offset, vocab_total
    if hist is not None:
        a.hist_ids, a.hist_offsets, a.hist_max_len = hist[0].data_ptr(), hist[1].data_ptr(), int(hist[2])
    f = packed.f32
    a.temperature, a.top_p = _ptr(f[0]), _ptr(f[1])
    a.repetition_penalty = _ptr(f[2]) if packed.any_rep else None
    a.presence_penalty = _ptr(f[3]) if packed.any_presence else None
    a.frequency_penalty = _ptr(f[4]) if packed.any_frequency else None
    a.top_k, a.greedy = _ptr(packed.top_k), _ptr(packed.greedy)
    a.uniforms = uniforms.data_ptr()
    a.out_ids = out.data_ptr()
    a.out_status = _ptr(status)
    a.out_probs = _ptr(probs)
    st = stream if stream is not None else torch.cuda.current_stream(logits.device)
    if workspace is None:
        need = _lib.workspace_size(B, V, a.dtype, a.hist_max_len if hist is not None else 0)
        workspace = workspace_for(logits.device, st, need)
    _lib.set_workspace(a, workspace)
    with torch.cuda.device(logits.device):
        _lib.check(lib.fg_sample(a, st.cuda_stream), "fg_sample")
    return out


def _status_error(status: torch.Tensor) -> Optional[str]:
    s = status.cpu().numpy()
    bad = np.nonzero(s & _lib.FG_ROW_ERROR_MASK)[0]
    if len(bad) == 0:
        return None
    names = {_lib.FG_ROW_NAN: "nan", _lib.FG_ROW_POS_INF: "+inf", _lib.FG_ROW_ALL_MASKED: "all -inf",
             _lib.FG_ROW_BAD_HISTORY: "history id out of range", _lib.FG_ROW_BAD_PARAM: "bad parameter",
             _lib.FG_ROW_BAD_UNIFORM: "uniform outside [0,1)", _lib.FG_ROW_TIMEOUT: "pipeline timeout"}
    r = int(bad[0])
    what = ", ".join(n for b, n in names.items() if s[r] & b)
    return f"probability tensor contains either `inf`, `nan` or element < 0 (row {r}: {what}; {len(bad)} row(s))"


class Sampler:
    """Token sampler supporting greedy, top-k, top-p, temperature and penalties.

    Example
    -------
    >>> sampler = Sampler()
    >>> tokens = sampler.sample(logits, [params_for_seq_0, params_for_seq_1])
    """

    def __init__(self, check_errors: bool = True):
        # check_errors=True reads the per-row status back (one small D2H copy
        # and a stream sync) and raises like the reference does on NaN/inf
        # probabilities; False keeps the call fully asynchronous.
        self.check_errors = check_errors
        self.last_status: Optional[torch.Tensor] = None
        self.last_probs: Optional[torch.Tensor] = None

    def sample(
        self,
        logits: torch.Tensor,          # [B, vocab_size]
        params: List[SamplingParams],
        *,
        token_histories: History = None,
        uniforms: Optional[torch.Tensor] = None,
        generator: Optional[torch.Generator] = None,
        return_probs: bool = False,
    ) -> torch.Tensor:
        """Sample one token per sequence in the batch. Returns [B] int64 ids."""
        assert logits.dim() == 2
        B, V = logits.shape
        assert len(params) == B
        if not logits.is_cuda:
            raise RuntimeError("flashgen_b200 samples on the GPU only; logits are on " + str(logits.device))
        logits = _row_logits(logits)
        dev = logits.device
        packed = PackedParams.from_params(params, dev)
        hist = None
        if token_histories is not None:
            if isinstance(token_histories, tuple) and len(token_histories) in (2, 3) and \
                    isinstance(token_histories[0], torch.Tensor):
                ids, offs = token_histories[0], token_histories[1]
                hmax = int(token_histories[2]) if len(token_histories) == 3 else \
                    int((offs[1:] - offs[:-1]).max().item()) if B > 0 else 0
                hist = (ids.to(dev, torch.int32).contiguous(), offs.to(dev, torch.int64).contiguous(), hmax)
            else:
                assert len(token_histories) == B
                hist = histories_to_csr(token_histories, dev)
        if B == 0:
            return torch.empty(0, dtype=torch.int64, device=dev)
        if uniforms is None:
            uniforms = torch.rand(B, device=dev, generator=generator, dtype=torch.float32)
        else:
            uniforms = uniforms.to(dev, torch.float32).contiguous()
        status = torch.empty(B, dtype=torch.int32, device=dev)
        probs = torch.empty(B, V, dtype=torch.float32, device=dev) if return_probs else None
        out = fused_sample(logits, packed, uniforms, hist, status=status, probs=probs)
        self.last_status, self.last_probs = status, probs
        if self.check_errors:
            msg = _status_error(status)
            if msg is not None:
                raise RuntimeError(msg)
        return out

    def sample_batch(
        self,
        logits: torch.Tensor,    # [B, vocab_size]
        params: SamplingParams,  # same params for all sequences
        **kwargs,
    ) -> torch.Tensor:
        """Batch sampling when all sequences share the same params."""
        return self.sample(logits, [params] * logits.shape[0], **kwargs)

    def _sample_one(self, logit: torch.Tensor, p: SamplingParams, **kwargs) -> torch.Tensor:
        """Sample one token from a single logit vector; returns a 0-d int64 tensor."""
        return self.sample(logit.reshape(1, -1), [p], **kwargs)[0]

    def apply_repetition_penalty(
        self,
        logits: torch.Tensor,          # [B, vocab]
        token_histories: List[List[int]],
        penalty: float,
    ) -> torch.Tensor:
        """Apply repetition penalty in place across a batch (one fused launch)."""
        if penalty == 1.0:
            return logits
        if not logits.is_cuda:
            raise RuntimeError("flashgen_b200 runs on the GPU only")
        assert logits.dim() == 2 and logits.stride(-1) == 1 and logits.dtype in _DTYPES
        B, V = logits.shape
        ids, offs, _ = histories_to_csr(token_histories, logits.device)
        pen = torch.full((B,), float(penalty), dtype=torch.float32, device=logits.device)
        lib = _lib.load()
        st = torch.cuda.current_stream(logits.device)
        with torch.cuda.device(logits.device):
            _lib.check(lib.fg_apply_repetition_penalty(
                logits.data_ptr(), _DTYPES[logits.dtype], B, V, logits.stride(0) if B > 1 else V,
                ids.data_ptr(), offs.data_ptr(), pen.data_ptr(), st.cuda_stream), "fg_apply_repetition_penalty")
        return logits

    @staticmethod
    def argmax(logits: torch.Tensor) -> torch.Tensor:
        """Row argmax (first maximum; NaN wins, as torch.argmax)."""
        logits = _row_logits(logits)
        B, V = logits.shape
        out = torch.empty(B, dtype=torch.int64, device=logits.device)
        lib = _lib.load()
        st = torch.cuda.current_stream(logits.device)
        with torch.cuda.device(logits.device):
            _lib.check(lib.fg_argmax(logits.data_ptr(), _DTYPES[logits.dtype], B, V,
                                     logits.stride(0) if B > 1 else V, out.data_ptr(), st.cuda_stream),
                       "fg_argmax")
        return out
