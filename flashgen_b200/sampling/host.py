"""Host-buffer entry point: sample a batch whose inputs live in host memory.

This is the call an engine makes when its logits are not already on the GPU
(FlashGen's C++ engine copies logits device-to-host and samples on one CPU
thread, csrc/runtime/pipeline.cpp:274-340). ``HostBatchSampler.sample`` copies
the step's inputs host-to-device from pinned staging buffers, runs one fused
``fg_sample`` launch and copies the ``B`` token ids back.

The pinned staging buffers (parameters, uniforms, ids) are double-buffered:
call i writes set ``i % 2`` only after the host-to-device copies that call
i - 2 enqueued from that set have completed (an event per set), so a step never
reads the parameters of a later step, however far the host runs ahead of the
stream. The returned id tensor belongs to set ``i % 2`` too: it stays valid
until call i + 2 starts.
"""
from __future__ import annotations

from typing import Optional

import numpy as np
import torch

from .sampler import PackedParams, fused_sample


class _Staging:
    """One set of pinned host buffers and their device twins."""

    def __init__(self, batch: int, device):
        self.f32_h = torch.empty(7, batch, dtype=torch.float32).pin_memory()   # 5 params, uniforms, spare
        self.i32_h = torch.empty(batch, dtype=torch.int32).pin_memory()
        self.u8_h = torch.empty(batch, dtype=torch.uint8).pin_memory()
        self.ids_h = torch.empty(batch, dtype=torch.int64).pin_memory()
        self.f32_d = torch.empty(7, batch, dtype=torch.float32, device=device)
        self.i32_d = torch.empty(batch, dtype=torch.int32, device=device)
        self.u8_d = torch.empty(batch, dtype=torch.uint8, device=device)
        self.copied = None   # event after this set's last host-to-device copies


class HostBatchSampler:
    def __init__(self, batch: int, vocab: int, dtype: torch.dtype, max_hist: int, device):
        self.B, self.V, self.dev = batch, vocab, torch.device(device)
        self.logits_d = torch.empty(batch, vocab, dtype=dtype, device=self.dev)
        self.ids_d = torch.empty(batch, dtype=torch.int64, device=self.dev)
        self.hist_ids_d = torch.empty(max(1, max_hist), dtype=torch.int32, device=self.dev)
        self.hist_off_d = torch.empty(batch + 1, dtype=torch.int64, device=self.dev)
        self.status_d = torch.empty(batch, dtype=torch.int32, device=self.dev)
        self.sets = [_Staging(batch, self.dev), _Staging(batch, self.dev)]
        self.calls = 0
        self.h2d_bytes = 0
        self.d2h_bytes = 0

    def sample(self, logits_h: torch.Tensor, params, hist_ids_h: Optional[torch.Tensor],
               hist_off_h: Optional[torch.Tensor], uniforms_h: np.ndarray, hist_max_len: int = 0) -> torch.Tensor:
        """logits_h: pinned [B, V] host tensor; params: SoA numpy (BatchParams);
        hist_*_h: pinned CSR tensors or None. Returns a pinned host id tensor,
        valid once the current stream has reached this call and until the
        call after next."""
        B = self.B
        st = torch.cuda.current_stream(self.dev)
        s = self.sets[self.calls & 1]
        self.calls += 1
        if s.copied is not None:
            s.copied.synchronize()   # the copies out of this set (two calls ago) are done
        h2d = 0
        self.logits_d.copy_(logits_h, non_blocking=True)
        h2d += logits_h.numel() * logits_h.element_size()
        f = s.f32_h.numpy()
        f[0], f[1], f[2], f[3], f[4], f[5] = (params.temperature, params.top_p, params.repetition_penalty,
                                              params.presence_penalty, params.frequency_penalty, uniforms_h)
        s.i32_h.numpy()[:] = params.top_k
        s.u8_h.numpy()[:] = params.greedy
        s.f32_d.copy_(s.f32_h, non_blocking=True)
        s.i32_d.copy_(s.i32_h, non_blocking=True)
        s.u8_d.copy_(s.u8_h, non_blocking=True)
        h2d += s.f32_h.numel() * 4 + B * 4 + B
        hist = None
        if hist_ids_h is not None:
            n = hist_ids_h.numel()
            self.hist_ids_d[:n].copy_(hist_ids_h, non_blocking=True)
            self.hist_off_d.copy_(hist_off_h, non_blocking=True)
            h2d += n * 4 + (B + 1) * 8
            hist = (self.hist_ids_d, self.hist_off_d, hist_max_len)
        packed = PackedParams.__new__(PackedParams)
        packed.f32 = s.f32_d[:5]
        packed.top_k, packed.greedy = s.i32_d, s.u8_d
        packed.any_rep = bool(np.any(params.repetition_penalty != 1.0))
        packed.any_presence = bool(np.any(params.presence_penalty != 0.0))
        packed.any_frequency = bool(np.any(params.frequency_penalty != 0.0))
        packed.all_greedy = False
        fused_sample(self.logits_d, packed, s.f32_d[5], hist, out=self.ids_d, status=self.status_d)
        s.ids_h.copy_(self.ids_d, non_blocking=True)
        ev = torch.cuda.Event()
        ev.record(st)
        s.copied = ev
        self.h2d_bytes, self.d2h_bytes = h2d, B * 8
        return s.ids_h

    def status(self) -> np.ndarray:
        """Per-row status words of the last call (synchronises the stream)."""
        return self.status_d.cpu().numpy()

