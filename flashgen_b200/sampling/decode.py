"""Batched decode-step sampling with device-resident token histories.

FlashGen's engine samples a decode step one request at a time: for every
request it runs the model, then ``self._sampler._sample_one(logit,
req.sampling).item()`` (flashgen/engine.py:350-368), a host round trip per
token, with the history-dependent penalties applied on the host
(sampler.py:123-147). ``DecodeBatch`` is the batched replacement for that
loop's sampling half: it keeps every row's token history on the GPU, hands
the step's ``[B, V]`` logits straight to one ``fg_sample`` call, and appends
the drawn ids to the histories on the device. Nothing crosses to the host
unless the caller reads the ids.

Histories live in a ``[B, capacity]`` int32 buffer with a length per row. Each
step rebuilds the compact CSR view ``fg_sample`` reads (ids, int64 offsets)
with device-only torch operations: a cumulative sum of the lengths and one
scatter of the valid entries, so the step never synchronises with the host.
A row whose history is full keeps its first ``capacity`` ids.
"""
from __future__ import annotations

from typing import List, Optional, Sequence

import torch

from .. import _lib
from ..core.config import SamplingParams
from .sampler import PackedParams, _status_error, fused_sample, workspace_for


class DecodeBatch:
    """Per-row sampling state of a batch of sequences decoding together.

    >>> dec = DecodeBatch(params, vocab=V, capacity=4096, device="cuda")
    >>> dec.set_history(i, prompt_ids)          # once per row
    >>> ids = dec.step(logits)                  # [B] int64, on the device
    """

    def __init__(self, params: Sequence[SamplingParams], vocab: int, capacity: int = 4096,
                 device="cuda", check_errors: bool = False):
        self.device = torch.device(device)
        self.B = len(params)
        self.V = int(vocab)
        self.capacity = int(capacity)
        self.params = list(params)
        self.packed = PackedParams.from_params(self.params, self.device)
        self.hist = torch.zeros(self.B, self.capacity, dtype=torch.int32, device=self.device)
        self.lens = torch.zeros(self.B, dtype=torch.int64, device=self.device)
        # the compact CSR view fg_sample reads (rebuilt each step)
        self.csr_ids = torch.zeros(self.B * self.capacity + 1, dtype=torch.int32, device=self.device)
        self.csr_off = torch.zeros(self.B + 1, dtype=torch.int64, device=self.device)
        self._col = torch.arange(self.capacity, device=self.device).unsqueeze(0)   # [1, capacity]
        self.status = torch.empty(self.B, dtype=torch.int32, device=self.device)
        self.out = torch.empty(self.B, dtype=torch.int64, device=self.device)
        self.check_errors = check_errors

    def set_history(self, row: int, ids: Sequence[int]) -> None:
        """Row `row`'s history so far (prompt and generated ids), from the host."""
        t = torch.as_tensor(list(ids)[: self.capacity], dtype=torch.int32)
        self.hist[row, : t.numel()] = t.to(self.device)
        self.lens[row] = t.numel()

    def histories(self) -> List[List[int]]:
        """The rows' histories on the host (reads the device state)."""
        h, n = self.hist.cpu(), self.lens.cpu()
        return [h[r, : int(n[r])].tolist() for r in range(self.B)]

    def _csr(self):
        lens = self.lens
        torch.cumsum(lens, 0, out=self.csr_off[1:])
        valid = self._col < lens.unsqueeze(1)                               # [B, capacity]
        dst = self.csr_off[:-1].unsqueeze(1) + self._col                    # compact position
        dump = self.csr_ids.numel() - 1                                     # invalid entries land here
        dst = torch.where(valid, dst, torch.full_like(dst, dump))
        self.csr_ids.index_put_((dst.reshape(-1),), self.hist.reshape(-1))
        return self.csr_ids, self.csr_off, self.capacity

    def step(self, logits: torch.Tensor, uniforms: Optional[torch.Tensor] = None,
             generator: Optional[torch.Generator] = None) -> torch.Tensor:
        """Sample one token per row from `logits` [B, V] (on this device) with the
        rows' penalties over their histories, append it to the histories and
        return the ids ([B] int64, on the device; the same buffer every step,
        so read or copy it before the next step)."""
        assert logits.shape == (self.B, self.V), (logits.shape, self.B, self.V)
        if uniforms is None:
            uniforms = torch.rand(self.B, device=self.device, generator=generator, dtype=torch.float32)
        stream = torch.cuda.current_stream(self.device)
        need = _lib.workspace_size(self.B, self.V, {torch.float32: _lib.FG_DTYPE_F32,
                                                    torch.float16: _lib.FG_DTYPE_F16,
                                                    torch.bfloat16: _lib.FG_DTYPE_BF16}[logits.dtype],
                                   self.capacity)
        ws = workspace_for(self.device, stream, need)
        ids = fused_sample(logits.contiguous(), self.packed, uniforms, self._csr(), out=self.out,
                           status=self.status, workspace=ws)
        if self.check_errors:
            msg = _status_error(self.status)
            if msg is not None:
                raise RuntimeError(msg)
        self._append(ids)
        return ids

    def _append(self, ids: torch.Tensor) -> None:
        """Append each row's id (skipping error rows, id -1) on the device; a
        full row keeps its first `capacity` ids."""
        take = (self.lens < self.capacity) & (ids >= 0)
        pos = torch.clamp(self.lens, max=self.capacity - 1)
        cur = self.hist.gather(1, pos.unsqueeze(1)).squeeze(1)
        new = torch.where(take, ids.to(torch.int32), cur)
        self.hist.scatter_(1, pos.unsqueeze(1), new.unsqueeze(1))
        self.lens += take.to(torch.int64)
