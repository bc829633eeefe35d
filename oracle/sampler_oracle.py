"""CPU oracle for FlashGen's decode-step sampling path.

TEST INFRASTRUCTURE ONLY. Only ``tests/``, ``__graft_entry__.smoke()`` and the
CPU-baseline / reference legs of ``bench.py`` may import this module, and only
as the checker or as the timed CPU baseline. The product path
(``flashgen_b200``) never calls it and has no CPU fallback.

What it restates (paths inside the FlashGen project):

* ``flashgen/sampling/sampler.py:123-147`` ``Sampler.apply_repetition_penalty``:
  per row, ``unique(history)``; ``x > 0 ? x / penalty : x * penalty``.
* presence / frequency penalties: absent from the reference; restated as the
  usual convention ``x - frequency * count - presence`` on ids present in the
  history, evaluated in fp32 left to right (the build's own specification).
* greedy: ``params.greedy or temperature == 0`` takes ``argmax`` (first index),
  like ``sampler.py:74-75,82-84`` and ``csrc/runtime/pipeline.cpp:284``.
* ``sampler.py:108-109`` temperature: ``x / T`` when ``T != 1 and T > 0``
  (fp32 IEEE division by the fp32 temperature).
* ``sampler.py:149-154`` ``_top_k_filter``: ``k = min(k, V)``; threshold is the
  k-th largest value; keep ``x >= threshold`` (all ties kept).
* ``sampler.py:156-169`` ``_top_p_filter``: sort descending, softmax, cumsum,
  remove where ``cumsum - p > top_p``. The reference's ``sort`` is not stable
  on CPU (tie order is implementation-defined), so the oracle sorts stably
  (ties in ascending id order, the order the CUDA kernel uses) and flags rows
  whose cut falls inside a run of tied values (``tie_at_cut``).
* ``sampler.py:120`` ``probs = softmax(filtered)``.
* draw: the reference calls ``torch.multinomial``, which cannot be driven by a
  caller-supplied uniform. Restated as an inverse CDF over the kept tokens in
  descending-probability order (ties in ascending id order), the order
  FlashGen's native sampler draws in (``csrc/runtime/pipeline.cpp:311-340``):
  the first token whose inclusive cumulative probability exceeds
  ``u * sum(probs)``, accumulated in float64.

Parity flags returned per row (a CUDA result may differ from the oracle only
on flagged rows):

* ``near_u``: ``u * S`` lies within ``1e-6 * S`` of a CDF boundary of the
  chosen token;
* ``near_p``: the exclusive prefix mass of the last kept or first removed
  token (in sorted order) lies within ``1e-6`` of ``top_p``, or the
  reference's own fp32 arithmetic (fp32 softmax over the sorted logits, whose
  sum drops the many tiny tail terms) puts the cut on a different token than
  the same computation in float64 — the cut then lies within the reference's
  rounding error of ``top_p``;
* ``tie_at_cut`` (informational): the top-p cut splits a run of equal values,
  where the reference's unstable sort leaves the kept subset unspecified.
"""
from __future__ import annotations

from dataclasses import dataclass, field
from typing import List, Optional, Sequence

import numpy as np
import torch
import torch.nn.functional as F

NEAR_TOL = 1e-6


@dataclass
class RowParams:
    """Structure-of-arrays sampling parameters (one entry per row)."""

    temperature: np.ndarray          # f32[B]
    top_p: np.ndarray                # f32[B]
    top_k: np.ndarray                # i32[B]
    repetition_penalty: np.ndarray   # f32[B]
    presence_penalty: np.ndarray     # f32[B]
    frequency_penalty: np.ndarray    # f32[B]
    greedy: np.ndarray               # bool[B]

    @property
    def batch(self) -> int:
        return int(self.temperature.shape[0])


@dataclass
class OracleResult:
    ids: np.ndarray                          # int64[B]
    near_u: np.ndarray                       # bool[B]
    near_p: np.ndarray                       # bool[B]
    tie_at_cut: np.ndarray                   # bool[B]
    greedy: np.ndarray                       # bool[B]
    error: np.ndarray                        # bool[B] (reference would raise)
    kept_ids: List[np.ndarray] = field(default_factory=list)    # ascending ids
    kept_probs: List[np.ndarray] = field(default_factory=list)  # f32 probs

    @property
    def flagged(self) -> np.ndarray:
        """Rows on which a correct implementation may draw a different id."""
        return self.near_u | self.near_p


def apply_repetition_penalty_row(x: torch.Tensor, history: Sequence[int],
                                 penalty: float) -> None:
    """In place on one fp32 row; follows sampler.py:134-146."""
    if penalty == 1.0 or len(history) == 0:
        return
    ids = torch.tensor(list(history), dtype=torch.long).unique()
    v = x[ids]
    x[ids] = torch.where(v > 0, v / penalty, v * penalty)


def apply_presence_frequency_row(x: torch.Tensor, history: Sequence[int],
                                 presence: float, frequency: float) -> None:
    """In place on one fp32 row: x[id] = (x[id] - f32(freq) * count) - f32(presence)."""
    if len(history) == 0 or (presence == 0.0 and frequency == 0.0):
        return
    ids, counts = torch.tensor(list(history), dtype=torch.long).unique(return_counts=True)
    v = x[ids]
    if frequency != 0.0:
        f = torch.tensor(frequency, dtype=torch.float32)
        v = v - f * counts.to(torch.float32)
    if presence != 0.0:
        v = v - torch.tensor(presence, dtype=torch.float32)
    x[ids] = v


def top_k_filter(logit: torch.Tensor, k: int) -> torch.Tensor:
    """sampler.py:149-154."""
    k = min(k, logit.shape[-1])
    threshold = logit.topk(k).values[-1]
    return logit.masked_fill(logit < threshold, float("-inf"))


def top_p_filter(logit: torch.Tensor, p: float, stable: bool = True):
    """sampler.py:156-169, with a selectable sort stability.

    Returns (filtered logits, near_p, tie_at_cut).
    """
    sorted_logits, sorted_indices = logit.sort(descending=True, stable=stable)
    probs_sorted = F.softmax(sorted_logits, dim=-1)
    cumulative_probs = probs_sorted.cumsum(dim=-1)
    excl = cumulative_probs - probs_sorted
    remove = excl > p
    # parity flags around the cut (sorted order)
    n_keep = int((~remove).sum())
    near = False
    tie = False
    V = logit.shape[-1]
    if n_keep < V:
        last = n_keep - 1
        for j in (last, last + 1):
            if 0 <= j < V and abs(float(excl[j]) - p) < NEAR_TOL:
                near = True
        if n_keep >= 1 and float(sorted_logits[n_keep - 1]) == float(sorted_logits[n_keep]) \
                and float(sorted_logits[n_keep]) != float("-inf"):
            tie = True
    # the same cut in float64 (exact to ~1e-16): a different position means the
    # reference's fp32 rounding decided the cut
    s64 = sorted_logits.to(torch.float64)
    e64 = torch.exp(s64 - s64[0])
    p64 = e64 / e64.sum()
    excl64 = torch.cumsum(p64, 0) - p64
    n_keep64 = int((~(excl64 > p)).sum())
    if n_keep64 != n_keep:
        near = True
    elif n_keep64 < V:
        for j in (n_keep64 - 1, n_keep64):
            if 0 <= j < V and abs(float(excl64[j]) - p) < NEAR_TOL:
                near = True
    sorted_logits = sorted_logits.masked_fill(remove, float("-inf"))
    return logit.scatter(0, sorted_indices, sorted_logits), near, tie


def inverse_cdf(filtered: torch.Tensor, probs: torch.Tensor, u: float):
    """Inverse CDF over the kept tokens (filtered != -inf) in descending value
    order, ties in ascending id order; cumulative sums in float64.

    Returns (token id, near_u).
    """
    kept = torch.nonzero(filtered != float("-inf")).flatten()
    order = kept[torch.sort(filtered[kept], descending=True, stable=True).indices]
    p64 = probs[order].to(torch.float64).numpy()
    cdf = np.cumsum(p64)
    total = float(cdf[-1])
    target = float(np.float64(np.float32(u))) * total
    j = int(np.searchsorted(cdf, target, side="right"))
    j = min(j, len(p64) - 1)
    while j > 0 and p64[j] == 0.0:   # never land on a zero-probability token
        j -= 1
    lo = cdf[j - 1] if j > 0 else 0.0
    hi = cdf[j]
    near = abs(target - lo) < NEAR_TOL * total or abs(hi - target) < NEAR_TOL * total
    return int(order[j]), near


def sample_rows(logits: torch.Tensor, params: RowParams,
                histories: Optional[Sequence[Sequence[int]]],
                uniforms: np.ndarray, stable: bool = True,
                want_kept: bool = True) -> OracleResult:
    """Run the whole chain row by row on the CPU (fp32 math, like the reference)."""
    assert logits.dim() == 2
    B, V = logits.shape
    ids = np.zeros(B, dtype=np.int64)
    near_u = np.zeros(B, dtype=bool)
    near_p = np.zeros(B, dtype=bool)
    tie = np.zeros(B, dtype=bool)
    gr = np.zeros(B, dtype=bool)
    err = np.zeros(B, dtype=bool)
    kept_ids: List[np.ndarray] = []
    kept_probs: List[np.ndarray] = []
    for r in range(B):
        x = logits[r].to(torch.float32).clone()
        hist = histories[r] if histories is not None else ()
        apply_repetition_penalty_row(x, hist, float(params.repetition_penalty[r]))
        apply_presence_frequency_row(x, hist, float(params.presence_penalty[r]),
                                     float(params.frequency_penalty[r]))
        T = float(params.temperature[r])
        if bool(params.greedy[r]) or T == 0.0:
            gr[r] = True
            ids[r] = int(x.argmax())
            if want_kept:
                kept_ids.append(np.array([ids[r]], dtype=np.int64))
                kept_probs.append(np.array([1.0], dtype=np.float32))
            continue
        if T != 1.0 and T > 0:
            x = x / torch.tensor(T, dtype=torch.float32)
        k = int(params.top_k[r])
        if k > 0:
            x = top_k_filter(x, k)
        p = float(params.top_p[r])
        if 0.0 < p < 1.0:
            x, near_p[r], tie[r] = top_p_filter(x, p, stable=stable)
        probs = F.softmax(x, dim=-1)
        if not bool(torch.isfinite(probs).all()):
            err[r] = True
            ids[r] = -1
            if want_kept:
                kept_ids.append(np.zeros(0, dtype=np.int64))
                kept_probs.append(np.zeros(0, dtype=np.float32))
            continue
        j, near_u[r] = inverse_cdf(x, probs, float(uniforms[r]))
        ids[r] = j
        if want_kept:
            nz = torch.nonzero(x != float("-inf")).flatten()
            kept_ids.append(nz.numpy().astype(np.int64))
            kept_probs.append(probs[nz].numpy().astype(np.float32))
    return OracleResult(ids, near_u, near_p, tie, gr, err, kept_ids, kept_probs)


def argmax_rows(logits: torch.Tensor) -> np.ndarray:
    """torch.argmax over fp32-upcast rows (sampler.py:74-75)."""
    return logits.to(torch.float32).argmax(dim=-1).numpy().astype(np.int64)


def repetition_penalty_inplace(logits: torch.Tensor,
                               histories: Sequence[Sequence[int]],
                               penalties: Sequence[float]) -> torch.Tensor:
    """Batched in-place repetition penalty in the buffer's own dtype
    (sampler.py:123-147, one penalty per row)."""
    for i, hist in enumerate(histories):
        pen = float(penalties[i])
        if pen == 1.0 or len(hist) == 0:
            continue
        uid = torch.tensor(list(hist), dtype=torch.long).unique()
        v = logits[i, uid]
        logits[i, uid] = torch.where(v > 0, v / pen, v * pen)
    return logits


def reference_chain_rows(logits: torch.Tensor, params: RowParams,
                         histories: Optional[Sequence[Sequence[int]]],
                         generator: Optional[torch.Generator] = None) -> np.ndarray:
    """The reference's own CPU sampling path, timed as the CPU baseline.

    The torch operations of FlashGen's decode step in the reference's order,
    without this module's parity flags, float64 cut and kept sets:
    ``Sampler.apply_repetition_penalty`` (sampler.py:123-147, unique history
    ids), then ``Sampler.sample`` (sampler.py:57-88): the all-greedy fast path
    (argmax of the batch), else per row argmax (greedy) or ``_sample_one``
    (sampler.py:102-121): ``x / T``, ``_top_k_filter``, ``_top_p_filter``
    (torch's default sort, sampler.py:156-169), softmax and
    ``torch.multinomial``. Presence and frequency penalties are absent from
    the reference and are not applied here.
    """
    B, V = logits.shape
    x = logits.to(torch.float32).clone()
    if histories is not None:
        for i in range(B):
            pen = float(params.repetition_penalty[i])
            if pen == 1.0 or len(histories[i]) == 0:
                continue
            uid = torch.as_tensor(np.asarray(histories[i], dtype=np.int64)).unique()
            v = x[i, uid]
            x[i, uid] = torch.where(v > 0, v / pen, v * pen)
    greedy = [bool(params.greedy[i]) or float(params.temperature[i]) == 0.0 for i in range(B)]
    if all(greedy):
        return x.argmax(dim=-1).numpy()
    out = np.empty(B, dtype=np.int64)
    for i in range(B):
        logit = x[i]
        if greedy[i]:
            out[i] = int(logit.argmax())
            continue
        T = float(params.temperature[i])
        if T != 1.0 and T > 0:
            logit = logit / T
        k = int(params.top_k[i])
        if k > 0:
            logit = top_k_filter(logit, k)
        p = float(params.top_p[i])
        if 0.0 < p < 1.0:
            sl, si = logit.sort(descending=True)
            cp = F.softmax(sl, dim=-1).cumsum(dim=-1)
            remove = cp - F.softmax(sl, dim=-1) > p
            sl = sl.masked_fill(remove, float("-inf"))
            logit = logit.scatter(0, si, sl)
        probs = F.softmax(logit, dim=-1)
        out[i] = int(torch.multinomial(probs.unsqueeze(0), 1, generator=generator).squeeze())
    return out
