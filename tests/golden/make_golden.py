"""Generate the golden fixtures for the sampling parity tests.

Run where FlashGen's reference sources are importable (they are not on the GPU
box):  ``python tests/golden/make_golden.py /path/to/FlashGen``

For every parity case it
  1. builds the seeded workload (flashgen_b200.workloads),
  2. runs FlashGen's own Sampler functions on it —
     ``apply_repetition_penalty`` (flashgen/sampling/sampler.py:123-147),
     ``_top_k_filter`` (:149-154) and ``_top_p_filter`` (:156-169) — and checks
     that the oracle's restatement with the reference's (unstable) sort gives
     bit-identical filtered logits, and that the oracle's stable variant
     differs only on rows flagged ``tie_at_cut``;
  3. stores the oracle's (stable) outputs: ids, parity flags, kept-set sizes,
     kept-mass checksums and an input checksum, as ``golden_cfg<N>.npz``.
"""
from __future__ import annotations

import hashlib
import json
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)

from flashgen_b200.workloads import make_workload  # noqa: E402
from oracle import sampler_oracle as O  # noqa: E402

# (config, batch) pairs; None = the configuration's own batch
CASES = [(1, None), (2, None), (3, 128), (4, 32), (5, None)]


def input_checksum(w) -> str:
    h = hashlib.sha256()
    lg = w.logits
    raw = lg.view(torch.int16) if lg.element_size() == 2 else lg.view(torch.int32)
    h.update(raw.numpy().tobytes())
    h.update(w.hist_ids.tobytes())
    h.update(w.hist_offsets.tobytes())
    for f in ("temperature", "top_p", "top_k", "repetition_penalty", "presence_penalty",
              "frequency_penalty", "greedy"):
        h.update(np.ascontiguousarray(getattr(w.params, f)).tobytes())
    h.update(w.uniforms.tobytes())
    return h.hexdigest()


def pin_against_reference(w, Sampler) -> dict:
    """Bit-exact comparison of the oracle's restatement with the reference."""
    S = Sampler()
    hist = w.histories()
    x_ref = w.logits.float().clone()
    x_or = w.logits.float().clone()
    for r in range(w.batch):
        S.apply_repetition_penalty(x_ref[r:r + 1], [list(map(int, hist[r]))],
                                   float(w.params.repetition_penalty[r]))
        O.apply_repetition_penalty_row(x_or[r], hist[r], float(w.params.repetition_penalty[r]))
    assert torch.equal(x_ref, x_or), "repetition penalty differs from the reference"
    stats = {"rows": w.batch, "sampled_rows": 0, "topk_rows": 0, "topp_rows": 0,
             "stable_differs": 0, "tie_at_cut": 0}
    for r in range(w.batch):
        O.apply_presence_frequency_row(x_ref[r], hist[r], float(w.params.presence_penalty[r]),
                                       float(w.params.frequency_penalty[r]))
        T = float(w.params.temperature[r])
        if T == 0.0 or bool(w.params.greedy[r]):
            continue
        stats["sampled_rows"] += 1
        y = x_ref[r]
        if T != 1.0 and T > 0:
            y = y / T
        y_o = y.clone()
        k = int(w.params.top_k[r])
        if k > 0:
            stats["topk_rows"] += 1
            y = S._top_k_filter(y, k)
            y_o = O.top_k_filter(y_o, k)
            assert torch.equal(y, y_o), "top-k differs from the reference"
        p = float(w.params.top_p[r])
        if 0.0 < p < 1.0:
            stats["topp_rows"] += 1
            y_ref = S._top_p_filter(y, p)
            y_u, _, _ = O.top_p_filter(y_o, p, stable=False)
            assert torch.equal(y_ref, y_u), "top-p differs from the reference"
            y_s, _, tie = O.top_p_filter(y_o, p, stable=True)
            stats["tie_at_cut"] += int(tie)
            if not torch.equal(y_s, y_ref):
                stats["stable_differs"] += 1
                assert tie, "stable and reference top-p differ on a row without a tie at the cut"
    return stats


def main(ref_root: str) -> None:
    sys.path.insert(0, ref_root)
    from flashgen.sampling.sampler import Sampler  # the reference
    summary = {}
    for cfg, B in CASES:
        w = make_workload(cfg, batch=B)
        stats = pin_against_reference(w, Sampler)
        res = O.sample_rows(w.logits, w.params, w.histories(), w.uniforms, stable=True)
        n_kept = np.array([len(k) for k in res.kept_ids], dtype=np.int64)
        kept_sum = np.array([float(np.sum(p, dtype=np.float64)) for p in res.kept_probs])
        kept_idsum = np.array([int(np.sum(k)) for k in res.kept_ids], dtype=np.int64)
        path = os.path.join(HERE, f"golden_cfg{cfg}.npz")
        np.savez_compressed(path, config=cfg, batch=w.batch, vocab=w.vocab, ids=res.ids,
                            near_u=res.near_u, near_p=res.near_p, tie_at_cut=res.tie_at_cut,
                            greedy=res.greedy, error=res.error, n_kept=n_kept, kept_sum=kept_sum,
                            kept_idsum=kept_idsum, checksum=input_checksum(w))
        stats.update({"flag_near_u": int(res.near_u.sum()), "flag_near_p": int(res.near_p.sum()),
                      "greedy": int(res.greedy.sum()), "max_kept": int(n_kept.max())})
        summary[f"cfg{cfg}"] = stats
        print(cfg, w.batch, w.vocab, stats, flush=True)
    with open(os.path.join(HERE, "pin_summary.json"), "w") as f:
        json.dump(summary, f, indent=1, sort_keys=True)


if __name__ == "__main__":
    ref = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("FLASHGEN_REF")
    if not ref:
        sys.exit("usage: python tests/golden/make_golden.py <path to the FlashGen source tree> "
                 "(or set FLASHGEN_REF)")
    main(ref)
