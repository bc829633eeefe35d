"""Shared helpers of the GPU tests: run the fused kernel through the C ABI on a
workload and compare it with the CPU oracle."""
from __future__ import annotations

import numpy as np
import torch

from flashgen_b200 import _lib
from flashgen_b200.sampling.sampler import PackedParams, fused_sample

# Kept-set probabilities: |p_gpu - p_oracle| <= REL_TOL * p_oracle + ABS_TOL.
# REL_TOL is the north-star tolerance (1e-5 relative in fp32). ABS_TOL covers
# masses so small that the kernel's fixed-point accumulator (2^-S of the row
# maximum's mass, S = 62 - ceil(log2 V)) rounds them, far below anything a
# draw can hit.
REL_TOL = 1e-5
ABS_TOL = 1e-12


def run_kernel(w, device="cuda", probs=False, hist=True):
    B, V = w.batch, w.vocab
    logits = w.logits.to(device)
    p = w.params
    packed = PackedParams(p.temperature, p.top_p, p.top_k, p.repetition_penalty, p.presence_penalty,
                          p.frequency_penalty, p.greedy, device)
    h = None
    if hist and w.hist_ids.size > 0:
        h = (torch.from_numpy(w.hist_ids).to(device), torch.from_numpy(w.hist_offsets).to(device),
             w.hist_max_len)
    u = torch.from_numpy(w.uniforms).to(device)
    status = torch.full((B,), -1, dtype=torch.int32, device=device)
    pr = torch.empty(B, V, dtype=torch.float32, device=device) if probs else None
    out = fused_sample(logits, packed, u, h, status=status, probs=pr)
    torch.cuda.synchronize()
    return (out.cpu().numpy(), status.cpu().numpy(), None if pr is None else pr.cpu().numpy())


def compare(w, res, ids, status, probs, check_probs=True):
    """Returns a dict of counts; asserts exactness on unflagged rows."""
    B = w.batch
    # status bits row by row: the rows on which the reference raises carry an
    # error bit and no id; every other row is clean
    err_bits = (status & _lib.FG_ROW_ERROR_MASK) != 0
    wrong = err_bits != res.error
    assert not wrong.any(), (f"status disagrees with the oracle on rows {np.nonzero(wrong)[0][:10]}: "
                             f"status {status[wrong][:10]}, oracle error {res.error[wrong][:10]}")
    assert (ids[res.error] == -1).all(), ids[res.error][:10]
    flagged = res.near_u | res.near_p
    mism = ids != res.ids
    bad = mism & ~flagged
    assert not bad.any(), (f"ids differ on unflagged rows {np.nonzero(bad)[0][:10]}: "
                           f"gpu {ids[bad][:10]} oracle {res.ids[bad][:10]}")
    if probs is not None and check_probs:
        for r in range(B):
            if res.near_p[r] or res.error[r]:
                continue
            kid, kp = res.kept_ids[r], res.kept_probs[r].astype(np.float64)
            row = probs[r].astype(np.float64)
            got = row[kid]
            err = np.abs(got - kp) - (REL_TOL * kp + ABS_TOL)
            assert (err <= 0).all(), (r, kid[np.argmax(err)], got[np.argmax(err)], kp[np.argmax(err)])
            outside = np.ones(w.vocab, bool)
            outside[kid] = False
            assert (row[outside] == 0).all(), (r, np.nonzero(row * outside)[0][:5])
    return {"rows": B, "flagged": int(flagged.sum()), "flagged_mismatch": int((mism & flagged).sum()),
            "general_path": int(((status & _lib.FG_ROW_GENERAL_PATH) != 0).sum())}
