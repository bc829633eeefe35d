"""Vocabulary-sharded sampling on one GPU: G shards run one after another
through the local stage (fg_sample_candidates), their candidates are merged
per row and drawn with fg_sample; the ids must equal the oracle's on the
full rows (and the unsharded kernel's) on every row the oracle does not flag."""
import numpy as np
import pytest
import torch

from flashgen_b200 import _lib
from flashgen_b200.sampling.sampler import PackedParams, fused_sample
from flashgen_b200.sampling.sharded import Candidates, local_candidates, merge_and_draw, merge_params
from flashgen_b200.workloads import make_workload
from oracle import sampler_oracle as O

pytestmark = pytest.mark.gpu


def _sharded_ids(w, G, cand_max, dev):
    p = w.params
    B, V = w.batch, w.vocab
    packed = PackedParams(p.temperature, p.top_p, p.top_k, p.repetition_penalty, p.presence_penalty,
                          p.frequency_penalty, p.greedy, dev)
    hist = (torch.from_numpy(w.hist_ids).to(dev), torch.from_numpy(w.hist_offsets).to(dev), w.hist_max_len)
    uni = torch.from_numpy(w.uniforms).to(dev)
    logits = w.logits.to(dev)
    edges = [V * g // G for g in range(G + 1)]
    parts = [local_candidates(logits[:, edges[g]:edges[g + 1]].contiguous(), packed, uni, hist, edges[g], V,
                              cand_max) for g in range(G)]
    vals = torch.cat([c.vals for c in parts], dim=1)
    gids = torch.cat([c.gids for c in parts], dim=1)
    st = parts[0].status.clone()
    for c in parts[1:]:
        st |= c.status
    mp = merge_params(p.top_p, p.top_k, p.greedy | (p.temperature == 0), dev)
    ids, status = merge_and_draw(vals, gids, st, mp, uni)
    torch.cuda.synchronize()
    return ids.cpu().numpy(), status.cpu().numpy(), parts


@pytest.mark.parametrize("G", [2, 4, 8])
def test_sharded_matches_oracle(cuda_device, G):
    w = make_workload(4, batch=24, seed=G)
    ids, status, _ = _sharded_ids(w, G, 320, cuda_device)
    assert not (status & _lib.FG_ROW_ERROR_MASK).any(), status
    res = O.sample_rows(w.logits, w.params, w.histories(), w.uniforms)
    ok = (ids == res.ids) | res.near_u | res.near_p
    assert ok.all(), (np.nonzero(~ok)[0], ids[~ok], res.ids[~ok])
    # and the unsharded kernel on the full rows
    p = w.params
    packed = PackedParams(p.temperature, p.top_p, p.top_k, p.repetition_penalty, p.presence_penalty,
                          p.frequency_penalty, p.greedy, cuda_device)
    hist = (torch.from_numpy(w.hist_ids).to(cuda_device), torch.from_numpy(w.hist_offsets).to(cuda_device),
            w.hist_max_len)
    full = fused_sample(w.logits.to(cuda_device), packed, torch.from_numpy(w.uniforms).to(cuda_device), hist)
    full = full.cpu().numpy()
    assert ((ids == full) | res.near_u | res.near_p).all()


def test_sharded_candidates_are_the_shard_topk(cuda_device):
    """Each shard's candidate set is exactly its elements at or above its k-th
    largest penalised, tempered value (ties included)."""
    G = 4
    w = make_workload(4, batch=8, seed=3)
    _, _, parts = _sharded_ids(w, G, 320, cuda_device)
    V = w.vocab
    edges = [V * g // G for g in range(G + 1)]
    from tests.test_gpu_parity import _penalised_y
    y = _penalised_y(w, cuda_device).cpu()
    for g, c in enumerate(parts):
        ys = y[:, edges[g]:edges[g + 1]]
        for r in range(w.batch):
            k = int(w.params.top_k[r])
            thr = torch.topk(ys[r], k).values[-1]
            want = (torch.nonzero(ys[r] >= thr)[:, 0] + edges[g]).numpy()
            n = int(c.counts[r])
            got = np.sort(c.gids[r, :n].cpu().numpy())
            np.testing.assert_array_equal(got, want)
            np.testing.assert_array_equal(np.sort(c.vals[r, :n].cpu().numpy()),
                                          np.sort(ys[r][want - edges[g]].numpy()))


def test_sharded_greedy_rows(cuda_device):
    w = make_workload(4, batch=8, seed=5)
    w.params.greedy[:4] = True
    ids, status, _ = _sharded_ids(w, 4, 320, cuda_device)
    res = O.sample_rows(w.logits, w.params, w.histories(), w.uniforms)
    assert not (status & _lib.FG_ROW_ERROR_MASK).any()
    ok = (ids == res.ids) | res.near_u | res.near_p
    assert ok.all(), (np.nonzero(~ok)[0], ids[~ok], res.ids[~ok])


def test_sharded_truncation_is_reported(cuda_device):
    w = make_workload(4, batch=4, seed=6)
    _, status, _ = _sharded_ids(w, 2, 64, cuda_device)   # cand_max below top_k = 256
    assert (status & _lib.FG_ROW_CAND_TRUNC).all()
