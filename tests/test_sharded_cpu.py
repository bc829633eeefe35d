"""Host logic of vocabulary-sharded sampling with world size 2 on CPU (gloo).

Each rank holds half the columns of every row. The local stage is restated
here with torch ops (what fg_sample_candidates computes on a GPU shard), the
exchange is flashgen_b200.sampling.sharded.exchange over gloo, and the merge
is the oracle run on the id-sorted union of the candidates. The drawn ids must
equal the oracle's on the full rows (unflagged rows).
"""
import os
import socket
import tempfile

import numpy as np
import pytest
import torch

from flashgen_b200.sampling.sharded import INT32_MAX, Candidates, exchange, sharded_step, sort_by_id
from flashgen_b200.workloads import BatchParams, Workload
from oracle import sampler_oracle as O

B, V, K, CMAX = 6, 2000, 16, 24


def _workload():
    rng = np.random.default_rng(7)
    x = torch.from_numpy(3.0 * rng.standard_normal((B, V), dtype=np.float32))
    p = BatchParams.uniform(B, temperature=1.0, top_p=0.9, top_k=K, rep=1.05)
    p.temperature[1] = 0.7
    p.greedy[2] = True
    hist = [rng.integers(0, V, 64).astype(np.int32) for _ in range(B)]
    offs = np.zeros(B + 1, np.int64)
    offs[1:] = np.cumsum([len(h) for h in hist])
    u = rng.random(B, dtype=np.float32)
    return Workload(4, "sharded-cpu", x, p, np.concatenate(hist), offs, u)


def _local_stage(w, g, G):
    """Shard g's top-k sets, as fg_sample_candidates computes them."""
    lo, hi = V * g // G, V * (g + 1) // G
    p = w.params
    x = w.logits[:, lo:hi].clone().float()
    vals = torch.full((B, CMAX), float("-inf"))
    gids = torch.full((B, CMAX), INT32_MAX, dtype=torch.int32)
    counts = torch.zeros(B, dtype=torch.int32)
    for r, h in enumerate(w.histories()):
        cols = np.unique(h[(h >= lo) & (h < hi)]) - lo
        xc = x[r, cols]
        x[r, cols] = torch.where(xc > 0, xc / float(p.repetition_penalty[r]), xc * float(p.repetition_penalty[r]))
        if p.greedy[r] or p.temperature[r] == 0:
            j = int(torch.argmax(x[r]))
            vals[r, 0], gids[r, 0], counts[r] = x[r, j], j + lo, 1
            continue
        y = x[r] / float(p.temperature[r]) if p.temperature[r] != 1.0 else x[r]
        thr = torch.topk(y, int(p.top_k[r])).values[-1]
        sel = torch.nonzero(y >= thr)[:, 0]
        n = len(sel)
        vals[r, :n], gids[r, :n], counts[r] = y[sel], (sel + lo).to(torch.int32), n
    return Candidates(vals, gids, counts, torch.zeros(B, dtype=torch.int32))


def _merge(w, own, rank, G):
    Bo = B // G
    rows = slice(rank * Bo, (rank + 1) * Bo)
    v, gsorted = sort_by_id(own.vals, own.gids)
    p = w.params.slice(rows.start, rows.stop)
    mp = BatchParams(np.ones(Bo, np.float32), p.top_p, p.top_k, np.ones(Bo, np.float32),
                     np.zeros(Bo, np.float32), np.zeros(Bo, np.float32), p.greedy | (p.temperature == 0))
    res = O.sample_rows(v, mp, None, w.uniforms[rows])
    ids = torch.gather(gsorted, 1, torch.from_numpy(res.ids)[:, None].long())[:, 0].long()
    return ids, own.status


def _worker(rank, world, port, out_path):
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        w = _workload()
        ids, _ = sharded_step(lambda: _local_stage(w, rank, world), lambda own: _merge(w, own, rank, world),
                              world, gather_ids=True)
        if rank == 0:
            np.save(out_path, ids.numpy())
    finally:
        dist.destroy_process_group()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_sharded_two_ranks_gloo():
    import torch.multiprocessing as mp
    with tempfile.TemporaryDirectory() as d:
        out = os.path.join(d, "ids.npy")
        mp.spawn(_worker, args=(2, _free_port(), out), nprocs=2, join=True)
        ids = np.load(out)
    w = _workload()
    res = O.sample_rows(w.logits, w.params, w.histories(), w.uniforms)
    ok = (ids == res.ids) | res.near_u | res.near_p
    assert ok.all(), (np.nonzero(~ok)[0], ids[~ok], res.ids[~ok])


def test_exchange_layout_single_rank():
    """World size 1: the step is the local stage followed by the merge."""
    w = _workload()
    c = _local_stage(w, 0, 1)
    ids, _ = sharded_step(lambda: c, lambda own: _merge(w, own, 0, 1), 1)
    res = O.sample_rows(w.logits, w.params, w.histories(), w.uniforms)
    ok = (ids.numpy() == res.ids) | res.near_u | res.near_p
    assert ok.all()
