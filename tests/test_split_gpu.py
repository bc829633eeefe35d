"""Small batches of fg_sample: a batch that would leave most SMs idle with one
CTA per row is sampled by the cluster kernel, one thread-block cluster per row
(fg_sample_set_split picks it: 0 never, 1 when it pays, 2 always). Token ids
must equal the oracle's on every row it does not flag, and the cluster
kernel's ids must equal the batch path's on the same rows."""
import numpy as np
import pytest
import torch

from flashgen_b200 import _lib
from flashgen_b200.workloads import BatchParams, Workload, make_workload
from oracle import sampler_oracle as O
from tests.gpu_helpers import compare, run_kernel

pytestmark = pytest.mark.gpu


@pytest.fixture
def split_mode():
    lib = _lib.load()

    def set_mode(m):
        assert lib.fg_sample_set_split(m) == _lib.FG_OK

    yield set_mode
    set_mode(1)


def _both(w, split_mode):
    split_mode(0)
    ids0, st0, _ = run_kernel(w)
    split_mode(2)
    ids1, st1, _ = run_kernel(w)
    res = O.sample_rows(w.logits, w.params, w.histories(), w.uniforms, stable=True)
    stats = compare(w, res, ids1, st1, None)
    flagged = res.near_u | res.near_p
    assert ((ids1 == ids0) | flagged).all(), (np.nonzero((ids1 != ids0) & ~flagged)[0], ids1, ids0)
    assert ((st1 & _lib.FG_ROW_ERROR_MASK) == (st0 & _lib.FG_ROW_ERROR_MASK)).all(), (st1, st0)
    return stats


def test_split_latency_config(cuda_device, split_mode):
    # configuration 5: one fp32 row of 256000 columns, top-p only, 4096-id history
    for seed in range(3):
        print(_both(make_workload(5, seed=seed), split_mode))


@pytest.mark.parametrize("cfg,batch", [(2, 4), (3, 6), (4, 2)])
def test_split_mixed_configs(cuda_device, split_mode, cfg, batch):
    # penalties (all three kinds), greedy rows, top-k 20..1000 (sets larger
    # than a shard's 256 candidates go to the fixup), top-p with top-k off
    print(_both(make_workload(cfg, batch=batch, seed=cfg), split_mode))


def test_split_edge_rows(cuda_device, split_mode):
    g = torch.Generator().manual_seed(5)
    B, V = 6, 8192
    x = torch.randn(B, V, generator=g)
    x[1] = 0.25                            # all equal: the nucleus is most of the row
    x[2, 100:4000] = float("-inf")         # masked columns across shards
    x[3] = torch.sort(x[3], descending=True).values
    x[4, 7] = 30.0                         # one outlier
    p = BatchParams.uniform(B, temperature=0.9, top_p=0.9, top_k=-1)
    p.top_k[:] = [0, 0, 40, 0, 0, 300]
    p.top_p[:] = [0.99, 0.5, 0.9, 0.95, 0.9, 1.0]
    p.greedy[5] = False
    rng = np.random.default_rng(1)
    u = rng.random(B, dtype=np.float32)
    offs = np.zeros(B + 1, np.int64)
    w = Workload(0, "split-edge", x, p, np.zeros(0, np.int32), offs, u)
    print(_both(w, split_mode))


def test_split_greedy_and_nan(cuda_device, split_mode):
    g = torch.Generator().manual_seed(9)
    B, V = 4, 16384
    x = torch.randn(B, V, generator=g).to(torch.bfloat16)
    x[0, 9000] = 5.0
    x[0, 12000] = 5.0                      # tie for the maximum in two shards: first one wins
    x[2, 333] = float("nan")
    p = BatchParams.uniform(B, temperature=0.0, top_p=1.0, top_k=-1)
    p.temperature[1] = 0.8
    p.temperature[2] = 0.8
    u = np.random.default_rng(2).random(B, dtype=np.float32)
    w = Workload(0, "split-greedy", x, p, np.zeros(0, np.int32), np.zeros(B + 1, np.int64), u)
    split_mode(2)
    ids, status, _ = run_kernel(w)
    assert ids[0] == 9000
    assert status[2] & _lib.FG_ROW_NAN and ids[2] == -1
    print(_both(w, split_mode))
