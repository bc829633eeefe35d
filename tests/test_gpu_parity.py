"""Parity of the sm_100a sampler with the CPU oracle (pinned to FlashGen's own
Sampler by tests/golden). Token ids must be identical on every row the oracle
does not flag as within 1e-6 of a CDF or top-p boundary; kept-set
probabilities must agree within 1e-5 relative (gpu_helpers.REL_TOL)."""
import os

import numpy as np
import pytest
import torch

from flashgen_b200 import _lib
from flashgen_b200.workloads import BatchParams, Workload, make_workload
from oracle import sampler_oracle as O
from tests.golden.make_golden import CASES
from tests.gpu_helpers import compare, run_kernel

pytestmark = pytest.mark.gpu
GOLDEN = os.path.join(os.path.dirname(__file__), "golden")


@pytest.mark.parametrize("cfg,batch", CASES)
def test_golden_configs(cuda_device, cfg, batch):
    w = make_workload(cfg, batch=batch)
    g = np.load(os.path.join(GOLDEN, f"golden_cfg{cfg}.npz"))
    ids, status, probs = run_kernel(w, probs=True)
    res = O.sample_rows(w.logits, w.params, w.histories(), w.uniforms, stable=True)
    np.testing.assert_array_equal(res.ids, g["ids"])
    stats = compare(w, res, ids, status, probs)
    print(f"cfg{cfg}", stats)


def _workload(logits, params, hist=None, uniforms=None, seed=0):
    B, V = logits.shape
    rng = np.random.default_rng(seed)
    rows = hist if hist is not None else [np.zeros(0, np.int32)] * B
    offs = np.zeros(B + 1, np.int64)
    offs[1:] = np.cumsum([len(h) for h in rows])
    ids = np.concatenate([np.asarray(h, np.int32) for h in rows]) if offs[-1] else np.zeros(0, np.int32)
    u = uniforms if uniforms is not None else rng.random(B, dtype=np.float32)
    return Workload(0, "edge", logits, params, ids, offs, u)


def _check(w, probs=True):
    ids, status, pr = run_kernel(w, probs=probs)
    res = O.sample_rows(w.logits, w.params, w.histories(), w.uniforms, stable=True)
    return compare(w, res, ids, status, pr), ids, status


@pytest.mark.parametrize("V", [1, 2, 7, 8, 9, 31, 33, 257, 4095, 4097, 12289, 50257])
@pytest.mark.parametrize("dtype", [torch.float32, torch.float16, torch.bfloat16])
def test_small_vocab_shapes(cuda_device, V, dtype):
    g = torch.Generator().manual_seed(V)
    B = 6
    logits = (torch.randn(B, V, generator=g) * 2).to(dtype)
    p = BatchParams.uniform(B, temperature=0.9, top_p=0.8, top_k=-1)
    p.top_k[:] = [-1, 1, 5, 0, 3, -1]
    p.top_p[:] = [0.8, 0.5, 1.0, 0.95, 0.3, 1.0]
    p.greedy[5] = True
    _check(_workload(logits, p, seed=V))


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_unaligned_rows(cuda_device, dtype):
    # row stride not a multiple of 16 bytes: ragged head/tail on every row
    g = torch.Generator().manual_seed(3)
    B, V, S = 5, 9001, 9003
    big = (torch.randn(B, S, generator=g) * 3).to(dtype)
    logits = big[:, 1:V + 1]
    p = BatchParams.uniform(B, temperature=0.7, top_p=0.9, top_k=40)
    w = _workload(logits.contiguous(), p)
    # run through the strided view directly
    from flashgen_b200.sampling.sampler import PackedParams, fused_sample
    dev = "cuda"
    lg = big.to(dev)[:, 1:V + 1]
    packed = PackedParams(p.temperature, p.top_p, p.top_k, p.repetition_penalty, p.presence_penalty,
                          p.frequency_penalty, p.greedy, dev)
    out = fused_sample(lg, packed, torch.from_numpy(w.uniforms).to(dev))
    res = O.sample_rows(w.logits, w.params, None, w.uniforms)
    flagged = res.near_u | res.near_p
    assert ((out.cpu().numpy() == res.ids) | flagged).all()


def test_ties_everywhere(cuda_device):
    # integer-valued logits: long runs of ties at every cut
    g = torch.Generator().manual_seed(11)
    B, V = 8, 20000
    logits = torch.randint(-4, 5, (B, V), generator=g).to(torch.bfloat16)
    p = BatchParams.uniform(B, temperature=1.0, top_p=0.6, top_k=-1)
    p.top_k[:4] = [10, 100, 5000, 3000]
    p.greedy[7] = True
    _check(_workload(logits, p))


def test_all_equal_rows(cuda_device):
    B, V = 4, 30000
    logits = torch.zeros(B, V, dtype=torch.float32)
    p = BatchParams.uniform(B, temperature=0.5, top_p=0.25, top_k=-1)
    p.top_k[1] = 7
    p.greedy[2] = True
    p.top_p[3] = 1.0
    _check(_workload(logits, p, uniforms=np.array([0.1, 0.5, 0.9, 0.999], np.float32)))


def test_masked_and_nan_rows(cuda_device):
    B, V = 5, 5000
    g = torch.Generator().manual_seed(5)
    logits = torch.randn(B, V, generator=g)
    logits[0, :4990] = float("-inf")         # mostly masked, sampling still valid
    logits[1, :] = float("-inf")             # fully masked -> error status
    logits[2, 17] = float("nan")             # NaN in a sampling row -> error status
    logits[3, 99] = float("nan")             # NaN in a greedy row -> first NaN (torch.argmax)
    logits[4, 1234] = float("inf")           # +inf in a sampling row -> error status
    p = BatchParams.uniform(B, temperature=0.8, top_p=0.9)
    p.greedy[3] = True
    w = _workload(logits, p)
    ids, status, _ = run_kernel(w)
    assert status[0] & _lib.FG_ROW_ERROR_MASK == 0 and ids[0] >= 4990
    assert status[1] & _lib.FG_ROW_ALL_MASKED and ids[1] == -1
    assert status[2] & _lib.FG_ROW_NAN and ids[2] == -1
    assert ids[3] == 99
    assert status[4] & _lib.FG_ROW_POS_INF and ids[4] == -1


def test_large_top_k_general_path(cuda_device):
    g = torch.Generator().manual_seed(7)
    B, V = 4, 60000
    logits = torch.randn(B, V, generator=g).to(torch.float16)
    p = BatchParams.uniform(B, temperature=1.3, top_p=0.97, top_k=5000)
    p.top_k[1] = 60000
    p.top_p[2] = 1.0
    stats, ids, status = _check(_workload(logits, p))
    assert (status & _lib.FG_ROW_GENERAL_PATH).all()


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_sorted_rows(cuda_device, dtype):
    # The candidate filter starts from a sample of the row's first tile. On
    # rows sorted in descending order that sample holds the row's largest
    # values, so a row with a large K keeps fewer than K elements and must
    # take the whole-row select; ascending rows start from the row's smallest
    # values.
    g = torch.Generator().manual_seed(11)
    B, V = 8, 128256
    x = torch.randn(B, V, generator=g)
    x[:4] = torch.sort(x[:4], dim=1, descending=True).values
    x[4:] = torch.sort(x[4:], dim=1).values
    p = BatchParams.uniform(B, temperature=0.9, top_p=0.95, top_k=-1)
    p.top_k[:] = [20, 1000, 0, 100, 20, 1000, 0, 100]
    stats, ids, status = _check(_workload(x.to(dtype), p, seed=3))
    assert status[1] & _lib.FG_ROW_GENERAL_PATH


def test_penalties_all_kinds(cuda_device):
    rng = np.random.default_rng(2)
    B, V = 16, 40000
    logits = torch.from_numpy(rng.standard_normal((B, V), dtype=np.float32) * 2).to(torch.bfloat16)
    p = BatchParams.uniform(B, temperature=0.8, top_p=0.9, top_k=50, rep=1.3, presence=0.5, frequency=0.3)
    p.repetition_penalty[::3] = 0.8          # < 1 raises repeated tokens
    p.greedy[5] = True
    hist = [rng.integers(0, 300 + 500 * r, 200 + 37 * r).astype(np.int32) for r in range(B)]
    hist[3] = np.zeros(0, np.int32)
    _check(_workload(logits, p, hist=hist))


def test_bad_inputs_status(cuda_device):
    B, V = 3, 1000
    logits = torch.randn(B, V)
    p = BatchParams.uniform(B, temperature=1.0, top_p=0.9)
    p.top_p[1] = 1.5                          # invalid
    hist = [np.array([5, 2000], np.int32), np.zeros(0, np.int32), np.zeros(0, np.int32)]
    w = _workload(logits, p, hist=hist, uniforms=np.array([0.5, 0.5, 1.0], np.float32))
    p.repetition_penalty[:] = 1.1
    ids, status, _ = run_kernel(w)
    assert status[0] & _lib.FG_ROW_BAD_HISTORY and ids[0] >= 0
    assert status[1] & _lib.FG_ROW_BAD_PARAM and ids[1] == -1
    assert status[2] & _lib.FG_ROW_BAD_UNIFORM and ids[2] == -1


def test_deterministic(cuda_device):
    w = make_workload(3, batch=64, seed=4)
    a = run_kernel(w)[0]
    b = run_kernel(w)[0]
    np.testing.assert_array_equal(a, b)


def test_sampler_api(cuda_device):
    from flashgen_b200 import Sampler, SamplingParams
    w = make_workload(2, batch=32)
    s = Sampler()
    params = [SamplingParams(temperature=0.7, top_k=50, top_p=0.95, repetition_penalty=1.1,
                             presence_penalty=0.2, frequency_penalty=0.1) for _ in range(32)]
    ids = s.sample(w.logits.cuda(), params, token_histories=[list(h) for h in w.histories()],
                   uniforms=torch.from_numpy(w.uniforms)).cpu().numpy()
    res = O.sample_rows(w.logits, w.params, w.histories(), w.uniforms)
    assert ((ids == res.ids) | res.near_u | res.near_p).all()
    one = s._sample_one(w.logits[0].cuda(), params[0], token_histories=[list(w.histories()[0])],
                        uniforms=torch.from_numpy(w.uniforms[:1]))
    assert one.dim() == 0 and int(one) == ids[0]
    gp = SamplingParams(greedy=True)
    g = s.sample_batch(w.logits.cuda(), gp)
    assert torch.equal(g.cpu(), w.logits.float().argmax(-1))
    bad = w.logits[:2].cuda().float()
    bad[0, 3] = float("nan")
    with pytest.raises(RuntimeError):
        s.sample(bad, [SamplingParams()] * 2)


def test_argmax_and_rep_penalty(cuda_device):
    from flashgen_b200 import Sampler
    g = torch.Generator().manual_seed(9)
    for dt in (torch.float32, torch.float16, torch.bfloat16):
        x = torch.randint(-3, 4, (7, 3001), generator=g).to(dt)
        x[2, 50] = float("nan")
        got = Sampler.argmax(x.cuda()).cpu()
        assert torch.equal(got, x.argmax(-1)), dt
        hist = [[1, 2, 2, 5], [], [7] * 10, list(range(0, 3000, 7)), [0], [3000], [4, 4]]
        ref = O.repetition_penalty_inplace(x.clone(), hist, [1.3] * 7)
        out = Sampler().apply_repetition_penalty(x.cuda(), hist, 1.3).cpu()
        iv = torch.int32 if dt == torch.float32 else torch.int16
        assert torch.equal(out.view(iv), ref.view(iv)), dt


@pytest.mark.parametrize("seed", [1, 2, 3])
def test_unaligned_rows_large_nucleus(cuda_device, seed):
    # rows that start off a 16-byte boundary have ragged columns outside the
    # streamed interior; with a nucleus larger than the candidate target the
    # cut is found by the multi-pass path, which must count every column once
    g = torch.Generator().manual_seed(seed)
    B, V = 6, 20001
    logits = torch.randn(B, V, generator=g).to(torch.float16)
    p = BatchParams.uniform(B, temperature=1.1, top_p=0.9, top_k=-1)
    p.top_p[:] = [0.9, 0.97, 0.5, 0.999, 0.8, 0.95]
    stats, ids, status = _check(_workload(logits, p, seed=seed))
    assert (status & _lib.FG_ROW_GENERAL_PATH).any()


def _penalised_y(w, dev):
    """Penalised, temperature-scaled logits of a workload, with torch ops on the
    GPU (the oracle's chain: repetition on unique ids, then presence/frequency,
    then x / T), for checks at full size."""
    B, V = w.batch, w.vocab
    x = w.logits.to(dev).float()
    p = w.params
    counts = torch.zeros(B, V, dtype=torch.float32, device=dev)
    rows = torch.repeat_interleave(torch.arange(B, device=dev),
                                   torch.from_numpy(np.diff(w.hist_offsets)).to(dev))
    counts.index_put_((rows, torch.from_numpy(w.hist_ids).long().to(dev)),
                      torch.ones(rows.numel(), device=dev), accumulate=True)
    rep = torch.from_numpy(p.repetition_penalty).to(dev)[:, None]
    pres = torch.from_numpy(p.presence_penalty).to(dev)[:, None]
    freq = torch.from_numpy(p.frequency_penalty).to(dev)[:, None]
    seen = counts > 0
    xr = torch.where(x > 0, x / rep, x * rep)
    x = torch.where(seen, xr, x)
    x = torch.where(seen, (x - freq * counts) - pres, x)
    T = torch.from_numpy(p.temperature).to(dev)[:, None]
    return torch.where(T > 0, x / torch.where(T > 0, T, torch.ones_like(T)), x)


def test_full_size_properties(cuda_device):
    """Configuration 3 at its full size (B=1024, V=128256 bf16): size-independent
    properties on every row, and the oracle on a prefix of rows."""
    dev = cuda_device
    w = make_workload(3, seed=11)
    ids, status, _ = run_kernel(w)
    assert not (status & _lib.FG_ROW_ERROR_MASK).any()
    ids2, status2, _ = run_kernel(w)
    np.testing.assert_array_equal(ids, ids2)          # deterministic
    np.testing.assert_array_equal(status, status2)
    y = _penalised_y(w, dev)
    p = w.params
    greedy = (p.temperature == 0) | p.greedy
    # greedy rows: first index of the maximum of the penalised logits
    g_rows = np.nonzero(greedy)[0]
    if len(g_rows):
        want = torch.argmax(y[torch.from_numpy(g_rows).to(dev)], dim=1).cpu().numpy()
        np.testing.assert_array_equal(ids[g_rows], want)
    # top-k rows: the drawn token is at or above the row's k-th largest value
    k_rows = np.nonzero(~greedy & (p.top_k > 0))[0]
    for k in np.unique(p.top_k[k_rows]):
        rr = k_rows[p.top_k[k_rows] == k]
        yr = y[torch.from_numpy(rr).to(dev)]
        kth = torch.topk(yr, int(k), dim=1).values[:, -1]
        got = yr.gather(1, torch.from_numpy(ids[rr]).long().to(dev)[:, None])[:, 0]
        assert bool((got >= kth).all()), rr[(got < kth).cpu().numpy()][:8]
    # every drawn id is a valid column
    assert ((ids >= 0) & (ids < w.vocab)).all()
    # a prefix of the full batch against the oracle
    n = 16
    res = O.sample_rows(w.logits[:n], p.slice(0, n), w.histories()[:n], w.uniforms[:n])
    ok = (ids[:n] == res.ids) | res.near_u | res.near_p
    assert ok.all(), (np.nonzero(~ok)[0], ids[:n][~ok], res.ids[~ok])


def test_full_size_all_greedy_equals_argmax(cuda_device):
    dev = cuda_device
    w = make_workload(3, seed=12)
    w.params.greedy[:] = True
    w.hist_offsets[:] = 0          # no history: greedy is the plain argmax
    w.hist_ids = np.zeros(0, np.int32)
    ids, status, _ = run_kernel(w, hist=False)
    assert not (status & _lib.FG_ROW_ERROR_MASK).any()
    want = torch.argmax(w.logits.to(dev), dim=1).cpu().numpy()
    np.testing.assert_array_equal(ids, want)
    from flashgen_b200.sampling.sampler import Sampler
    np.testing.assert_array_equal(Sampler.argmax(w.logits.to(dev)).cpu().numpy(), want)


def test_host_sampler_back_to_back(cuda_device):
    """Two HostBatchSampler steps with different parameters and uniforms,
    enqueued back to back without a sync in between: each step must see its
    own staging buffers (they are double-buffered), and both results must
    match the oracle."""
    from flashgen_b200.sampling.host import HostBatchSampler
    wa = make_workload(2, batch=64, seed=21)
    wb = make_workload(3, batch=64, seed=22, vocab=32000)
    wb.logits = wb.logits.to(torch.float16)
    hs = HostBatchSampler(64, 32000, torch.float16, max(wa.hist_ids.size, wb.hist_ids.size), cuda_device)
    outs = []
    for w in (wa, wb):
        ids_h = hs.sample(w.logits.pin_memory(), w.params, torch.from_numpy(w.hist_ids).pin_memory(),
                          torch.from_numpy(w.hist_offsets).pin_memory(), w.uniforms, w.hist_max_len)
        outs.append(ids_h)
    torch.cuda.synchronize()
    for w, ids_h in zip((wa, wb), outs):
        res = O.sample_rows(w.logits, w.params, w.histories(), w.uniforms)
        ids = ids_h.numpy()
        assert ((ids == res.ids) | res.near_u | res.near_p).all(), (w.config, ids[:8], res.ids[:8])
