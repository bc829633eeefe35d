"""Parity of the batch path (history prep, stream, decide, and the 16-bit
deep-nucleus finish) with the CPU oracle. Batches here are large enough that
fg_sample takes the batch path rather than one cluster per row, and no
kept-set probabilities are requested (a call that wants them is sampled by the
cluster kernel), so the ids compared are the batch path's own.

Token ids must be identical on every row the oracle does not flag as within
1e-6 of a CDF or top-p boundary (reference: flashgen/sampling/sampler.py:57-169,
draw order of csrc/runtime/pipeline.cpp:311-340)."""
import numpy as np
import pytest
import torch

from flashgen_b200 import _lib
from flashgen_b200.workloads import BatchParams, Workload, make_workload
from oracle import sampler_oracle as O
from tests.gpu_helpers import compare, run_kernel

pytestmark = pytest.mark.gpu


def _oracle(w):
    return O.sample_rows(w.logits, w.params, w.histories(), w.uniforms, stable=True)


@pytest.mark.parametrize("cfg,batch", [(2, 256), (3, 256), (4, 192)])
def test_batch_path_configs(cuda_device, cfg, batch):
    w = make_workload(cfg, batch=batch, seed=21)
    ids, status, _ = run_kernel(w, probs=False)
    stats = compare(w, _oracle(w), ids, status, None)
    print(f"cfg{cfg}", stats)
    # the batch path decided most rows itself
    assert stats["general_path"] <= batch // 4, stats


def test_config3_every_row(cuda_device):
    """Configuration 3 at its full size: every one of the 1024 rows against the
    oracle, with the flagged-row and tie counts printed."""
    w = make_workload(3, seed=11)
    ids, status, _ = run_kernel(w, probs=False)
    res = _oracle(w)
    stats = compare(w, res, ids, status, None)
    stats["tie_at_cut"] = int(res.tie_at_cut.sum())
    print("cfg3 full", stats)


def _deep_workload(dtype, B, V, hist, seed, top_ps=(0.85, 0.88, 0.9, 0.92, 0.95)):
    rng = np.random.default_rng(seed)
    x = rng.standard_normal((B, V), dtype=np.float32)
    for r in range(B):
        x[r, rng.choice(V, V // 100, replace=False)] += 6.0
    p = BatchParams.uniform(B)
    p.temperature[:] = rng.uniform(0.6, 1.2, B).astype(np.float32)
    p.top_k[:] = 0
    p.top_p[:] = rng.choice(np.array(top_ps, np.float32), B)
    rows = [np.zeros(0, np.int32)] * B
    if hist:
        p.repetition_penalty[:] = rng.uniform(1.0, 1.3, B).astype(np.float32)
        p.presence_penalty[:] = rng.uniform(0.0, 0.4, B).astype(np.float32)
        p.frequency_penalty[:] = rng.uniform(0.0, 0.2, B).astype(np.float32)
        rows = [((rng.zipf(1.1, 512) - 1) % V).astype(np.int32) for _ in range(B)]
    offs = np.zeros(B + 1, np.int64)
    offs[1:] = np.cumsum([len(h) for h in rows])
    ids = np.concatenate(rows).astype(np.int32) if offs[-1] else np.zeros(0, np.int32)
    u = rng.random(B, dtype=np.float32)
    return Workload(0, "deep", torch.from_numpy(x).to(dtype), p, ids, offs, u)


@pytest.mark.parametrize("hist", [False, True])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_deep_nucleus_16bit(cuda_device, dtype, hist):
    """Top-p cuts and draws below the candidate set: the 16-bit finish counts
    the row's values below the candidates' threshold and walks them."""
    w = _deep_workload(dtype, 192, 32000, hist, seed=5 + int(hist))
    ids, status, _ = run_kernel(w, probs=False)
    stats = compare(w, _oracle(w), ids, status, None)
    print(dtype, hist, stats)
    # the deep rows were finished on the batch path, not handed to the cluster kernel
    assert stats["general_path"] <= w.batch // 8, stats


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_deep_nucleus_16bit_tail(cuda_device, dtype):
    """Nuclei reaching the negative values of the row (top-p near 1) and rows
    with top-p 1 (a draw over the whole row)."""
    w = _deep_workload(dtype, 192, 32000, True, seed=9, top_ps=(0.97, 0.99, 0.995, 0.999, 1.0))
    ids, status, _ = run_kernel(w, probs=False)
    stats = compare(w, _oracle(w), ids, status, None)
    print(dtype, "tail", stats)


def test_pybind_sample_matches_oracle(cuda_device):
    """fg_sample through the PyBind11 module (_C.sample, GIL released) on
    configuration 2 rows, against the oracle."""
    import importlib

    from flashgen_b200 import build as _build
    from flashgen_b200.sampling.sampler import PackedParams, workspace_for

    _build.build_bindings()
    C = importlib.import_module("flashgen_b200._C")
    dev = cuda_device
    w = make_workload(2, batch=96, seed=4)
    p = w.params
    packed = PackedParams(p.temperature, p.top_p, p.top_k, p.repetition_penalty, p.presence_penalty,
                          p.frequency_penalty, p.greedy, dev)
    lg = w.logits.to(dev)
    u = torch.from_numpy(w.uniforms).to(dev)
    hid, hoff = torch.from_numpy(w.hist_ids).to(dev), torch.from_numpy(w.hist_offsets).to(dev)
    out = torch.empty(w.batch, dtype=torch.int64, device=dev)
    status = torch.empty(w.batch, dtype=torch.int32, device=dev)
    stream = torch.cuda.current_stream(dev)
    ws = workspace_for(dev, stream, C.workspace_size(w.batch, w.vocab, C.DTYPE_F16, w.hist_max_len))
    f = packed.f32
    C.sample(lg.data_ptr(), C.DTYPE_F16, w.batch, w.vocab, w.vocab, f[0].data_ptr(), f[1].data_ptr(),
             packed.top_k.data_ptr(), u.data_ptr(), out.data_ptr(), status=status.data_ptr(),
             repetition_penalty=f[2].data_ptr(), presence_penalty=f[3].data_ptr(),
             frequency_penalty=f[4].data_ptr(), greedy=packed.greedy.data_ptr(), hist_ids=hid.data_ptr(),
             hist_offsets=hoff.data_ptr(), hist_max_len=w.hist_max_len, workspace=ws.data_ptr(),
             workspace_bytes=ws.numel() * 4, stream=stream.cuda_stream)
    torch.cuda.synchronize()
    compare(w, _oracle(w), out.cpu().numpy(), status.cpu().numpy(), None)


def test_decode_batch_steps(cuda_device):
    """Several decode steps through DecodeBatch (device-resident histories,
    one fg_sample call per step, ids appended on the device): every step's ids
    against the oracle with the histories as they stood before that step."""
    from flashgen_b200.core.config import SamplingParams
    from flashgen_b200.sampling.decode import DecodeBatch

    rng = np.random.default_rng(12)
    B, V, steps = 64, 32000, 4
    params = [SamplingParams(temperature=float(rng.uniform(0.6, 1.1)), top_p=float(rng.uniform(0.8, 0.99)),
                             top_k=int(rng.choice([-1, 20, 100])), repetition_penalty=float(rng.uniform(1.0, 1.3)),
                             presence_penalty=float(rng.uniform(0, 0.3)), frequency_penalty=float(rng.uniform(0, 0.2)))
              for _ in range(B)]
    dec = DecodeBatch(params, vocab=V, capacity=256, device=cuda_device)
    for r in range(B):
        dec.set_history(r, rng.integers(0, V, int(rng.integers(0, 200))).tolist())
    bp = BatchParams(*(np.array([getattr(p, f) for p in params], dtype=dt) for f, dt in (
        ("temperature", np.float32), ("top_p", np.float32), ("top_k", np.int32), ("repetition_penalty", np.float32),
        ("presence_penalty", np.float32), ("frequency_penalty", np.float32), ("greedy", bool))))
    for s in range(steps):
        x = rng.standard_normal((B, V), dtype=np.float32)
        x[:, rng.integers(0, V, 40)] += 5.0
        logits = torch.from_numpy(x).to(torch.float16)
        u = rng.random(B, dtype=np.float32)
        before = dec.histories()
        ids = dec.step(logits.to(cuda_device), uniforms=torch.from_numpy(u).to(cuda_device))
        torch.cuda.synchronize()
        got = ids.cpu().numpy()
        offs = np.zeros(B + 1, np.int64)
        offs[1:] = np.cumsum([len(h) for h in before])
        hid = np.concatenate([np.asarray(h, np.int32) for h in before]) if offs[-1] else np.zeros(0, np.int32)
        w = Workload(0, "decode", logits, bp, hid, offs, u)
        compare(w, _oracle(w), got, dec.status.cpu().numpy(), None)
        after = dec.histories()
        assert all(a == b + [int(i)] for a, b, i in zip(after, before, got))
