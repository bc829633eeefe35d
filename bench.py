#!/usr/bin/env python
"""Benchmark of the B200 decode-step sampler.

Metric: sampled rows/s and logits GB/s vs the HBM peak on the
Llama-3 mixed-parameter batch (configuration 3: B=1024, V=128256, bf16, full
penalty / temperature / top-k / top-p / draw chain), plus the p50/p99 step
latency at B=1 (configuration 5: V=256000 fp32).

A step is one ``fg_sample`` call over one batch (its launches: history prep,
stream, decide, the 16-bit deep-row finish and the cluster kernel for rows
handed on). Inputs are seeded synthetic data (flashgen_b200.workloads); two
distinct logits buffers (2 x 263 MB, each larger than the 126 MB L2) alternate
between steps so no step reads the previous step's logits from L2.

With ``--gpus N`` (torchrun, one process per GPU) the B=1024 batch is split
into N row blocks, rank g sampling rows [g*B/N, (g+1)*B/N) (strong scaling,
no collective on the data path); the time is the max over ranks. The same
line also carries weak scaling (every rank samples a full batch) and the
configuration-4 vocabulary-sharded step (local candidates, NCCL all-to-all,
owner merge) at the same N. At N=1 it adds the other configurations' 1-GPU
lines, the B=1 latency over 10k steps rotating over five seeded rows, parity
against the CPU oracle on every row of the timed batch, and the CPU baseline.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl flashgen_b200|reference]
"""
from __future__ import annotations

import argparse
import json
import os
import subprocess
import sys
import threading
import time

import numpy as np
import torch

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

FALLBACK_HBM_GBS = 6650.0


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=2000)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--impl", default="flashgen_b200", choices=["flashgen_b200", "reference"])
    ap.add_argument("--config", type=int, default=3)
    ap.add_argument("--e2e-steps", type=int, default=20)
    ap.add_argument("--latency-steps", type=int, default=10000)
    ap.add_argument("--cpu-seconds", type=float, default=12.0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--batch", type=int, default=0, help="rows of the timed batch (default: the configuration's)")
    ap.add_argument("--only-step", action="store_true",
                    help="time the fg_sample step alone (no other legs): the command the ncu captures use")
    return ap.parse_args()


def measured_peak():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(p) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), "measured"
    except Exception:
        return FALLBACK_HBM_GBS, "fallback"


def ncu_traffic(config: int):
    """DRAM bytes of one fg_sample call (all of its launches) from the ncu
    capture committed as profiles/traffic_cfg<config>.json (the command that
    made it is in the file), or None."""
    p = os.path.join(ROOT, "profiles", f"traffic_cfg{config}.json")
    try:
        with open(p) as f:
            d = json.load(f)
        return float(d["dram_bytes_per_call"]), d.get("kernels")
    except (OSError, ValueError, KeyError):
        return None, None


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled every 100 ms in a thread."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device_index: int):
        self.samples = []
        self.proc = None
        self.windows = []
        try:
            props = torch.cuda.get_device_properties(device_index)
            self.target = f"{props.pci_domain_id:08X}:{props.pci_bus_id:02X}:{props.pci_device_id:02X}.0"
        except Exception:
            self.target = str(device_index)

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits", "-lms", "100",
                 "-i", self.target], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except Exception:
            self.proc = None
            return
        self.thread = threading.Thread(target=self._read, daemon=True)
        self.thread.start()

    def _read(self):
        for line in self.proc.stdout:
            self.samples.append((time.time(), [x.strip() for x in line.split(",")]))

    def mark(self, t0, t1):
        self.windows.append((t0, t1))

    def stop(self):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()

    def summary(self):
        rows = [s for t, s in self.samples if any(a - 0.05 <= t <= b + 0.15 for a, b in self.windows)]
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"], "samples": 0}
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = set()
        mhz, mx = [], []
        for s in rows:
            try:
                mhz.append(float(s[1]))
                mx.append(float(s[2]))
            except (ValueError, IndexError):
                continue
            for n, v in zip(names, s[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        return {"sm_mhz": float(np.median(mhz)) if mhz else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": sorted(reasons), "samples": len(rows)}


def dist_setup(n_gpus):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime
        torch.cuda.set_device(local)
        torch.distributed.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                             device_id=torch.device(f"cuda:{local}"))
    else:
        torch.cuda.set_device(0)
    return world, rank, local


def barrier(world):
    if world > 1:
        torch.distributed.barrier()


def max_over_ranks(x: float, world: int) -> float:
    if world == 1:
        return x
    t = torch.tensor([x], dtype=torch.float64, device="cuda")
    torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
    return float(t.item())


def launches_per_call(w) -> int:
    """fg_sample's launches on the batch path: history prep (rows with
    penalties), stream, decide, the 16-bit deep-row finish, cluster kernel."""
    pen = w.hist_ids.size > 0 and bool(np.any(w.params.repetition_penalty != 1.0) or
                                       np.any(w.params.presence_penalty != 0.0) or
                                       np.any(w.params.frequency_penalty != 0.0))
    return int(pen) + 2 + int(w.logits.element_size() == 2) + 1


def cpu_reference_rate(w, seconds: float, rows_per_chunk: int = 16):
    """Rows/s of the reference's own CPU path (oracle.reference_chain_rows:
    FlashGen's penalty + Sampler.sample torch operations) on a bounded prefix
    of the workload's rows, with every host thread."""
    from oracle import sampler_oracle as O
    torch.set_num_threads(os.cpu_count() or 1)
    hist = w.histories()
    gen = torch.Generator().manual_seed(0)
    done, t0 = 0, time.perf_counter()
    while done < w.batch and (time.perf_counter() - t0) < seconds:
        r1 = min(w.batch, done + rows_per_chunk)
        O.reference_chain_rows(w.logits[done:r1], w.params.slice(done, r1), hist[done:r1], gen)
        done = r1
    dt = time.perf_counter() - t0
    return done / dt, done, dt


def run_reference(args, world, rank):
    """Reference arm: the reference's own CPU sampling path (FlashGen's torch
    Sampler chain, oracle.reference_chain_rows) on the host cores with every
    thread. Each step samples 16 rows of the same configuration-3 batch as the
    GPU arm, cycling through its 1024 rows."""
    from flashgen_b200.workloads import CONFIG_NAMES, make_workload
    from oracle import sampler_oracle as O
    if rank != 0:
        return
    torch.set_num_threads(os.cpu_count() or 1)
    rows_per_step = 16
    w = make_workload(args.config, seed=1)
    hist = w.histories()
    gen = torch.Generator().manual_seed(0)
    nchunk = max(1, w.batch // rows_per_step)

    def step(i):
        r0 = (i % nchunk) * rows_per_step
        r1 = min(w.batch, r0 + rows_per_step)
        O.reference_chain_rows(w.logits[r0:r1], w.params.slice(r0, r1), hist[r0:r1], gen)

    for i in range(args.warmup):
        step(i)
    t0 = time.perf_counter()
    for i in range(args.steps):
        step(args.warmup + i)
    dt = time.perf_counter() - t0
    rows_s = rows_per_step * args.steps / dt
    line = {
        "impl": "reference", "metric": "sampled_rows_per_s", "value": rows_s, "unit": "rows/s",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": 1e3 * dt / args.steps, "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded; flashgen_b200.workloads)",
        "config": {"workload": CONFIG_NAMES[args.config], "rows_per_step": rows_per_step},
        "cpu_baseline": {"value": rows_s, "unit": "rows/s", "cores": torch.get_num_threads(), "kind": "port",
                         "sample": f"{rows_per_step} rows of {CONFIG_NAMES[args.config]} per step, cycling "
                                   f"through its {w.batch} rows (FlashGen's Sampler torch chain restated)"},
        "e2e": {"value": rows_s, "unit": "rows/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def _args_for(lib_mod, logits, w, packed, uni, hist, out, status, ws):
    a = lib_mod.FgSampleArgs()
    from flashgen_b200.sampling.sampler import _DTYPES
    B, V = logits.shape
    a.logits = logits.data_ptr()
    a.dtype = _DTYPES[logits.dtype]
    a.batch, a.vocab, a.row_stride = B, V, V
    if hist is not None:
        a.hist_ids, a.hist_offsets, a.hist_max_len = hist[0].data_ptr(), hist[1].data_ptr(), hist[2]
    f = packed.f32
    a.temperature, a.top_p = f[0].data_ptr(), f[1].data_ptr()
    a.repetition_penalty, a.presence_penalty, a.frequency_penalty = (f[2].data_ptr(), f[3].data_ptr(),
                                                                     f[4].data_ptr())
    a.top_k, a.greedy = packed.top_k.data_ptr(), packed.greedy.data_ptr()
    a.uniforms = uni.data_ptr()
    a.out_ids, a.out_status = out.data_ptr(), status.data_ptr()
    lib_mod.set_workspace(a, ws)
    return a


class Batch:
    """A workload resident on the device, with `copies` logits buffers that
    alternate between steps (together larger than L2) and one fg_sample
    argument block per buffer."""

    def __init__(self, w, dev, copies=2, w2=None):
        from flashgen_b200 import _lib
        from flashgen_b200.sampling.sampler import PackedParams, _DTYPES
        self.w, self.dev = w, dev
        B, V = w.batch, w.vocab
        p = w.params
        self.packed = PackedParams(p.temperature, p.top_p, p.top_k, p.repetition_penalty, p.presence_penalty,
                                   p.frequency_penalty, p.greedy, dev)
        self.hist = None
        if w.hist_ids.size > 0:
            self.hist = (torch.from_numpy(w.hist_ids).to(dev), torch.from_numpy(w.hist_offsets).to(dev),
                         w.hist_max_len)
        base = [w.logits.to(dev)] + ([w2.logits.to(dev)] if w2 is not None else [])
        self.logits = [base[i % len(base)] if i < len(base) else base[i % len(base)].clone() for i in range(copies)]
        self.uni = torch.from_numpy(w.uniforms).to(dev)
        self.out = torch.empty(B, dtype=torch.int64, device=dev)
        self.status = torch.empty(B, dtype=torch.int32, device=dev)
        need = _lib.workspace_size(B, V, _DTYPES[base[0].dtype], w.hist_max_len)
        self.ws = torch.zeros((need + 3) // 4, dtype=torch.int32, device=dev)
        self.argv = [_args_for(_lib, lg, w, self.packed, self.uni, self.hist, self.out, self.status, self.ws)
                     for lg in self.logits]
        self.lib = _lib.load(build_if_missing=False)
        self.sh = torch.cuda.current_stream(dev).cuda_stream

    def launch(self, i):
        rc = self.lib.fg_sample(self.argv[i % len(self.argv)], self.sh)
        if rc != 0:
            raise RuntimeError(f"fg_sample rc={rc}")

    def time(self, steps, warmup):
        for i in range(warmup):
            self.launch(i)
        torch.cuda.synchronize(self.dev)
        stream = torch.cuda.current_stream(self.dev)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for i in range(steps):
            self.launch(i)
        e1.record(stream)
        e1.synchronize()
        return e0.elapsed_time(e1)


def per_config_lines(dev, steps=50):
    """One GPU, configurations 1, 2, 4 and 5: rows/s, ms per call and the
    fraction of the measured HBM peak; buffers cycle so that together they
    exceed L2."""
    from flashgen_b200 import _lib
    from flashgen_b200.workloads import CONFIG_NAMES, make_workload
    peak, _ = measured_peak()
    res = {}
    for cfg in (1, 2, 4, 5):
        w = make_workload(cfg, seed=3)
        nbytes = w.logits.numel() * w.logits.element_size()
        copies = max(2, int(np.ceil(200e6 / nbytes)))
        bt = Batch(w, dev, copies=min(copies, 256))
        ms = bt.time(steps, 5) / steps
        st = bt.status.cpu().numpy()
        gbs = w.algorithmic_bytes() / (ms / 1e3) / 1e9
        res[CONFIG_NAMES[cfg]] = {"rows_s": w.batch / (ms / 1e3), "ms": ms, "gbs": gbs, "frac": gbs / peak,
                                  "steps": steps, "buffers": len(bt.logits),
                                  "general_path_rows": int(((st & _lib.FG_ROW_GENERAL_PATH) != 0).sum()),
                                  "error_rows": int(((st & _lib.FG_ROW_ERROR_MASK) != 0).sum())}
        del bt, w
        torch.cuda.empty_cache()
    return res


def parity_summary(w, ids, status):
    """The timed batch against the CPU oracle on every row: ids must agree
    except on rows the oracle flags (a uniform or top-p cut within 1e-6 of a
    CDF boundary). tie_id_diff: rows whose top-p cut splits a run of equal
    values and where the reference's own (unstable) sort draws another id than
    the stable order the build keeps."""
    from flashgen_b200 import _lib
    from oracle import sampler_oracle as O
    torch.set_num_threads(os.cpu_count() or 1)
    res = O.sample_rows(w.logits, w.params, w.histories(), w.uniforms, stable=True, want_kept=False)
    flagged = res.near_u | res.near_p
    mism = ids != res.ids
    out = {"rows": int(w.batch), "flagged": int(flagged.sum()), "flagged_mismatch": int((mism & flagged).sum()),
           "unflagged_mismatch": int((mism & ~flagged).sum()),
           "status_mismatch": int((((status & _lib.FG_ROW_ERROR_MASK) != 0) != res.error).sum()),
           "tie_rows": int(res.tie_at_cut.sum())}
    tie = np.nonzero(res.tie_at_cut)[0]
    out["tie_id_diff"] = 0
    if tie.size:
        from flashgen_b200.workloads import BatchParams
        pt = BatchParams(*(getattr(w.params, f)[tie] for f in ("temperature", "top_p", "top_k", "repetition_penalty",
                                                              "presence_penalty", "frequency_penalty", "greedy")))
        hist = w.histories()
        uns = O.sample_rows(w.logits[torch.from_numpy(tie)], pt, [hist[i] for i in tie], w.uniforms[tie],
                            stable=False, want_kept=False)
        out["tie_id_diff"] = int((uns.ids != res.ids[tie]).sum())
    return out


def vocab_sharded_leg(world, rank, local, steps, warmup):
    """Configuration 4 (B=4096, V=152064 fp32, top-k 256) vocabulary-sharded
    over the N ranks: the local candidate stage on each rank's V/N columns,
    one NCCL all-to-all by row owner, the owner's merge and draw. Strong
    scaling (fixed total work). Every rank takes the same collective steps."""
    from flashgen_b200 import _lib
    from flashgen_b200.sampling.sampler import PackedParams
    from flashgen_b200.sampling.sharded import local_candidates, merge_and_draw, merge_params, sharded_step
    from flashgen_b200.workloads import BatchParams

    dev = torch.device(f"cuda:{local}")
    B, V, K, CMAX = 4096, 152064, 256, 320
    lo, hi = V * rank // world, V * (rank + 1) // world
    g = torch.Generator(device=dev).manual_seed(1234 + rank)
    shard = 3.0 * torch.randn(B, hi - lo, generator=g, device=dev, dtype=torch.float32)
    rng = np.random.default_rng(99)
    hist = rng.integers(0, V, (B, 256)).astype(np.int32)
    offs = np.arange(0, B * 256 + 1, 256, dtype=np.int64)
    p = BatchParams.uniform(B, temperature=1.0, top_p=0.9, top_k=K, rep=1.05)
    u = torch.from_numpy(rng.random(B, dtype=np.float32)).to(dev)
    packed = PackedParams(p.temperature, p.top_p, p.top_k, p.repetition_penalty, p.presence_penalty,
                          p.frequency_penalty, p.greedy, dev)
    Bo = B // world
    own = slice(rank * Bo, (rank + 1) * Bo)
    mp = merge_params(p.top_p[own], p.top_k[own], p.greedy[own], dev)
    u_own = u[own].contiguous()
    h = (torch.from_numpy(hist.reshape(-1)).to(dev), torch.from_numpy(offs).to(dev), 256)

    def step():
        return sharded_step(lambda: local_candidates(shard, packed, u, h, lo, V, CMAX),
                            lambda c: merge_and_draw(c.vals, c.gids, c.status, mp, u_own), world)

    for _ in range(warmup):
        ids, st = step()
    torch.cuda.synchronize(dev)
    bad = int(((st & _lib.FG_ROW_ERROR_MASK) != 0).sum())
    barrier(world)
    torch.cuda.synchronize(dev)
    stream = torch.cuda.current_stream(dev)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(steps):
        ids, st = step()
    e1.record(stream)
    e1.synchronize()
    barrier(world)
    ms = max_over_ranks(e0.elapsed_time(e1), world) / steps
    peak, _ = measured_peak()
    bytes_local = B * (hi - lo) * 4 + hist.size * 4 + B * 49
    del shard
    torch.cuda.empty_cache()
    return {"workload": "tp-vocab-b4096-v152064-f32", "parallelism": f"vocab-sharded x{world}",
            "rows_s": B / (ms / 1e3), "ms": ms, "steps": steps,
            "frac_local": bytes_local / (ms / 1e3) / 1e9 / peak, "error_rows": bad}


def run_sharded(args, world, rank, local):
    """Configuration 4: vocabulary-sharded sampling (B=4096, V=152064 fp32
    split V/N per GPU). A step is the local stage on the rank's shard, the
    all-to-all by row owner and the owner merge and draw; total work is fixed
    as N grows (strong scaling). Each rank generates its own shard, seeded by
    rank (3 * N(0,1)); histories, parameters and uniforms are shared."""
    from flashgen_b200 import _lib
    from flashgen_b200.sampling.sampler import PackedParams
    from flashgen_b200.sampling.sharded import local_candidates, merge_and_draw, merge_params, sharded_step
    from flashgen_b200.workloads import BatchParams, CONFIG_NAMES

    dev = torch.device(f"cuda:{local}")
    B, V, K, CMAX = 4096, 152064, 256, 320
    if B % world:
        raise SystemExit(f"batch {B} is not a multiple of {world}")
    lo, hi = V * rank // world, V * (rank + 1) // world
    g = torch.Generator(device=dev).manual_seed(1234 + rank)
    shard = 3.0 * torch.randn(B, hi - lo, generator=g, device=dev, dtype=torch.float32)
    rng = np.random.default_rng(99)
    hist = rng.integers(0, V, (B, 256)).astype(np.int32)
    offs = np.arange(0, B * 256 + 1, 256, dtype=np.int64)
    p = BatchParams.uniform(B, temperature=1.0, top_p=0.9, top_k=K, rep=1.05)
    u = torch.from_numpy(rng.random(B, dtype=np.float32)).to(dev)
    packed = PackedParams(p.temperature, p.top_p, p.top_k, p.repetition_penalty, p.presence_penalty,
                          p.frequency_penalty, p.greedy, dev)
    Bo = B // world
    own = slice(rank * Bo, (rank + 1) * Bo)
    mp = merge_params(p.top_p[own], p.top_k[own], p.greedy[own], dev)
    u_own = u[own].contiguous()
    h = (torch.from_numpy(hist.reshape(-1)).to(dev), torch.from_numpy(offs).to(dev), 256)

    def step():
        return sharded_step(lambda: local_candidates(shard, packed, u, h, lo, V, CMAX),
                            lambda c: merge_and_draw(c.vals, c.gids, c.status, mp, u_own), world)

    for _ in range(args.warmup):
        ids, st = step()
    torch.cuda.synchronize(dev)
    bad = int(((st & _lib.FG_ROW_ERROR_MASK) != 0).sum())
    barrier(world)
    torch.cuda.synchronize(dev)
    stream = torch.cuda.current_stream(dev)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(args.steps):
        ids, st = step()
    e1.record(stream)
    e1.synchronize()
    barrier(world)
    ms = max_over_ranks(e0.elapsed_time(e1), world)
    step_s = ms / 1e3 / args.steps
    bytes_local = B * (hi - lo) * 4 + hist.size * 4 + B * 49
    peak, peak_kind = measured_peak()
    if rank == 0:
        line = {
            "metric": "sampled_rows_per_s", "value": B / step_s, "unit": "rows/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms / args.steps, "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "float32",
            "data": "synthetic (seeded per rank: 3*N(0,1) shards; shared histories, params, uniforms)",
            "config": {"workload": CONFIG_NAMES[4], "batch": B, "vocab": V, "top_k": K, "cand_max": CMAX,
                       "parallelism": f"vocab-sharded x{world} (local top-k, all-to-all by row owner, merge)",
                       "l2": f"shard of {B * (hi - lo) * 4 / 1e6:.0f} MB per GPU"},
            "roofline": {"bound": "hbm", "achieved": bytes_local / step_s / 1e9, "peak": peak, "unit": "GB/s",
                         "frac": bytes_local / step_s / 1e9 / peak, "peak_kind": peak_kind, "traffic": None,
                         "algorithmic_bytes_per_launch": bytes_local},
            "error_rows": bad,
            "gpu_launches": args.steps * 2,
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        torch.distributed.destroy_process_group()


def main():
    args = parse()
    if args.impl == "reference":
        world = int(os.environ.get("WORLD_SIZE", "1"))
        rank = int(os.environ.get("RANK", "0"))
        run_reference(args, world, rank)
        return
    from flashgen_b200 import _lib
    from flashgen_b200.sampling.host import HostBatchSampler
    from flashgen_b200.workloads import CONFIG_NAMES, make_workload

    world, rank, local = dist_setup(args.gpus)
    if args.config == 4:
        run_sharded(args, world, rank, local)
        return
    dev = torch.device(f"cuda:{local}")
    _lib.load(build_if_missing=False)
    cfg = args.config
    # one global batch (same seed on every rank); rank g samples its row block
    wfull = make_workload(cfg, seed=1, batch=args.batch or None)
    wfull2 = make_workload(cfg, seed=2, batch=args.batch or None)
    Bg, V = wfull.batch, wfull.vocab
    if Bg % world:
        raise SystemExit(f"batch {Bg} is not a multiple of {world}")
    lo, hi = rank * Bg // world, (rank + 1) * Bg // world
    w, w2 = wfull.rows(lo, hi), wfull2.rows(lo, hi)
    # enough buffers that the rank's steps cycle through more than L2 (126 MB)
    # even when its row block is small
    nbytes = w.logits.numel() * w.logits.element_size()
    copies = max(2, int(np.ceil(300e6 / max(1, nbytes))))
    bt = Batch(w, dev, copies=copies, w2=w2)

    clocks = ClockSampler(local)
    clocks.start()
    for i in range(args.warmup):
        bt.launch(i)
    torch.cuda.synchronize(dev)
    st = bt.status.cpu().numpy()
    if (st & _lib.FG_ROW_ERROR_MASK).any():
        raise RuntimeError(f"error rows in warm-up: {np.nonzero(st & _lib.FG_ROW_ERROR_MASK)[0][:8]}")
    barrier(world)
    torch.cuda.synchronize(dev)
    t_wall0 = time.time()
    ms_local = bt.time(args.steps, 0)
    t_wall1 = time.time()
    barrier(world)
    torch.cuda.synchronize(dev)
    clocks.mark(t_wall0, t_wall1)
    ms = max_over_ranks(ms_local, world)
    # if the timed region was too short for the 100 ms clock sampler, load the GPU
    # with the same launches for ~1 s more (untimed) to read clocks under load
    if t_wall1 - t_wall0 < 0.5:
        t0 = time.time()
        n_soak = max(1, int(1.0 / max(1e-6, ms_local / 1e3 / max(1, args.steps))))
        for i in range(n_soak):
            bt.launch(i)
        torch.cuda.synchronize(dev)
        clocks.mark(t0, time.time())
    clocks.stop()
    step_s = ms / 1e3 / args.steps
    rows_s = Bg / step_s
    bytes_step = wfull.algorithmic_bytes()          # the whole batch, all ranks
    gbs = bytes_step / step_s / 1e9
    bytes_rank = w.algorithmic_bytes()
    peak, peak_kind = measured_peak()
    # the id / status of buffer 0 (parity below)
    bt.launch(0)
    torch.cuda.synchronize(dev)
    ids0, st0 = bt.out.cpu().numpy(), bt.status.cpu().numpy()
    general_rows = int(((st0 & _lib.FG_ROW_GENERAL_PATH) != 0).sum())
    del bt
    torch.cuda.empty_cache()

    if args.only_step:
        if rank == 0:
            print(json.dumps({"metric": "sampled_rows_per_s", "value": rows_s, "unit": "rows/s", "n_gpus": world,
                              "steps": args.steps, "ms_per_step": ms / args.steps, "batch": Bg,
                              "workload": CONFIG_NAMES[cfg], "general_path_rows": general_rows}), flush=True)
        if world > 1:
            torch.distributed.destroy_process_group()
        return

    # ---- weak scaling: every rank samples a full batch of its own ----
    weak = None
    if world > 1:
        bw = Batch(make_workload(cfg, seed=1000 + rank), dev, copies=2, w2=make_workload(cfg, seed=1001 + rank))
        barrier(world)
        wms = max_over_ranks(bw.time(max(1, args.steps // 2), 3), world) / max(1, args.steps // 2)
        weak = {"value": Bg * world / (wms / 1e3), "unit": "rows/s", "ms_per_step": wms,
                "batch_per_gpu": Bg}
        del bw
        torch.cuda.empty_cache()

    # ---- configuration 4, vocabulary-sharded over the same N ranks ----
    vocab_leg = vocab_sharded_leg(world, rank, local, steps=max(5, min(50, args.steps // 10)), warmup=3)

    # ---- end to end through the host-buffer API (the rank's rows) ----
    e2e = None
    stream = torch.cuda.current_stream(dev)
    if args.e2e_steps > 0:
        p = w.params
        hs = HostBatchSampler(w.batch, V, w.logits.dtype, max(1, w.hist_ids.size), dev)
        lh = [w.logits.contiguous().pin_memory(), w2.logits.contiguous().pin_memory()]
        hid, hoff = torch.from_numpy(w.hist_ids).pin_memory(), torch.from_numpy(w.hist_offsets).pin_memory()
        for i in range(2):
            hs.sample(lh[i], p, hid, hoff, w.uniforms, w.hist_max_len)
        torch.cuda.synchronize(dev)
        barrier(world)
        f0, f1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        f0.record(stream)
        for i in range(args.e2e_steps):
            hs.sample(lh[i & 1], p, hid, hoff, w.uniforms, w.hist_max_len)
        f1.record(stream)
        f1.synchronize()
        e2e_ms = max_over_ranks(f0.elapsed_time(f1), world)
        e2e = {"value": Bg / (e2e_ms / 1e3 / args.e2e_steps), "unit": "rows/s",
               "h2d_bytes_per_step": hs.h2d_bytes * world, "d2h_bytes_per_step": hs.d2h_bytes * world}
        del hs, lh

    lat = per_cfg = par = cpu = None
    if rank == 0 and world == 1:
        # ---- B=1 latency (configuration 5), CUDA-graph launched, fresh uniforms ----
        if args.latency_steps > 0:
            lat = latency_b1(dev, args.latency_steps)
        per_cfg = per_config_lines(dev)
        par = parity_summary(w, ids0, st0)
        if not args.no_cpu_baseline:
            rate, rows, secs = cpu_reference_rate(w, args.cpu_seconds)
            cpu = {"value": rate, "unit": "rows/s", "cores": torch.get_num_threads(), "kind": "port",
                   "sample": f"first {rows} rows of {CONFIG_NAMES[cfg]}: FlashGen's own penalty + Sampler.sample "
                             f"torch chain (oracle.reference_chain_rows), {secs:.1f} s"}

    if rank == 0:
        traffic, traffic_kernels = ncu_traffic(cfg)
        line = {
            "metric": "sampled_rows_per_s", "value": rows_s, "unit": "rows/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms / args.steps,
            "higher_is_better": True, "scaling": "strong" if world > 1 else "weak", "vs_baseline": None,
            "dtype": str(w.logits.dtype).replace("torch.", ""),
            "data": "synthetic (seeded; flashgen_b200.workloads)",
            "config": {"workload": CONFIG_NAMES[cfg], "batch": Bg, "batch_per_gpu": w.batch, "vocab": V,
                       "parallelism": f"row-sharded x{world} (rank g samples rows [g*B/N, (g+1)*B/N))",
                       "l2": f"inputs larger than L2: {copies} logits buffers of {nbytes / 1e6:.0f} MB per GPU cycle"},
            "logits_gbs": gbs,
            "roofline": {"bound": "hbm", "achieved": bytes_rank / step_s / 1e9, "peak": peak, "unit": "GB/s",
                         "frac": bytes_rank / step_s / 1e9 / peak, "peak_kind": peak_kind,
                         "traffic": traffic, "traffic_kernels": traffic_kernels,
                         "algorithmic_bytes_per_launch": bytes_rank,
                         "unit_of_launch": "one fg_sample call (all of its kernels) on one GPU"},
            "clocks": clocks.summary(),
            "gpu_launches": args.steps * launches_per_call(w),
            "general_path_rows": general_rows,
            "e2e": e2e,
            "weak_scaling": weak,
            "vocab_sharded_cfg4": vocab_leg,
            "latency_b1": lat,
            "per_config": per_cfg,
            "parity": par,
            "cpu_baseline": cpu,
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        torch.distributed.destroy_process_group()


def latency_b1(dev, steps, seeds=(0, 1, 2, 3, 7)):
    """Configuration 5 at B=1: per-step latency of a CUDA graph that draws a
    fresh uniform and calls fg_sample, rotating over several seeded rows
    (steps / len(seeds) each); p50 / p99 overall and per seed."""
    from flashgen_b200.sampling.sampler import PackedParams, fused_sample
    from flashgen_b200.workloads import make_workload
    per = max(1, steps // len(seeds))
    all_t, by_seed = [], {}
    s = torch.cuda.Stream(dev)
    for seed in seeds:
        w = make_workload(5, seed=seed)
        p = w.params
        logits = w.logits.to(dev)
        packed = PackedParams(p.temperature, p.top_p, p.top_k, p.repetition_penalty, p.presence_penalty,
                              p.frequency_penalty, p.greedy, dev)
        hist = (torch.from_numpy(w.hist_ids).to(dev), torch.from_numpy(w.hist_offsets).to(dev), w.hist_max_len)
        u = torch.rand(1, device=dev)
        out = torch.empty(1, dtype=torch.int64, device=dev)
        with torch.cuda.stream(s):
            for _ in range(3):
                u.uniform_()
                fused_sample(logits, packed, u, hist, out=out, stream=s)
            s.synchronize()
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=s):
                u.uniform_()
                fused_sample(logits, packed, u, hist, out=out, stream=s)
            for _ in range(10):
                g.replay()
            s.synchronize()
            ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(per)]
            for a, b in ev:
                a.record(s)
                g.replay()
                b.record(s)
            s.synchronize()
        t = np.array([a.elapsed_time(b) * 1e3 for a, b in ev])
        all_t.append(t)
        by_seed[str(seed)] = {"p50_us": float(np.percentile(t, 50)), "p99_us": float(np.percentile(t, 99))}
        del g
    t = np.concatenate(all_t)
    return {"p50_us": float(np.percentile(t, 50)), "p99_us": float(np.percentile(t, 99)), "steps": int(t.size),
            "per_seed": by_seed,
            "workload": f"latency-b1-v256000-f32, rows of seeds {list(seeds)} (graph: uniform draw + fg_sample)"}


if __name__ == "__main__":
    main()
