#!/usr/bin/env python
"""Benchmark of the B200 decode-step sampler.

Metric: sampled rows/s and logits GB/s vs the HBM peak on the
Llama-3 mixed-parameter batch (configuration 3: B=1024, V=128256, bf16, full
penalty / temperature / top-k / top-p / draw chain), plus the p50 step latency
at B=1 (configuration 5: V=256000 fp32).

A step is one fused ``fg_sample`` launch over one batch. Inputs are seeded
synthetic data (flashgen_b200.workloads); two distinct logits buffers (2 x 263
MB, each larger than the 126 MB L2) alternate between steps so no step reads
the previous step's logits from L2. With ``--gpus N`` every rank samples its
own batch (data-parallel replicas, weak scaling, no collective on the data
path); the time is the max over ranks.

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
    ap.add_argument("--latency-steps", type=int, default=2000)
    ap.add_argument("--cpu-seconds", type=float, default=12.0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
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
    """DRAM bytes per launch from the committed ncu summary, if any."""
    p = os.path.join(ROOT, "profiles", f"fg_sample_kernel_cfg{config}.md")
    try:
        for line in open(p):
            if line.startswith("traffic_bytes_per_launch:"):
                return float(line.split(":", 1)[1].strip())
    except OSError:
        pass
    return None


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


def cpu_oracle_rate(w, seconds: float, rows_per_chunk: int = 16):
    """Rows/s of the CPU oracle (the reference chain restated) on a bounded
    prefix of the workload's rows."""
    from oracle import sampler_oracle as O
    hist = w.histories()
    done, t0 = 0, time.perf_counter()
    while done < w.batch and (time.perf_counter() - t0) < seconds:
        r1 = min(w.batch, done + rows_per_chunk)
        O.sample_rows(w.logits[done:r1], w.params.slice(done, r1), hist[done:r1], w.uniforms[done:r1],
                      want_kept=False)
        done = r1
    dt = time.perf_counter() - t0
    return done / dt, done, dt


def run_reference(args, world, rank):
    """CPU baseline arm: the oracle (FlashGen's sampler chain restated on torch
    CPU ops) with every host thread, each step a bounded row sample."""
    from flashgen_b200.workloads import CONFIG_NAMES, make_workload
    from oracle import sampler_oracle as O
    if rank != 0:
        return
    torch.set_num_threads(os.cpu_count() or 1)
    rows_per_step = 16
    w = make_workload(args.config, batch=rows_per_step * 4, seed=0)
    hist = w.histories()

    def step(i):
        r0 = (i % 4) * rows_per_step
        r1 = r0 + rows_per_step
        O.sample_rows(w.logits[r0:r1], w.params.slice(r0, r1), hist[r0:r1], w.uniforms[r0:r1], want_kept=False)

    for i in range(args.warmup):
        step(i)
    t0 = time.perf_counter()
    for i in range(args.steps):
        step(i)
    dt = time.perf_counter() - t0
    rows_s = rows_per_step * args.steps / dt
    line = {
        "impl": "reference", "metric": "sampled_rows_per_s", "value": rows_s, "unit": "rows/s",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": 1e3 * dt / args.steps, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": CONFIG_NAMES[args.config], "rows_per_step": rows_per_step},
        "cpu_baseline": {"value": rows_s, "unit": "rows/s", "cores": torch.get_num_threads(), "kind": "port",
                         "sample": f"{rows_per_step} rows of {CONFIG_NAMES[args.config]} per step"},
        "e2e": {"value": rows_s, "unit": "rows/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


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
    from flashgen_b200.sampling.sampler import PackedParams, _DTYPES
    from flashgen_b200.workloads import CONFIG_NAMES, make_workload

    world, rank, local = dist_setup(args.gpus)
    if args.config == 4:
        run_sharded(args, world, rank, local)
        return
    dev = torch.device(f"cuda:{local}")
    lib = _lib.load(build_if_missing=False)
    cfg = args.config
    w = make_workload(cfg, seed=1000 * rank)
    w2 = make_workload(cfg, seed=1000 * rank + 1)
    B, V = w.batch, w.vocab
    p = w.params
    logits = [w.logits.to(dev), w2.logits.to(dev)]
    uni = [torch.from_numpy(w.uniforms).to(dev), torch.from_numpy(w2.uniforms).to(dev)]
    packed = PackedParams(p.temperature, p.top_p, p.top_k, p.repetition_penalty, p.presence_penalty,
                          p.frequency_penalty, p.greedy, dev)
    hist_ids = torch.from_numpy(w.hist_ids).to(dev)
    hist_off = torch.from_numpy(w.hist_offsets).to(dev)
    out = torch.empty(B, dtype=torch.int64, device=dev)
    status = torch.empty(B, dtype=torch.int32, device=dev)
    stream = torch.cuda.current_stream(dev)
    need = _lib.workspace_size(B, V, _DTYPES[logits[0].dtype], w.hist_max_len)
    wspace = torch.zeros((need + 3) // 4, dtype=torch.int32, device=dev)

    def make_args(i):
        a = _lib.FgSampleArgs()
        a.logits = logits[i].data_ptr()
        a.dtype = _DTYPES[logits[i].dtype]
        a.batch, a.vocab, a.row_stride = B, V, V
        a.hist_ids, a.hist_offsets, a.hist_max_len = hist_ids.data_ptr(), hist_off.data_ptr(), w.hist_max_len
        f = packed.f32
        a.temperature, a.top_p = f[0].data_ptr(), f[1].data_ptr()
        a.repetition_penalty, a.presence_penalty, a.frequency_penalty = (f[2].data_ptr(), f[3].data_ptr(),
                                                                         f[4].data_ptr())
        a.top_k, a.greedy = packed.top_k.data_ptr(), packed.greedy.data_ptr()
        a.uniforms = uni[i].data_ptr()
        a.out_ids, a.out_status = out.data_ptr(), status.data_ptr()
        _lib.set_workspace(a, wspace)
        return a

    argv = [make_args(0), make_args(1)]
    sh = stream.cuda_stream

    def launch(i):
        rc = lib.fg_sample(argv[i & 1], sh)
        if rc != 0:
            raise RuntimeError(f"fg_sample rc={rc}")

    clocks = ClockSampler(local)
    clocks.start()
    for i in range(args.warmup):
        launch(i)
    torch.cuda.synchronize(dev)
    st = status.cpu().numpy()
    if (st & _lib.FG_ROW_ERROR_MASK).any():
        raise RuntimeError(f"error rows in warm-up: {np.nonzero(st & _lib.FG_ROW_ERROR_MASK)[0][:8]}")
    general_rows = int(((st & _lib.FG_ROW_GENERAL_PATH) != 0).sum())
    barrier(world)
    torch.cuda.synchronize(dev)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t_wall0 = time.time()
    e0.record(stream)
    for i in range(args.steps):
        launch(i)
    e1.record(stream)
    e1.synchronize()
    t_wall1 = time.time()
    barrier(world)
    torch.cuda.synchronize(dev)
    clocks.mark(t_wall0, t_wall1)
    ms_local = e0.elapsed_time(e1)
    ms = max_over_ranks(ms_local, world)
    # if the timed region was too short for the 100 ms clock sampler, load the GPU
    # with the same launches for ~1 s more (untimed) to read clocks under load
    if t_wall1 - t_wall0 < 0.5:
        t0 = time.time()
        n_soak = max(1, int(1.0 / max(1e-6, ms_local / 1e3 / max(1, args.steps))))
        for i in range(n_soak):
            launch(i)
        torch.cuda.synchronize(dev)
        clocks.mark(t0, time.time())
    clocks.stop()
    step_s = ms / 1e3 / args.steps
    rows_total = B * world
    rows_s = rows_total / step_s
    bytes_step = w.algorithmic_bytes()
    gbs = bytes_step / step_s / 1e9          # per GPU (each GPU moves its own batch)
    peak, peak_kind = measured_peak()

    # ---- end to end through the host-buffer API ----
    e2e = None
    if args.e2e_steps > 0:
        hs = HostBatchSampler(B, V, w.logits.dtype, max(1, w.hist_ids.size), dev)
        lh = [w.logits.pin_memory(), w2.logits.pin_memory()]
        hid, hoff = torch.from_numpy(w.hist_ids).pin_memory(), torch.from_numpy(w.hist_offsets).pin_memory()
        for i in range(2):
            hs.sample(lh[i], p, hid, hoff, w.uniforms, w.hist_max_len)
        torch.cuda.synchronize(dev)
        barrier(world)
        f0, f1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        f0.record(stream)
        for i in range(args.e2e_steps):
            ids_h = hs.sample(lh[i & 1], p, hid, hoff, w.uniforms, w.hist_max_len)
        f1.record(stream)
        f1.synchronize()
        e2e_ms = max_over_ranks(f0.elapsed_time(f1), world)
        e2e = {"value": rows_total / (e2e_ms / 1e3 / args.e2e_steps), "unit": "rows/s",
               "h2d_bytes_per_step": hs.h2d_bytes, "d2h_bytes_per_step": hs.d2h_bytes}
        del hs, lh

    # ---- B=1 latency (configuration 5), CUDA-graph launched, fresh uniforms ----
    lat = None
    if args.latency_steps > 0 and rank == 0:
        lat = latency_b1(lib, dev, args.latency_steps)

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        rate, rows, secs = cpu_oracle_rate(w, args.cpu_seconds)
        cpu = {"value": rate, "unit": "rows/s", "cores": torch.get_num_threads(), "kind": "port",
               "sample": f"first {rows} rows of {CONFIG_NAMES[cfg]} (oracle restating FlashGen's "
                         f"torch sampler chain), {secs:.1f} s"}

    if rank == 0:
        traffic = ncu_traffic(cfg)
        line = {
            "metric": "sampled_rows_per_s", "value": rows_s, "unit": "rows/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms / args.steps,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": str(w.logits.dtype).replace("torch.", ""),
            "data": "synthetic (seeded; flashgen_b200.workloads)",
            "config": {"workload": CONFIG_NAMES[cfg], "batch_per_gpu": B, "vocab": V,
                       "parallelism": f"row-sharded x{world} (independent batches)",
                       "l2": "inputs larger than L2: two 263 MB logits buffers alternate"},
            "logits_gbs_per_gpu": gbs,
            "roofline": {"bound": "hbm", "achieved": gbs, "peak": peak, "unit": "GB/s", "frac": gbs / peak,
                         "peak_kind": peak_kind, "traffic": traffic,
                         "algorithmic_bytes_per_launch": bytes_step},
            "clocks": clocks.summary(),
            "gpu_launches": args.steps,
            "general_path_rows": general_rows,
            "e2e": e2e,
            "latency_b1": lat,
            "cpu_baseline": cpu,
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        torch.distributed.destroy_process_group()


def latency_b1(lib, dev, steps):
    from flashgen_b200.sampling.sampler import PackedParams, fused_sample
    from flashgen_b200.workloads import make_workload
    w = make_workload(5, seed=7)
    p = w.params
    logits = w.logits.to(dev)
    packed = PackedParams(p.temperature, p.top_p, p.top_k, p.repetition_penalty, p.presence_penalty,
                          p.frequency_penalty, p.greedy, dev)
    hist = (torch.from_numpy(w.hist_ids).to(dev), torch.from_numpy(w.hist_offsets).to(dev), w.hist_max_len)
    u = torch.rand(1, device=dev)
    out = torch.empty(1, dtype=torch.int64, device=dev)
    s = torch.cuda.Stream(dev)
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
        ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(steps)]
        for a, b in ev:
            a.record(s)
            g.replay()
            b.record(s)
        s.synchronize()
    t = np.array([a.elapsed_time(b) * 1e3 for a, b in ev])
    return {"p50_us": float(np.percentile(t, 50)), "p99_us": float(np.percentile(t, 99)), "steps": steps,
            "workload": "latency-b1-v256000-f32 (graph: uniform draw + fused sample)"}


if __name__ == "__main__":
    main()
