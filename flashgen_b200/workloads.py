"""Seeded synthetic decode-step inputs shaped like the benchmark configurations.

No public dataset is involved: every configuration below is synthetic logits,
histories, parameters and uniforms drawn from ``numpy.random.default_rng``
(PCG64, stable across numpy versions) so that the same seed gives the same
bytes on the development container and on the GPU box.

Configurations (vocab sizes follow the model each one is named after):

1. GPT-2 CPU case: B=8, V=50257, fp32 ``2*N(0,1)``; T=0.8, top_p=0.9,
   top_k off, no penalties.
2. LLaMA-2 decode: B=256, V=32000, fp16 ``N(0,1)`` plus +6 on 20 ids per row;
   T=0.7, top_k=50, top_p=0.95, repetition 1.1, presence 0.2, frequency 0.1;
   512 uniform history ids per row.
3. Llama-3 mixed batch (headline): B=1024, V=128256, bf16 ``N(0,1)`` plus +8 on
   1% of ids per row; per row T~U[0.5,1.2], top_k in {0,20,100,1000},
   top_p~U[0.8,1.0], 10% greedy (T=0); 1024 history ids per row,
   ``(zipf(1.1)-1) mod V``. The benchmark text fixes no penalty values for this
   configuration; to exercise the full chain the build draws repetition
   ~U[1.0,1.2], presence ~U[0,0.4] and frequency ~U[0,0.2] per row.
4. Tensor-parallel vocab-sharded: B=4096, V=152064, fp32 ``3*N(0,1)``; T=1.0,
   top_k=256, top_p=0.9, repetition 1.05; 256 uniform history ids.
5. Latency: B=1, V=256000, fp32 ``N(0,1)`` + 12 on one id + tail bias
   ``-1.1*ln(1+r_i)`` (r a seeded permutation); T=0.9, top_p=0.9, top_k off,
   repetition 1.2; 4096 uniform history ids.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import List, Optional

import numpy as np
import torch

CONFIG_NAMES = {
    1: "gpt2-cpu-b8-v50257-f32",
    2: "llama2-b256-v32000-f16",
    3: "llama3-mixed-b1024-v128256-bf16",
    4: "tp-vocab-b4096-v152064-f32",
    5: "latency-b1-v256000-f32",
}
CONFIG_SHAPES = {1: (8, 50257), 2: (256, 32000), 3: (1024, 128256),
                 4: (4096, 152064), 5: (1, 256000)}
CONFIG_DTYPES = {1: torch.float32, 2: torch.float16, 3: torch.bfloat16,
                 4: torch.float32, 5: torch.float32}


@dataclass
class BatchParams:
    """Per-row sampling parameters as structure-of-arrays (host numpy)."""

    temperature: np.ndarray
    top_p: np.ndarray
    top_k: np.ndarray
    repetition_penalty: np.ndarray
    presence_penalty: np.ndarray
    frequency_penalty: np.ndarray
    greedy: np.ndarray

    @property
    def batch(self) -> int:
        return int(self.temperature.shape[0])

    @staticmethod
    def uniform(B: int, temperature=1.0, top_p=1.0, top_k=-1, rep=1.0,
                presence=0.0, frequency=0.0, greedy=False) -> "BatchParams":
        return BatchParams(
            np.full(B, temperature, np.float32), np.full(B, top_p, np.float32),
            np.full(B, top_k, np.int32), np.full(B, rep, np.float32),
            np.full(B, presence, np.float32), np.full(B, frequency, np.float32),
            np.full(B, greedy, bool))

    def slice(self, lo: int, hi: int) -> "BatchParams":
        return BatchParams(*(getattr(self, f)[lo:hi] for f in (
            "temperature", "top_p", "top_k", "repetition_penalty",
            "presence_penalty", "frequency_penalty", "greedy")))


@dataclass
class Workload:
    config: int
    name: str
    logits: torch.Tensor              # [B, V] CPU, dtype of the config
    params: BatchParams
    hist_ids: np.ndarray              # int32 CSR ids
    hist_offsets: np.ndarray          # int64 [B+1]
    uniforms: np.ndarray              # float32 [B]

    @property
    def batch(self) -> int:
        return int(self.logits.shape[0])

    @property
    def vocab(self) -> int:
        return int(self.logits.shape[1])

    def histories(self) -> List[np.ndarray]:
        o = self.hist_offsets
        return [self.hist_ids[o[i]:o[i + 1]] for i in range(self.batch)]

    @property
    def hist_max_len(self) -> int:
        if len(self.hist_offsets) < 2:
            return 0
        return int(np.diff(self.hist_offsets).max(initial=0))

    def rows(self, lo: int, hi: int) -> "Workload":
        """Rows [lo, hi) as a workload of their own (a rank's block of a
        row-sharded batch); the history CSR is rebased."""
        o = self.hist_offsets
        ids = self.hist_ids[o[lo]:o[hi]]
        offs = (o[lo:hi + 1] - o[lo]).astype(np.int64)
        return Workload(self.config, self.name, self.logits[lo:hi], self.params.slice(lo, hi), ids, offs,
                        self.uniforms[lo:hi])

    def algorithmic_bytes(self) -> int:
        """Bytes one sampling step must move: logits + histories + per-row
        params (7 fields), uniform, id and offsets."""
        B, V = self.logits.shape
        return (B * V * self.logits.element_size() + 4 * int(self.hist_ids.size)
                + B * (4 + 8 + 4 * 6 + 1 + 8))


def _csr(rows: List[np.ndarray]):
    offs = np.zeros(len(rows) + 1, dtype=np.int64)
    offs[1:] = np.cumsum([len(r) for r in rows])
    ids = np.concatenate(rows).astype(np.int32) if rows else np.zeros(0, np.int32)
    return ids, offs


def _bump_rows(rng, x: np.ndarray, n_per_row: int, value: float) -> None:
    B, V = x.shape
    for r in range(B):
        idx = rng.choice(V, size=n_per_row, replace=False)
        x[r, idx] += value


def make_workload(config: int, batch: Optional[int] = None, seed: int = 0,
                  vocab: Optional[int] = None) -> Workload:
    """Build configuration ``config`` (1..5); ``batch`` overrides B for parity
    tests at reduced size (rows are generated in the same order, so a smaller
    batch is a prefix of the full one only for logits drawn row by row)."""
    B0, V0 = CONFIG_SHAPES[config]
    B = B0 if batch is None else int(batch)
    V = V0 if vocab is None else int(vocab)
    dtype = CONFIG_DTYPES[config]
    rng = np.random.default_rng(seed)
    if config == 1:
        x = 2.0 * rng.standard_normal((B, V), dtype=np.float32)
        params = BatchParams.uniform(B, temperature=0.8, top_p=0.9, top_k=-1)
        hist = [np.zeros(0, np.int32) for _ in range(B)]
    elif config == 2:
        x = rng.standard_normal((B, V), dtype=np.float32)
        _bump_rows(rng, x, 20, 6.0)
        params = BatchParams.uniform(B, temperature=0.7, top_p=0.95, top_k=50,
                                     rep=1.1, presence=0.2, frequency=0.1)
        hist = [rng.integers(0, V, 512).astype(np.int32) for _ in range(B)]
    elif config == 3:
        x = rng.standard_normal((B, V), dtype=np.float32)
        _bump_rows(rng, x, int(round(0.01 * V)), 8.0)
        T = rng.uniform(0.5, 1.2, B).astype(np.float32)
        greedy_rows = rng.random(B) < 0.10
        T[greedy_rows] = 0.0
        params = BatchParams(
            temperature=T,
            top_p=rng.uniform(0.8, 1.0, B).astype(np.float32),
            top_k=rng.choice(np.array([0, 20, 100, 1000], np.int32), B),
            repetition_penalty=rng.uniform(1.0, 1.2, B).astype(np.float32),
            presence_penalty=rng.uniform(0.0, 0.4, B).astype(np.float32),
            frequency_penalty=rng.uniform(0.0, 0.2, B).astype(np.float32),
            greedy=np.zeros(B, bool))
        hist = [((rng.zipf(1.1, 1024) - 1) % V).astype(np.int32) for _ in range(B)]
    elif config == 4:
        x = 3.0 * rng.standard_normal((B, V), dtype=np.float32)
        params = BatchParams.uniform(B, temperature=1.0, top_p=0.9, top_k=256, rep=1.05)
        hist = [rng.integers(0, V, 256).astype(np.int32) for _ in range(B)]
    elif config == 5:
        x = rng.standard_normal((B, V), dtype=np.float32)
        for r in range(B):
            perm = rng.permutation(V)
            x[r] += (-1.1 * np.log1p(perm.astype(np.float64))).astype(np.float32)
            x[r, rng.integers(0, V)] += 12.0
        params = BatchParams.uniform(B, temperature=0.9, top_p=0.9, top_k=-1, rep=1.2)
        hist = [rng.integers(0, V, 4096).astype(np.int32) for _ in range(B)]
    else:
        raise ValueError(f"unknown configuration {config}")
    uniforms = rng.random(B, dtype=np.float32)
    hist_ids, hist_offsets = _csr(hist)
    logits = torch.from_numpy(x).to(dtype)
    return Workload(config, CONFIG_NAMES[config], logits, params, hist_ids,
                    hist_offsets, uniforms)
