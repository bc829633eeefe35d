"""Vocabulary-sharded sampling for tensor-parallel LM-head logits.

Rank g of G holds columns [g*V/G, (g+1)*V/G) of every row (the logits a
column-parallel LM head leaves on each GPU). One sampling step:

1. local stage (``fg_sample_candidates`` on the rank's shard): penalties on
   the shard's history columns, temperature, and per row the shard's top-k
   set with ties, as (y = penalised logit / T, global id). Greedy rows give
   their first maximum.
2. exchange: one all-to-all by row owner (rank h owns rows
   [h*B/G, (h+1)*B/G)); per row and shard cand_max values, ids, a count and
   the shard's status word cross the link.
3. merge (owner): each row's G*cand_max candidates are sorted by global id and
   sampled with ``fg_sample`` itself: temperature 1 (already applied), no
   penalties (already applied), the row's top_k and top_p and uniform. The
   top-k of the union of the shards' top-k sets is the global top-k; top-p
   then runs on that k-filtered set, as FlashGen's sampler does
   (flashgen/sampling/sampler.py:113-117, 156-169); and the draw's tie order
   (ascending id) follows the sort.
4. optionally an all-gather of the drawn ids.

The local stage and the merge are passed in as functions so that the
exchange logic can be checked with gloo on CPU (tests/test_sharded_cpu.py);
on GPUs they are the kernels below.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Callable, Optional, Tuple

import numpy as np
import torch

from .. import _lib
from .sampler import PackedParams, _DTYPES, _ptr, fused_sample, workspace_for

INT32_MAX = 2 ** 31 - 1


@dataclass
class Candidates:
    vals: torch.Tensor     # [B, cmax] float32, -inf padded
    gids: torch.Tensor     # [B, cmax] int32, INT32_MAX padded
    counts: torch.Tensor   # [B] int32
    status: torch.Tensor   # [B] int32 (FG_ROW_* bits of the shard)


def local_candidates(shard: torch.Tensor, packed: PackedParams, uniforms: torch.Tensor,
                     hist: Optional[Tuple[torch.Tensor, torch.Tensor, int]], vocab_offset: int,
                     vocab_total: int, cand_max: int, stream: Optional[torch.cuda.Stream] = None) -> Candidates:
    """Local stage on one GPU shard [B, V/G] (fg_sample_candidates)."""
    lib = _lib.load()
    B, V = shard.shape
    dev = shard.device
    vals = torch.empty(B, cand_max, dtype=torch.float32, device=dev)
    gids = torch.empty(B, cand_max, dtype=torch.int32, device=dev)
    counts = torch.empty(B, dtype=torch.int32, device=dev)
    status = torch.empty(B, dtype=torch.int32, device=dev)
    out = torch.empty(B, dtype=torch.int64, device=dev)
    a = _lib.FgSampleArgs()
    a.logits = shard.data_ptr()
    a.dtype = _DTYPES[shard.dtype]
    a.batch, a.vocab = B, V
    a.row_stride = shard.stride(0) if B > 1 else V
    a.vocab_offset, a.vocab_total = vocab_offset, vocab_total
    if hist is not None:
        a.hist_ids, a.hist_offsets, a.hist_max_len = hist[0].data_ptr(), hist[1].data_ptr(), int(hist[2])
    f = packed.f32
    a.temperature, a.top_p = _ptr(f[0]), _ptr(f[1])
    a.repetition_penalty = _ptr(f[2]) if packed.any_rep else None
    a.presence_penalty = _ptr(f[3]) if packed.any_presence else None
    a.frequency_penalty = _ptr(f[4]) if packed.any_frequency else None
    a.top_k, a.greedy = _ptr(packed.top_k), _ptr(packed.greedy)
    a.uniforms = uniforms.data_ptr()
    a.out_ids, a.out_status = out.data_ptr(), status.data_ptr()
    st = stream if stream is not None else torch.cuda.current_stream(dev)
    _lib.set_workspace(a, workspace_for(dev, st))
    with torch.cuda.device(dev):
        _lib.check(lib.fg_sample_candidates(a, vals.data_ptr(), gids.data_ptr(), counts.data_ptr(), cand_max,
                                            st.cuda_stream), "fg_sample_candidates")
    return Candidates(vals, gids, counts, status)


def merge_params(top_p: np.ndarray, top_k: np.ndarray, greedy: np.ndarray, device) -> PackedParams:
    """Parameters of the merge: temperature 1 and no penalties (both already
    applied by the local stage); greedy rows stay greedy."""
    B = len(top_p)
    return PackedParams(np.ones(B, np.float32), top_p, top_k, np.ones(B, np.float32), np.zeros(B, np.float32),
                        np.zeros(B, np.float32), greedy, device)


def sort_by_id(vals: torch.Tensor, gids: torch.Tensor) -> Tuple[torch.Tensor, torch.Tensor]:
    """Each row's candidates in ascending global id (padding last)."""
    order = torch.argsort(gids, dim=1)
    return torch.gather(vals, 1, order), torch.gather(gids, 1, order)


def merge_and_draw(vals: torch.Tensor, gids: torch.Tensor, shard_status: torch.Tensor, mp: PackedParams,
                   uniforms: torch.Tensor) -> Tuple[torch.Tensor, torch.Tensor]:
    """Owner merge on GPU: fg_sample over the id-sorted union of the shards'
    candidates. Returns (global ids, status)."""
    v, g = sort_by_id(vals, gids)
    status = torch.empty(v.shape[0], dtype=torch.int32, device=v.device)
    pos = fused_sample(v.contiguous(), mp, uniforms, None, status=status)
    ids = torch.gather(g, 1, pos.clamp_min(0)[:, None])[:, 0].to(torch.int64)
    ids = torch.where(pos >= 0, ids, torch.full_like(ids, -1))
    status = status | shard_status
    ids = torch.where((status & _lib.FG_ROW_ERROR_MASK) != 0, torch.full_like(ids, -1), ids)
    return ids, status


def exchange(c: Candidates, world: int, group=None) -> Candidates:
    """All-to-all by row owner: rank h receives, for its B/G rows, every
    shard's candidates; returns [B/G, G*cmax] vals/gids and the OR of the
    shards' status words. One NCCL all-to-all carries everything: each row
    is packed as [value bits (cmax), global ids (cmax), status] int32 words."""
    import torch.distributed as dist
    B, cmax = c.vals.shape
    if B % world:
        raise ValueError(f"batch {B} is not a multiple of the world size {world}")
    Bo = B // world
    # send buffer: rows already grouped by owner (contiguous row blocks)
    send = torch.cat([c.vals.contiguous().view(torch.int32), c.gids.contiguous(),
                      c.status.contiguous().view(B, 1)], dim=1)
    recv = torch.empty_like(send)
    dist.all_to_all_single(recv, send, group=group)
    # received: [world (source shard), Bo, 2 * cmax + 1]
    r = recv.view(world, Bo, 2 * cmax + 1)
    vals = r[:, :, :cmax].contiguous().view(torch.float32).permute(1, 0, 2).reshape(Bo, world * cmax)
    gids = r[:, :, cmax:2 * cmax].permute(1, 0, 2).reshape(Bo, world * cmax)
    status = r[:, :, 2 * cmax]
    st = status[0].clone()
    for i in range(1, world):
        st |= status[i]
    counts = (gids != INT32_MAX).sum(dim=1).to(torch.int32)
    return Candidates(vals, gids, counts, st)


def sharded_step(local_fn: Callable[[], Candidates], merge_fn: Callable[[Candidates], Tuple[torch.Tensor, torch.Tensor]],
                 world: int, group=None, gather_ids: bool = False):
    """One vocabulary-sharded sampling step: local stage, exchange, owner
    merge, and (gather_ids) an all-gather of the drawn ids."""
    import torch.distributed as dist
    c = local_fn()
    own = exchange(c, world, group) if world > 1 else c
    ids, status = merge_fn(own)
    if gather_ids and world > 1:
        all_ids = torch.empty(ids.numel() * world, dtype=ids.dtype, device=ids.device)
        dist.all_gather_into_tensor(all_ids, ids.contiguous(), group=group)
        return all_ids, status
    return ids, status
