"""fg_sample_noalloc: the same results as fg_sample, with no caller workspace.

Some callers cannot allocate device memory at sampling time (an engine loop
that must not allocate, a plain-FFI host without a device allocator), so the
library offers this entry point, whose scratch is a fixed static device array.
Its results must match fg_sample's within the parity tolerance of the other
tests: ids equal on every row the CPU oracle does not flag as within 1e-6 of
a CDF or top-p boundary (the two calls may take different kernels, which
round masses at the same scale but sum them in another order), error bits
equal on every row.

Collected last (file name), and independent of the tests before it: the
static scratch is cleared on a device's first call and every launch leaves it
zero, so the result is the same alone and after the other tests.
"""
import ctypes

import numpy as np
import pytest
import torch

from flashgen_b200 import _lib
from flashgen_b200.sampling.sampler import PackedParams, _DTYPES
from flashgen_b200.workloads import make_workload
from oracle import sampler_oracle as O


def _args(w, logits, packed, hist, uni, out, status, workspace):
    a = _lib.FgSampleArgs()
    a.logits = logits.data_ptr()
    a.dtype = _DTYPES[logits.dtype]
    a.batch, a.vocab, a.row_stride = w.batch, w.vocab, w.vocab
    a.hist_ids, a.hist_offsets, a.hist_max_len = hist[0].data_ptr(), hist[1].data_ptr(), w.hist_max_len
    f = packed.f32
    a.temperature, a.top_p = f[0].data_ptr(), f[1].data_ptr()
    a.repetition_penalty, a.presence_penalty, a.frequency_penalty = f[2].data_ptr(), f[3].data_ptr(), f[4].data_ptr()
    a.top_k, a.greedy = packed.top_k.data_ptr(), packed.greedy.data_ptr()
    a.uniforms = uni.data_ptr()
    a.out_ids, a.out_status = out.data_ptr(), status.data_ptr()
    if workspace is not None:
        _lib.set_workspace(a, workspace)
    return a


@pytest.mark.gpu
@pytest.mark.parametrize("cfg,batch", [(3, 64), (2, 96)])
def test_noalloc_matches_fg_sample(cuda_device, cfg, batch):
    lib = _lib.load(build_if_missing=False)
    dev = cuda_device
    w = make_workload(cfg, batch=batch, seed=17)
    p = w.params
    packed = PackedParams(p.temperature, p.top_p, p.top_k, p.repetition_penalty, p.presence_penalty,
                          p.frequency_penalty, p.greedy, dev)
    logits = w.logits.to(dev)
    hist = (torch.from_numpy(w.hist_ids).to(dev), torch.from_numpy(w.hist_offsets).to(dev))
    uni = torch.from_numpy(w.uniforms).to(dev)
    need = _lib.workspace_size(w.batch, w.vocab, _DTYPES[logits.dtype], w.hist_max_len)
    ws = torch.zeros((need + 3) // 4, dtype=torch.int32, device=dev)
    res = O.sample_rows(w.logits, w.params, w.histories(), w.uniforms, want_kept=False)
    flagged = res.near_u | res.near_p
    stream = torch.cuda.current_stream(dev).cuda_stream
    for call in range(2):   # two calls in a row: the scratch must come back zero
        out_a = torch.full((w.batch,), -7, dtype=torch.int64, device=dev)
        out_b = torch.full((w.batch,), -7, dtype=torch.int64, device=dev)
        st_a = torch.full((w.batch,), -7, dtype=torch.int32, device=dev)
        st_b = torch.full((w.batch,), -7, dtype=torch.int32, device=dev)
        a = _args(w, logits, packed, hist, uni, out_a, st_a, ws)
        b = _args(w, logits, packed, hist, uni, out_b, st_b, None)
        assert lib.fg_sample(ctypes.byref(a), stream) == _lib.FG_OK
        assert lib.fg_sample_noalloc(ctypes.byref(b), stream) == _lib.FG_OK
        torch.cuda.synchronize(dev)
        ids_a, ids_b = out_a.cpu().numpy(), out_b.cpu().numpy()
        sa, sb = st_a.cpu().numpy(), st_b.cpu().numpy()
        assert (sb & _lib.FG_ROW_ERROR_MASK == 0).all(), call
        np.testing.assert_array_equal(sb & _lib.FG_ROW_ERROR_MASK, sa & _lib.FG_ROW_ERROR_MASK)
        ok = (ids_a == ids_b) | flagged
        assert ok.all(), (call, np.nonzero(~ok)[0][:8], ids_a[~ok][:8], ids_b[~ok][:8])
        assert ((ids_b == res.ids) | flagged).all(), call
    assert (ws[:64].cpu().numpy() == 0).all()   # the row-queue counters
