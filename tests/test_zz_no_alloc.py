"""fg_sample_noalloc: the same results as fg_sample, with no caller workspace.

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
    ws = torch.zeros(_lib.FG_SAMPLE_WORKSPACE_BYTES // 4, dtype=torch.int32, device=dev)
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
        assert (st_b.cpu().numpy() & _lib.FG_ROW_ERROR_MASK == 0).all(), call
        np.testing.assert_array_equal(out_b.cpu().numpy(), out_a.cpu().numpy())
        np.testing.assert_array_equal(st_b.cpu().numpy(), st_a.cpu().numpy())
    assert (ws[:64].cpu().numpy() == 0).all()   # the row-queue counters
