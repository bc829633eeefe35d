"""DecodeBatch's device-resident histories (flashgen_b200/sampling/decode.py),
on the CPU: the compact CSR view fg_sample reads, and the append of each
step's ids (the sampling itself is covered by the GPU tests)."""
import numpy as np
import torch

from flashgen_b200.core.config import SamplingParams
from flashgen_b200.sampling.decode import DecodeBatch


def test_csr_and_append():
    rng = np.random.default_rng(0)
    B, cap = 5, 8
    dec = DecodeBatch([SamplingParams(repetition_penalty=1.2)] * B, vocab=100, capacity=cap, device="cpu")
    hist = [list(rng.integers(0, 100, n)) for n in (0, 3, 8, 5, 1)]
    for r, h in enumerate(hist):
        dec.set_history(r, h)
    ids, off, hmax = dec._csr()
    assert hmax == cap
    assert off.tolist() == [0] + list(np.cumsum([len(h) for h in hist]))
    for r, h in enumerate(hist):
        assert ids[off[r]:off[r + 1]].tolist() == h
    step = torch.tensor([7, 8, 9, -1, 11])
    dec._append(step)
    for r, h in enumerate(hist):
        if len(h) < cap and int(step[r]) >= 0:
            h.append(int(step[r]))
    assert dec.histories() == hist
    ids, off, _ = dec._csr()
    for r, h in enumerate(hist):
        assert ids[off[r]:off[r + 1]].tolist() == h
