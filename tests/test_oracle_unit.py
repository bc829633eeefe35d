"""Hand-checked cases for the oracle's restatement of the reference chain."""
import numpy as np
import torch

from flashgen_b200.workloads import BatchParams
from oracle import sampler_oracle as O


def test_top_k_keeps_ties():
    x = torch.tensor([1.0, 3.0, 2.0, 3.0, 2.0, 0.0])
    y = O.top_k_filter(x, 3)       # 3rd largest is 2.0 -> both 2.0s kept (sampler.py:154)
    assert torch.isfinite(y).tolist() == [False, True, True, True, True, False]


def test_top_p_keeps_crossing_token():
    x = torch.log(torch.tensor([0.5, 0.3, 0.15, 0.05]))
    y, near, tie = O.top_p_filter(x, 0.6)   # exclusive masses 0, .5, .8, .95
    assert torch.isfinite(y).tolist() == [True, True, False, False]
    assert not tie


def test_top_p_tie_order_is_ascending_id():
    x = torch.log(torch.tensor([0.1, 0.3, 0.3, 0.3]))
    y, near, tie = O.top_p_filter(x, 0.4)   # excl 0, .3, .6 -> two of the three 0.3s
    assert torch.isfinite(y).tolist() == [False, True, True, False]
    assert tie


def test_inverse_cdf_descending_probability():
    x = torch.log(torch.tensor([0.0, 0.25, 0.0, 0.5, 0.25]))   # order: 3, then ties 1, 4
    p = torch.softmax(x, -1)
    assert O.inverse_cdf(x, p, 0.0)[0] == 3
    assert O.inverse_cdf(x, p, 0.4999)[0] == 3
    assert O.inverse_cdf(x, p, 0.51)[0] == 1
    assert O.inverse_cdf(x, p, 0.76)[0] == 4
    assert O.inverse_cdf(x, p, 0.9999)[0] == 4


def test_penalties_order():
    x = torch.tensor([2.0, -2.0, 1.0, 4.0])
    hist = [0, 1, 1, 3, 3, 3]
    O.apply_repetition_penalty_row(x, hist, 2.0)
    assert x.tolist() == [1.0, -4.0, 1.0, 2.0]
    O.apply_presence_frequency_row(x, hist, 0.5, 0.25)
    assert x.tolist() == [1.0 - 0.25 - 0.5, -4.0 - 0.5 - 0.5, 1.0, 2.0 - 0.75 - 0.5]


def test_greedy_and_zero_temperature():
    logits = torch.tensor([[0.0, 5.0, 5.0, 1.0], [3.0, 1.0, 2.0, 3.0]])
    p = BatchParams.uniform(2, temperature=0.0)
    r = O.sample_rows(logits, p, None, np.array([0.3, 0.7], np.float32))
    assert r.ids.tolist() == [1, 0] and r.greedy.all()
