"""The CPU oracle against the golden fixtures pinned to FlashGen's own Sampler
(tests/golden/make_golden.py ran the reference functions on the same inputs)."""
import os

import numpy as np
import pytest

from flashgen_b200.workloads import make_workload
from oracle import sampler_oracle as O
from tests.golden.make_golden import CASES, input_checksum

GOLDEN = os.path.join(os.path.dirname(__file__), "golden")


@pytest.mark.parametrize("cfg,batch", CASES)
def test_oracle_matches_golden(cfg, batch):
    g = np.load(os.path.join(GOLDEN, f"golden_cfg{cfg}.npz"))
    w = make_workload(cfg, batch=batch)
    assert input_checksum(w) == str(g["checksum"]), "workload generator drifted"
    res = O.sample_rows(w.logits, w.params, w.histories(), w.uniforms, stable=True)
    np.testing.assert_array_equal(res.ids, g["ids"])
    np.testing.assert_array_equal(res.near_u, g["near_u"])
    np.testing.assert_array_equal(res.near_p, g["near_p"])
    np.testing.assert_array_equal(res.tie_at_cut, g["tie_at_cut"])
    np.testing.assert_array_equal([len(k) for k in res.kept_ids], g["n_kept"])
    np.testing.assert_array_equal([int(np.sum(k)) for k in res.kept_ids], g["kept_idsum"])
