"""The PyBind11 module flashgen_b200._C (the counterpart of the reference's
`_C` extension, csrc/bindings/flashgen_bindings.cpp:89,153-162): it builds,
mirrors the reference's C++ SamplingParams (csrc/include/request.hpp:14-22)
with presence and frequency added, packs parameters, and turns error codes
into RuntimeError. No GPU needed: only argument validation is reached."""
import importlib

import pytest

from flashgen_b200 import _lib
from flashgen_b200 import build as _build


@pytest.fixture(scope="module")
def C():
    _lib.load()
    _build.build_bindings()
    return importlib.import_module("flashgen_b200._C")


def test_sampling_params_mirror(C):
    p = C.SamplingParams()
    assert p.temperature == 1.0 and p.top_k == -1 and p.repetition_penalty == 1.0 and not p.greedy
    assert abs(p.top_p - 0.9) < 1e-7 and p.max_tokens == 128 and p.stop_token_ids == [50256]
    assert p.presence_penalty == 0.0 and p.frequency_penalty == 0.0
    p.presence_penalty, p.frequency_penalty, p.top_k, p.greedy = 0.25, 0.5, 40, True
    t, tp, k, rep, pres, freq, g = C.pack_params([p, C.SamplingParams()])
    assert k == [40, -1] and g == [1, 0] and pres == [0.25, 0.0] and freq == [0.5, 0.0]


def test_workspace_size_matches_c_abi(C):
    for b, v, dt, h in [(1, 256000, C.DTYPE_F32, 4096), (1024, 128256, C.DTYPE_BF16, 1024), (256, 32000, C.DTYPE_F16, 0)]:
        assert C.workspace_size(b, v, dt, h) == _lib.workspace_size(b, v, dt, h) > 0


def test_errors_raise(C):
    with pytest.raises(RuntimeError, match="invalid argument"):
        C.sample(0, C.DTYPE_BF16, 4, 100, 0, 0, 0, 0, 0, 0)
    with pytest.raises(RuntimeError, match="invalid argument"):
        C.argmax(0, C.DTYPE_F32, 2, 10, 0, 0)
    assert C.version() == _lib.load().fg_version()
