"""SamplingParams mirrors the reference's fields, defaults and validation
(flashgen/core/config.py:26-51)."""
import pytest

from flashgen_b200 import SamplingParams


def test_defaults():
    p = SamplingParams()
    assert (p.temperature, p.top_p, p.top_k, p.repetition_penalty, p.greedy, p.max_tokens) == \
        (1.0, 0.9, -1, 1.0, False, 128)
    assert p.stop_token_ids == [50256]
    assert (p.presence_penalty, p.frequency_penalty) == (0.0, 0.0)


@pytest.mark.parametrize("kw", [dict(temperature=-0.1), dict(top_p=0.0), dict(top_p=1.5), dict(max_tokens=0)])
def test_validation(kw):
    with pytest.raises(ValueError):
        SamplingParams(**kw)


def test_valid_edges():
    SamplingParams(temperature=0.0, top_p=1.0, top_k=0)
