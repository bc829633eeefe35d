"""Sampling parameters: drop-in for FlashGen's ``SamplingParams``.

Mirrors ``flashgen/core/config.py:26-51`` (fields, defaults and validation)
and ``csrc/include/request.hpp:14-22``, plus ``presence_penalty`` and
``frequency_penalty`` (default 0.0, i.e. off), which the reference lacks.
"""
from __future__ import annotations

from dataclasses import dataclass, field
from typing import List


@dataclass
class SamplingParams:
    """Controls token sampling during autoregressive generation.

    temperature < 1 sharpens, > 1 flattens; 0 (or ``greedy=True``) decodes
    greedily. ``top_k <= 0`` disables top-k; ``top_p == 1`` disables top-p.
    ``repetition_penalty`` divides positive (multiplies negative) logits of
    tokens already in the history; ``presence_penalty`` subtracts a constant
    from them and ``frequency_penalty`` subtracts it once per occurrence.
    """

    temperature: float = 1.0
    top_p: float = 0.9
    top_k: int = -1                  # -1 = disabled
    repetition_penalty: float = 1.0
    greedy: bool = False
    max_tokens: int = 128
    stop_token_ids: List[int] = field(default_factory=lambda: [50256])  # GPT-2 EOS
    presence_penalty: float = 0.0
    frequency_penalty: float = 0.0

    def __post_init__(self):
        if self.temperature < 0:
            raise ValueError(f"temperature must be >= 0, got {self.temperature}")
        if not 0 < self.top_p <= 1:
            raise ValueError(f"top_p must be in (0, 1], got {self.top_p}")
        if self.max_tokens <= 0:
            raise ValueError(f"max_tokens must be > 0, got {self.max_tokens}")
