"""flashgen_b200: B200-native (sm_100a) decode-step token sampler.

Drop-in for FlashGen's sampling path: ``SamplingParams`` and ``Sampler`` keep
the reference's call surface (flashgen/core/config.py, flashgen/sampling/
sampler.py) and run one fused CUDA kernel per call through the C ABI declared
in include/flashgen_sampler.h.
"""
from .core.config import SamplingParams  # noqa: F401
from .sampling.sampler import Sampler  # noqa: F401

__version__ = "0.1.0"
__all__ = ["SamplingParams", "Sampler"]
