from .config import SamplingParams  # noqa: F401
