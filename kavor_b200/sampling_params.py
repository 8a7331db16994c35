"""SamplingParams (drop-in for kavor/sampling_params.py:4-11)."""
from dataclasses import dataclass


@dataclass(slots=True)
class SamplingParams:
    temperature: float = 1.0
    max_tokens: int = 64
    ignore_eos: bool = False

    def __post_init__(self):
        # same contract as the reference: temperature 0 is reserved for the
        # engine-internal greedy path (Sequence.temperature = 0)
        assert self.temperature > 1e-10, "greedy sampling is not permitted"
        assert self.max_tokens >= 1, "max_tokens must be positive"
