"""kavor_b200: B200-native (sm_100a) kernels and drop-in Python surface for
Kavor's Qwen3 tensor-parallel decode/prefill path.

    from kavor_b200 import LLM, SamplingParams
"""
__all__ = ["LLM", "SamplingParams"]


def __getattr__(name):
    # lazy: importing the package must not require a GPU or the built library
    if name == "LLM":
        from kavor_b200.llm import LLM

        return LLM
    if name == "SamplingParams":
        from kavor_b200.sampling_params import SamplingParams

        return SamplingParams
    raise AttributeError(name)
