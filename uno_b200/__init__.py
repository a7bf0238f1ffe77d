"""uno_b200: a Blackwell-native (sm_100a) Uno inference and training framework.

Public API mirrors the reference package (``nano_vllm_uno/__init__.py:6-19``):
``LLM``, ``SamplingParams`` and ``AsyncLLMEngine`` are exported lazily so that
importing the package does not import torch extensions or CUDA state.
"""

__version__ = "0.1.0"

__all__ = ["AsyncLLMEngine", "LLM", "LLMEngine", "SamplingParams", "Config", "__version__"]


def __getattr__(name: str):
    if name == "AsyncLLMEngine":
        from uno_b200.engine.async_engine import AsyncLLMEngine

        return AsyncLLMEngine
    if name == "LLM":
        from uno_b200.llm import LLM

        return LLM
    if name == "LLMEngine":
        from uno_b200.engine.llm_engine import LLMEngine

        return LLMEngine
    if name == "SamplingParams":
        from uno_b200.sampling_params import SamplingParams

        return SamplingParams
    if name == "Config":
        from uno_b200.config import Config

        return Config
    raise AttributeError(f"module {__name__!r} has no attribute {name!r}")
