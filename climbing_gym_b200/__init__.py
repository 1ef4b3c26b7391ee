"""B200-native LFM2.5 rollout engine: a drop-in for Climbing Gym's native inference package.

The exported names are those of the reference's ``climbing_gym.inference`` package
(src/climbing_gym/inference/__init__.py:1-59). Engine classes import torch and the CUDA library
lazily so that configuration and synthetic-data helpers stay importable on a machine without a
GPU; constructing an engine without the built sm_100a library raises.
"""
from .config import InferenceEngineConfig, LFM2Config, LFM25SamplingConfig, SamplingConfig

_LAZY = {
    "LFM25Engine": "engine", "flatten_token_batches": "engine",
    "LFM25PackedWeights": "weights", "describe_lfm25_checkpoint": "weights",
    "LFM25GenerationSession": "session", "LFM25ContinuationHandle": "session", "LFM25SessionResult": "session",
    "LFM25PrefixSnapshot": "session",
    "LFM25GenerationOutput": "types", "LFM25PrefixBatch": "types", "LFM25DecodeBatch": "types",
    "LFM25StepOutput": "types", "GenerationOutput": "types", "GenerationResult": "types", "BehaviorTopK": "types",
    "PagedHybridCache": "paged", "LFM25HybridCache": "paged",
    "LFM25AsyncInferenceEngine": "async_engine", "AsyncInferenceEngine": "async_engine",
    "B200Decoder": "decoder",
}


def __getattr__(name: str):
    module = _LAZY.get(name)
    if module is None:
        raise AttributeError(f"module {__name__!r} has no attribute {name!r}")
    from importlib import import_module

    loaded = import_module(f".{module}", __name__)
    if name == "LFM25HybridCache":
        return loaded.PagedHybridCache
    if name == "AsyncInferenceEngine":
        return loaded.LFM25AsyncInferenceEngine
    return getattr(loaded, name)


__all__ = ["InferenceEngineConfig", "LFM2Config", "LFM25SamplingConfig", "SamplingConfig", *_LAZY]
