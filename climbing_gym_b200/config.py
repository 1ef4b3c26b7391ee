"""Model, sampling and adapter configuration contracts of the LFM2.5 rollout engine.

Field names, defaults and validation messages follow the reference so callers and
checkpoints written for it work unchanged:
  LFM2Config ............ src/climbing_gym/models/lfm2.py:176-262 (+ models/config.py:9-56,
                          models/lfm2_compat.py:8-33 for the Transformers 4/5 spellings)
  LFM25SamplingConfig ... src/climbing_gym/inference/lfm25_engine.py:22-54
  SamplingConfig / InferenceEngineConfig ... src/climbing_gym/inference/config.py:17-87
"""
from __future__ import annotations

import json
import math
from collections.abc import Mapping as MappingABC, Sequence
from dataclasses import MISSING, dataclass, field, fields
from numbers import Real
from pathlib import Path
from typing import Any, Mapping

_LFM25_1P2B_LAYERS = (
    "conv", "conv", "full_attention", "conv", "conv", "full_attention", "conv", "conv",
    "full_attention", "conv", "full_attention", "conv", "full_attention", "conv",
    "full_attention", "conv",
)


@dataclass
class LFM2Config:
    vocab_size: int = 65536
    hidden_size: int = 2048
    mlp_hidden_size: int = 8192
    num_hidden_layers: int = 16
    num_attention_heads: int = 32
    num_key_value_heads: int = 8
    max_position_embeddings: int = 128000
    rope_theta: float = 1_000_000.0
    norm_eps: float = 1e-5
    conv_kernel_size: int = 3
    conv_bias: bool = False
    layer_types: tuple = _LFM25_1P2B_LAYERS
    tie_embedding: bool = True
    pad_token_id: int = 0
    bos_token_id: int = 1
    eos_token_id: int = 7

    @property
    def head_dim(self) -> int:
        return self.hidden_size // self.num_attention_heads

    def validate(self) -> None:
        if len(self.layer_types) != self.num_hidden_layers:
            raise ValueError("len(layer_types) must match num_hidden_layers")
        if self.hidden_size % self.num_attention_heads != 0:
            raise ValueError("hidden_size must be divisible by num_attention_heads")
        if self.num_attention_heads % self.num_key_value_heads != 0:
            raise ValueError("num_attention_heads must be divisible by num_key_value_heads")
        if self.mlp_hidden_size <= 0:
            raise ValueError("mlp_hidden_size must be > 0")
        if self.conv_kernel_size <= 0:
            raise ValueError("conv_kernel_size must be > 0")
        if any(kind not in {"conv", "full_attention"} for kind in self.layer_types):
            raise ValueError("layer_types entries must be either 'conv' or 'full_attention'")

    @classmethod
    def from_dict(cls, payload: Mapping[str, Any]) -> "LFM2Config":
        data = dict(payload)
        rope = data.get("rope_parameters") or data.get("rope_scaling")
        if rope is not None:
            if not isinstance(rope, MappingABC):
                raise ValueError("LFM2 rope_parameters must be an object")
            kind = rope.get("rope_type", rope.get("type", "default"))
            if kind != "default":
                raise ValueError(f"Unsupported LFM2 rope_type: {kind!r}; expected 'default'")
            if rope.get("rope_theta") is not None:
                data["rope_theta"] = float(rope["rope_theta"])
        if data.get("tie_embedding") is None and data.get("tie_word_embeddings") is not None:
            data["tie_embedding"] = bool(data["tie_word_embeddings"])
        if data.get("mlp_hidden_size") is None:
            data["mlp_hidden_size"] = _legacy_mlp_width(data)
        if data.get("conv_kernel_size") is None and data.get("conv_L_cache") is not None:
            data["conv_kernel_size"] = data["conv_L_cache"]
        kwargs = {}
        for item in fields(cls):
            value = data.get(item.name)
            if value is None:
                continue
            default = None if item.default is MISSING else item.default
            kwargs[item.name] = tuple(value) if isinstance(value, list) and isinstance(default, tuple) else value
        config = cls(**kwargs)
        config.validate()
        return config

    @classmethod
    def from_pretrained(cls, model_dir) -> "LFM2Config":
        path = Path(model_dir) / "config.json"
        if not path.exists():
            return cls()
        payload = json.loads(path.read_text(encoding="utf-8"))
        if not isinstance(payload, dict):
            raise TypeError(f"Expected config payload to be an object, got {type(payload)!r}.")
        return cls.from_dict(payload)

    def to_dict(self) -> dict:
        return {f.name: (list(getattr(self, f.name)) if isinstance(getattr(self, f.name), tuple)
                         else getattr(self, f.name)) for f in fields(self)}


def _legacy_mlp_width(payload: Mapping[str, Any]) -> int:
    """Hugging Face checkpoints store ``intermediate_size`` before the 2/3 SwiGLU adjustment."""
    if payload.get("intermediate_size") is None:
        return 8192
    size = int(payload["intermediate_size"])
    if not bool(payload.get("block_auto_adjust_ff_dim", True)):
        return size
    multiple = int(payload.get("block_multiple_of", 256))
    if multiple <= 0:
        raise ValueError("block_multiple_of must be > 0 when normalizing legacy LFM2 configs")
    adjusted = int(float(payload.get("block_ffn_dim_multiplier", 1.0)) * int(2 * size / 3))
    return multiple * ((adjusted + multiple - 1) // multiple)


@dataclass(frozen=True, slots=True)
class LFM25SamplingConfig:
    temperature: float = 1.0
    top_k: int = 0
    top_p: float = 1.0
    repetition_penalty: float = 1.0
    max_new_tokens: int = 256
    stop_token_ids: tuple = ()
    return_logprobs: bool = True
    seed: int = 0
    ignore_eos: bool = False
    stop_token_sequences: tuple = ()
    stop_table: Any = None
    behavior_topk: int = 0

    def __post_init__(self) -> None:
        if self.temperature < 0:
            raise ValueError("temperature must be >= 0")
        if self.top_k < 0:
            raise ValueError("top_k must be 0 or positive")
        if not 0.0 < self.top_p <= 1.0:
            raise ValueError("top_p must be in (0, 1]")
        if self.repetition_penalty <= 0.0:
            raise ValueError("repetition_penalty must be > 0")
        if self.max_new_tokens <= 0:
            raise ValueError("max_new_tokens must be > 0")
        if type(self.behavior_topk) is not int or not 0 <= self.behavior_topk <= 128:
            raise ValueError("behavior_topk must be an integer between 0 and 128")
        if self.behavior_topk and (not self.return_logprobs or self.temperature != 1.0
                                   or self.top_k or self.top_p != 1.0 or self.repetition_penalty != 1.0):
            raise ValueError("behavior_topk requires actual full-support temperature-1 logprobs")
        if any(not sequence for sequence in self.stop_token_sequences):
            raise ValueError("Stop token sequences must be nonempty")


def _finite_real(value: Any) -> bool:
    return isinstance(value, Real) and not isinstance(value, bool) and math.isfinite(value)


@dataclass(frozen=True, slots=True)
class SamplingConfig:
    """Sampling controls of the async adapter (text-level requests)."""

    temperature: float = 0.0
    top_k: int = -1
    top_p: float = 1.0
    max_tokens: int = 256
    n: int = 1
    stop: tuple = ()
    logprobs: int | None = None
    extra_params: Mapping[str, Any] = field(default_factory=dict)

    def __post_init__(self) -> None:
        if not _finite_real(self.temperature) or self.temperature < 0:
            raise ValueError("temperature must be finite and >= 0")
        if type(self.top_k) is not int or self.top_k < -1 or self.top_k == 0:
            raise ValueError("top_k must be -1 or >= 1")
        if not _finite_real(self.top_p) or not 0.0 < self.top_p <= 1.0:
            raise ValueError("top_p must be finite and in (0, 1]")
        if type(self.max_tokens) is not int or self.max_tokens <= 0:
            raise ValueError("max_tokens must be a positive integer")
        if type(self.n) is not int or self.n <= 0:
            raise ValueError("n must be a positive integer")
        if self.logprobs is not None and (type(self.logprobs) is not int or self.logprobs <= 0):
            raise ValueError("logprobs must be a positive integer when provided")
        if (not isinstance(self.stop, Sequence) or isinstance(self.stop, (str, bytes))
                or any(not isinstance(item, str) or not item for item in self.stop)):
            raise ValueError("stop must be a sequence of nonempty strings")
        object.__setattr__(self, "stop", tuple(self.stop))
        if not isinstance(self.extra_params, MappingABC):
            raise ValueError("extra_params must be a mapping")
        unknown = set(self.extra_params) - {"repetition_penalty", "ignore_eos", "behavior_topk"}
        if unknown:
            raise ValueError(f"Unsupported native sampling extra_params: {sorted(map(str, unknown))}")
        penalty = self.extra_params.get("repetition_penalty", 1.0)
        if not _finite_real(penalty) or penalty <= 0:
            raise ValueError("repetition_penalty must be finite and > 0")
        if type(self.extra_params.get("ignore_eos", False)) is not bool:
            raise ValueError("ignore_eos must be a boolean")
        head = self.extra_params.get("behavior_topk", 0)
        if type(head) is not int or not 0 <= head <= 128:
            raise ValueError("behavior_topk must be an integer between 0 and 128")


@dataclass(frozen=True, slots=True)
class InferenceEngineConfig:
    """Configuration of the local async inference adapter (one engine replica per GPU)."""

    model_path: str
    dtype: str = "auto"
    seed: int = 0
    gpu_memory_utilization: float = 0.9
    max_model_len: int | None = None
    max_num_seqs: int | None = None
    enforce_eager: bool = False
    enable_sleep_mode: bool = True
    apply_chat_template: bool = False
    chat_template_enable_thinking: bool = True
    assistant_prefill: str = ""
    default_sampling: SamplingConfig = field(default_factory=SamplingConfig)

    def __post_init__(self) -> None:
        if not 0.0 < self.gpu_memory_utilization <= 1.0:
            raise ValueError("gpu_memory_utilization must be between 0 and 1")
        if self.max_model_len is not None and self.max_model_len <= 0:
            raise ValueError("max_model_len must be > 0 when provided")
        if self.max_num_seqs is not None and self.max_num_seqs <= 0:
            raise ValueError("max_num_seqs must be > 0 when provided")
