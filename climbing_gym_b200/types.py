"""Result and request containers of the rollout engine.

Shapes and field names follow the reference so downstream rollout code reads them unchanged:
token-level outputs (src/climbing_gym/inference/lfm25_engine.py:434-476) and the text-level
request/response contracts of the async adapter (src/climbing_gym/inference/types.py:1-67).
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Any, Mapping, Sequence

import torch

PromptInput = str | Sequence[int] | Mapping[str, Any]


@dataclass(frozen=True, slots=True)
class LFM25GenerationOutput:
    token_ids: torch.Tensor          # [prompts, repeats, max_new] int64, 0 after a row finished
    lengths: torch.Tensor            # [prompts, repeats] int32
    logprobs: torch.Tensor | None    # [prompts, repeats, max_new] fp32 raw (untempered) log-probs
    finish_reasons: torch.Tensor     # [prompts, repeats] int8: 1 EOS, 2 stop, 3 length
    topk_token_ids: torch.Tensor | None = None
    topk_logprobs: torch.Tensor | None = None


@dataclass(frozen=True, slots=True)
class LFM25PrefixBatch:
    cache: Any
    next_token_logits: torch.Tensor
    prompt_lengths: torch.Tensor
    input_ids: torch.Tensor
    slots: torch.Tensor | None = None

    @property
    def batch_size(self) -> int:
        return int(self.prompt_lengths.numel())


@dataclass(slots=True)
class LFM25DecodeBatch:
    cache: Any
    active_slot_ids: torch.Tensor
    prompt_indices: torch.Tensor
    repeat_indices: torch.Tensor
    alive: torch.Tensor

    @property
    def batch_size(self) -> int:
        return int(self.prompt_indices.numel())


@dataclass(frozen=True, slots=True)
class LFM25StepOutput:
    token_ids: torch.Tensor
    raw_logprobs: torch.Tensor | None
    sampling_logprobs: torch.Tensor | None
    finished: torch.Tensor
    finish_reasons: torch.Tensor
    logits: torch.Tensor


@dataclass(frozen=True, slots=True)
class BehaviorTopK:
    """Unfiltered sampler head aligned with the generated tokens (normally CPU tensors)."""

    token_ids: torch.Tensor
    logprobs: torch.Tensor

    def __post_init__(self):
        if self.token_ids.ndim != 2 or self.token_ids.shape != self.logprobs.shape:
            raise ValueError("Behavior head IDs/logprobs must be aligned [tokens, k] tensors")
        if self.token_ids.dtype not in (torch.int32, torch.int64) or self.logprobs.dtype != torch.float32:
            raise ValueError("Behavior head requires integer IDs and FP32 logprobs")


@dataclass(frozen=True, slots=True)
class GenerationOutput:
    index: int
    text: str
    token_ids: tuple
    completion_logprobs: tuple | None
    finish_reason: str | None
    stop_reason: str | None
    behavior_topk: BehaviorTopK | None = None


@dataclass(frozen=True, slots=True)
class GenerationResult:
    request_id: str
    prompt: PromptInput
    prompt_token_ids: tuple
    outputs: tuple
    finished: bool
    raw_output: Any

    @property
    def text(self) -> str:
        return self.outputs[0].text if self.outputs else ""

    @property
    def token_ids(self) -> tuple:
        return self.outputs[0].token_ids if self.outputs else ()

    @property
    def completion_logprobs(self):
        return self.outputs[0].completion_logprobs if self.outputs else None
