"""Packed LFM2.5 weights resident in HBM.

Same packing and in-place synchronisation contract as the reference's
``LFM25PackedWeights`` (src/climbing_gym/inference/lfm25_engine.py:88-367): q/k/v rows are
concatenated into one ``qkv`` matrix, w1/w3 into ``w13``, the depthwise conv weight
``[H, 1, 3]`` is stored as ``[H, 3]``, tied checkpoints alias the LM head to the embedding,
and ``copy_from_model_`` validates every source shape before the first byte is written so
captured CUDA graphs (which hold these addresses) always see a consistent policy.

All matrices are ``[out_features, in_features]`` row-major, i.e. K-major for both GEMM
operands: exactly the layout TMA + tcgen05 consume without a transpose.
"""
from __future__ import annotations

import json
from dataclasses import dataclass
from pathlib import Path
from typing import Any, Mapping

import torch

from . import _native as nv
from .config import LFM2Config


@dataclass(frozen=True, slots=True)
class LFM25AttentionWeights:
    qkv_weight: torch.Tensor
    out_weight: torch.Tensor
    q_norm_weight: torch.Tensor
    k_norm_weight: torch.Tensor
    cache_index: int


@dataclass(frozen=True, slots=True)
class LFM25ConvWeights:
    in_weight: torch.Tensor
    conv_weight: torch.Tensor
    out_weight: torch.Tensor
    cache_index: int


@dataclass(frozen=True, slots=True)
class LFM25LayerWeights:
    operator_norm_weight: torch.Tensor
    ffn_norm_weight: torch.Tensor
    w13_weight: torch.Tensor
    w2_weight: torch.Tensor
    attention: LFM25AttentionWeights | None = None
    conv: LFM25ConvWeights | None = None

    @property
    def is_attention_layer(self) -> bool:
        return self.attention is not None


def _find(state: Mapping[str, Any], key: str):
    for candidate in (key, key.removeprefix("model.") if key.startswith("model.") else f"model.{key}"):
        value = state.get(candidate)
        if value is not None:
            return value
    raise KeyError(f"Missing tensor {key!r} in LFM2 checkpoint")


def _has(state: Mapping[str, Any], key: str) -> bool:
    other = key.removeprefix("model.") if key.startswith("model.") else f"model.{key}"
    return key in state or other in state


def _as_tensor(value) -> torch.Tensor:
    return value if torch.is_tensor(value) else torch.as_tensor(value)


def coerce_config(config: Any) -> LFM2Config:
    """Accept this package's config, the reference's LFM2Config, or any object with to_dict()."""
    if isinstance(config, LFM2Config):
        return config
    if config is None:
        raise TypeError("LFM25 weight synchronization requires a model with an LFM2 config")
    to_dict = getattr(config, "to_dict", None)
    if not callable(to_dict):
        raise TypeError("LFM25 weight synchronization requires an LFM2 config exposing to_dict()")
    payload = to_dict()
    if not isinstance(payload, Mapping):
        raise TypeError("LFM2 config.to_dict() must return a mapping")
    return LFM2Config.from_dict(dict(payload))


_SYNC_FIELDS = ("vocab_size", "hidden_size", "mlp_hidden_size", "num_hidden_layers", "num_attention_heads",
                "num_key_value_heads", "max_position_embeddings", "rope_theta", "norm_eps", "conv_kernel_size",
                "conv_bias", "layer_types", "tie_embedding", "pad_token_id", "bos_token_id", "eos_token_id")


@dataclass(frozen=True, slots=True)
class LFM25PackedWeights:
    config: LFM2Config
    embed_tokens: torch.Tensor
    embedding_norm_weight: torch.Tensor
    lm_head_weight: torch.Tensor
    layers: tuple
    device: torch.device
    dtype: torch.dtype

    @property
    def num_attention_layers(self) -> int:
        return sum(1 for layer in self.layers if layer.attention is not None)

    @property
    def num_conv_layers(self) -> int:
        return sum(1 for layer in self.layers if layer.conv is not None)

    @classmethod
    def from_pretrained(cls, model_dir, *, device, dtype) -> "LFM25PackedWeights":
        path = Path(model_dir)
        return cls.from_state_dict(LFM2Config.from_pretrained(path), load_state_dict(path), device=device, dtype=dtype)

    @classmethod
    def from_model(cls, model: Any, *, device=None, dtype=None) -> "LFM25PackedWeights":
        first = next(model.parameters())
        return cls.from_state_dict(coerce_config(getattr(model, "config", None)), model.state_dict(),
                                   device=device or first.device, dtype=dtype or first.dtype)

    @classmethod
    def from_state_dict(cls, config: LFM2Config, state: Mapping[str, Any], *, device, dtype) -> "LFM25PackedWeights":
        config = coerce_config(config)
        config.validate()
        device = torch.device(device)

        def put(key: str) -> torch.Tensor:
            return _as_tensor(_find(state, key)).detach().to(device=device, dtype=dtype).contiguous()

        embed = put("model.embed_tokens.weight")
        head = put("model.lm_head.weight") if _has(state, "model.lm_head.weight") else embed
        layers, n_attn, n_conv = [], 0, 0
        for index, kind in enumerate(config.layer_types):
            p = f"model.layers.{index}"
            shared = dict(
                operator_norm_weight=put(f"{p}.operator_norm.weight"), ffn_norm_weight=put(f"{p}.ffn_norm.weight"),
                w13_weight=torch.cat([put(f"{p}.feed_forward.w1.weight"), put(f"{p}.feed_forward.w3.weight")], 0).contiguous(),
                w2_weight=put(f"{p}.feed_forward.w2.weight"))
            if kind == "full_attention":
                qkv = torch.cat([put(f"{p}.self_attn.{n}_proj.weight") for n in "qkv"], 0).contiguous()
                layers.append(LFM25LayerWeights(**shared, attention=LFM25AttentionWeights(
                    qkv, put(f"{p}.self_attn.out_proj.weight"), put(f"{p}.self_attn.q_layernorm.weight"),
                    put(f"{p}.self_attn.k_layernorm.weight"), n_attn)))
                n_attn += 1
            elif kind == "conv":
                conv_w = put(f"{p}.conv.conv.weight")
                if conv_w.ndim != 3 or conv_w.size(1) != 1:
                    raise ValueError(f"Expected depthwise conv weight [H,1,K], got {tuple(conv_w.shape)}")
                layers.append(LFM25LayerWeights(**shared, conv=LFM25ConvWeights(
                    put(f"{p}.conv.in_proj.weight"), conv_w[:, 0, :].contiguous(),
                    put(f"{p}.conv.out_proj.weight"), n_conv)))
                n_conv += 1
            else:
                raise ValueError(f"Unsupported LFM2 layer type: {kind!r}")
        return cls(config, embed, put("model.embedding_norm.weight"), head, tuple(layers), device, dtype)

    def tensors(self):
        """Every distinct packed tensor in a fixed order (the weight-broadcast schedule)."""
        seen, out = set(), []

        def add(t):
            if t.data_ptr() not in seen:
                seen.add(t.data_ptr())
                out.append(t)

        add(self.embed_tokens)
        add(self.embedding_norm_weight)
        add(self.lm_head_weight)
        for layer in self.layers:
            for t in (layer.operator_norm_weight, layer.ffn_norm_weight, layer.w13_weight, layer.w2_weight):
                add(t)
            if layer.attention is not None:
                a = layer.attention
                for t in (a.qkv_weight, a.out_weight, a.q_norm_weight, a.k_norm_weight):
                    add(t)
            if layer.conv is not None:
                c = layer.conv
                for t in (c.in_weight, c.conv_weight, c.out_weight):
                    add(t)
        return out

    @torch.inference_mode()
    def copy_from_model_(self, model: Any) -> None:
        """In-place policy sync; nothing is written unless every source tensor fits."""
        source_config = coerce_config(getattr(model, "config", None))
        source_config.validate()
        mismatches = [f"{name}: engine={getattr(self.config, name)!r}, model={getattr(source_config, name)!r}"
                      for name in _SYNC_FIELDS if getattr(self.config, name) != getattr(source_config, name)]
        if mismatches:
            raise ValueError("Cannot synchronize an incompatible LFM2 config (" + "; ".join(mismatches) + ")")
        state = model.state_dict()
        if not isinstance(state, Mapping):
            raise TypeError("model.state_dict() must return a mapping of tensor names to tensors")
        plan: list[tuple[torch.Tensor, torch.Tensor]] = []

        def stage(name: str, destination: torch.Tensor, source=None) -> None:
            source = _find(state, name) if source is None else source
            if not torch.is_tensor(source):
                raise TypeError(f"LFM25 sync source {name!r} is not a tensor")
            if tuple(source.shape) != tuple(destination.shape):
                raise ValueError(f"LFM25 sync shape mismatch for {name!r}: expected {tuple(destination.shape)}, "
                                 f"got {tuple(source.shape)}")
            plan.append((destination, source))

        cfg = source_config
        stage("model.embed_tokens.weight", self.embed_tokens)
        stage("model.embedding_norm.weight", self.embedding_norm_weight)
        stage("model.lm_head.weight", self.lm_head_weight,
              _find(state, "model.lm_head.weight" if _has(state, "model.lm_head.weight") else "model.embed_tokens.weight"))
        f = int(cfg.mlp_hidden_size)
        q_rows = int(cfg.num_attention_heads * cfg.head_dim)
        kv_rows = int(cfg.num_key_value_heads * cfg.head_dim)
        for index, (kind, layer) in enumerate(zip(cfg.layer_types, self.layers, strict=True)):
            p = f"model.layers.{index}"
            stage(f"{p}.operator_norm.weight", layer.operator_norm_weight)
            stage(f"{p}.ffn_norm.weight", layer.ffn_norm_weight)
            stage(f"{p}.feed_forward.w1.weight", layer.w13_weight[:f])
            stage(f"{p}.feed_forward.w3.weight", layer.w13_weight[f:])
            stage(f"{p}.feed_forward.w2.weight", layer.w2_weight)
            if kind == "full_attention":
                a = layer.attention
                if a is None or layer.conv is not None:
                    raise ValueError(f"LFM25 packed layer {index} does not match full_attention config")
                stage(f"{p}.self_attn.q_proj.weight", a.qkv_weight[:q_rows])
                stage(f"{p}.self_attn.k_proj.weight", a.qkv_weight[q_rows:q_rows + kv_rows])
                stage(f"{p}.self_attn.v_proj.weight", a.qkv_weight[q_rows + kv_rows:])
                stage(f"{p}.self_attn.out_proj.weight", a.out_weight)
                stage(f"{p}.self_attn.q_layernorm.weight", a.q_norm_weight)
                stage(f"{p}.self_attn.k_layernorm.weight", a.k_norm_weight)
            else:
                c = layer.conv
                if c is None or layer.attention is not None:
                    raise ValueError(f"LFM25 packed layer {index} does not match conv config")
                stage(f"{p}.conv.in_proj.weight", c.in_weight)
                name = f"{p}.conv.conv.weight"
                taps = _find(state, name)
                want = (c.conv_weight.size(0), 1, c.conv_weight.size(1))
                if not torch.is_tensor(taps):
                    raise TypeError(f"LFM25 sync source {name!r} is not a tensor")
                if tuple(taps.shape) != want:
                    raise ValueError(f"LFM25 sync shape mismatch for {name!r}: expected {want}, got {tuple(taps.shape)}")
                plan.append((c.conv_weight, taps[:, 0, :]))
                stage(f"{p}.conv.out_proj.weight", c.out_weight)
        for destination, source in plan:
            destination.copy_(source.detach(), non_blocking=False)


def load_state_dict(model_dir: Path) -> dict:
    """safetensors first, then .pt / .bin (optionally wrapped in {'state_dict'|'model': ...})."""
    files = sorted(model_dir.glob("*.safetensors"))
    if files:
        from safetensors.torch import load_file

        return load_file(files[0], device="cpu")
    files = sorted(model_dir.glob("*.pt")) or sorted(model_dir.glob("*.bin"))
    if files:
        payload = torch.load(files[0], map_location="cpu", weights_only=False)
        if isinstance(payload, dict):
            for key in ("state_dict", "model"):
                if isinstance(payload.get(key), dict):
                    return payload[key]
            return payload
    raise FileNotFoundError(f"No safetensors, .pt, or .bin weights found in: {model_dir}")


class PackedFP8Weight:
    """e4m3 copy of one projection with per-output-channel fp32 scales, refreshed in place after a
    policy sync so captured graphs keep valid addresses (reference: lfm25_fp8.py:119-135)."""

    def __init__(self, original: torch.Tensor):
        if original.dtype != torch.bfloat16 or original.ndim != 2 or not original.is_contiguous():
            raise ValueError("FP8 quantization requires a contiguous 2D CUDA BF16 tensor")
        self.original = original
        self.values = torch.empty(original.shape, device=original.device, dtype=torch.uint8)
        self.scales = torch.empty(original.size(0), device=original.device, dtype=torch.float32)
        self.refresh()

    def refresh(self) -> None:
        rows, width = self.original.shape
        nv.call("cgym_quantize_rows", nv.ptr(self.values), nv.ptr(self.scales), nv.ptr(self.original), rows, width,
                nv.BF16, nv.stream_ptr(self.original.device))


class PackedBF16Weight:
    """Lossless 12-bit stream of a bf16 matrix for single-request decode (reference:
    src/climbing_gym/inference/lfm25_bf16.py:61-102). ``original`` stays the matrix every other path uses;
    ``mantissa`` / ``exponent`` are refreshed in place after a policy sync, so captured graphs keep their
    addresses."""

    def __init__(self, original: torch.Tensor, base: int = 110):
        if original.dtype != torch.bfloat16 or not original.is_cuda or not original.is_contiguous():
            raise ValueError("lossless BF16 packing requires contiguous CUDA BF16 weights")
        if original.ndim != 2 or original.size(1) % 2:
            raise ValueError("lossless BF16 packing requires a matrix with even input width")
        self.original, self.base = original, base
        self.mantissa = torch.empty(original.shape, device=original.device, dtype=torch.uint8)
        self.exponent = torch.empty((original.size(0), original.size(1) // 2), device=original.device, dtype=torch.uint8)
        self.refresh()

    @classmethod
    def from_weight(cls, weight: torch.Tensor) -> "PackedBF16Weight":
        return cls(weight)

    def refresh(self) -> None:
        nv.call("cgym_bf16_stream_pack", nv.ptr(self.mantissa), nv.ptr(self.exponent), nv.ptr(self.original),
                self.original.numel(), self.base, nv.stream_ptr(self.original.device))

    def unpack(self) -> torch.Tensor:
        out = torch.empty_like(self.original)
        nv.call("cgym_bf16_stream_unpack", nv.ptr(out), nv.ptr(self.original), nv.ptr(self.mantissa),
                nv.ptr(self.exponent), out.numel(), self.base, nv.stream_ptr(out.device))
        return out

    def linear(self, x: torch.Tensor, out: torch.Tensor | None = None, row_mask: torch.Tensor | None = None) -> torch.Tensor:
        rows, width = self.original.shape
        if tuple(x.shape) != (1, width) or x.dtype != torch.bfloat16 or not x.is_contiguous():
            raise ValueError("packed BF16 GEMV requires one contiguous BF16 input row")
        out = torch.empty((1, rows), device=x.device, dtype=x.dtype) if out is None else out
        nv.call("cgym_bf16_stream_gemv", nv.ptr(out), nv.ptr(x), nv.ptr(self.original), nv.ptr(self.mantissa),
                nv.ptr(self.exponent), nv.ptr(row_mask), rows, width, self.base, nv.stream_ptr(x.device))
        return out


def describe_lfm25_checkpoint(model_dir) -> dict:
    config = LFM2Config.from_pretrained(model_dir)
    attention = [i for i, kind in enumerate(config.layer_types) if kind == "full_attention"]
    conv = [i for i, kind in enumerate(config.layer_types) if kind == "conv"]
    return {
        "model_dir": str(Path(model_dir).expanduser().resolve()),
        "num_hidden_layers": config.num_hidden_layers, "attention_layers": attention, "conv_layers": conv,
        "hidden_size": config.hidden_size, "num_attention_heads": config.num_attention_heads,
        "num_key_value_heads": config.num_key_value_heads, "head_dim": config.head_dim,
        "mlp_hidden_size": config.mlp_hidden_size, "conv_kernel_size": config.conv_kernel_size,
        "vocab_size": config.vocab_size, "tie_embedding": config.tie_embedding,
        "max_position_embeddings": config.max_position_embeddings,
        "kv_bytes_per_token_per_sequence_bf16": len(attention) * 2 * config.num_key_value_heads * config.head_dim * 2,
        "conv_state_bytes_per_sequence_bf16": len(conv) * config.hidden_size * config.conv_kernel_size * 2,
    }


def write_checkpoint_description(model_dir, output_path) -> Path:
    path = Path(output_path)
    path.parent.mkdir(parents=True, exist_ok=True)
    path.write_text(json.dumps(describe_lfm25_checkpoint(model_dir), indent=2) + "\n", encoding="utf-8")
    return path


def load_tokenizer(model_dir, **kwargs):
    """The checkpoint's tokenizer (models/lfm2_compat.py:36-48 of the reference): AutoTokenizer, or the
    generic fast tokenizer when the export names a tokenizer class this transformers does not know."""
    from transformers import AutoTokenizer, PreTrainedTokenizerFast

    try:
        return AutoTokenizer.from_pretrained(str(model_dir), **kwargs)
    except ValueError as exc:
        if "does not exist" not in str(exc):
            raise
        return PreTrainedTokenizerFast.from_pretrained(str(model_dir), **kwargs)
