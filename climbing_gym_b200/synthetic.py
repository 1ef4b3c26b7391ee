"""Seeded synthetic checkpoints and request streams for parity tests and benchmarks.

No LFM2.5 weights, tokenizer or task prompts are available offline, so every
measurement and parity case runs on random-init weights of the named architecture
and seeded random token ids whose length distributions follow the workload being
stood in for. Generation is numpy-only (PCG64) so the same seed rebuilds the same
arrays on any machine without the reference installed.

State-dict keys are the Hugging Face LFM2 names the engine's packer consumes
(``model.layers.N.{operator_norm,ffn_norm,feed_forward.w{1,2,3},conv.*,self_attn.*}``).
"""
from __future__ import annotations

import numpy as np

from .config import LFM2Config


def tiny_config(**overrides) -> LFM2Config:
    """The CPU-runnable plumbing model: hidden 256, conv/conv/attn/conv, 4q/2kv heads."""
    values = dict(vocab_size=4096, hidden_size=256, mlp_hidden_size=768, num_hidden_layers=4,
                  layer_types=("conv", "conv", "full_attention", "conv"), num_attention_heads=4,
                  num_key_value_heads=2, rope_theta=1_000_000.0, eos_token_id=2)
    values.update(overrides)
    config = LFM2Config(**values)
    config.validate()
    return config


def lfm25_1p2b_config() -> LFM2Config:
    return LFM2Config()


def make_state_dict(config: LFM2Config, seed: int = 0, *, std: float = 0.02,
                    untied_head: bool = False) -> dict[str, np.ndarray]:
    """Normal(0, std) matrices, norm weights 1 + 0.1 N(0,1), conv taps 0.3 N(0,1)."""
    rng = np.random.default_rng(seed)
    h, f, v = config.hidden_size, config.mlp_hidden_size, config.vocab_size
    d, hq, hkv = config.head_dim, config.num_attention_heads, config.num_key_value_heads

    def mat(*shape):
        return (rng.standard_normal(shape, dtype=np.float32) * np.float32(std)).astype(np.float32)

    def norm(n):
        return (1.0 + 0.1 * rng.standard_normal(n, dtype=np.float32)).astype(np.float32)

    state = {"model.embed_tokens.weight": mat(v, h), "model.embedding_norm.weight": norm(h)}
    if untied_head:
        state["model.lm_head.weight"] = mat(v, h)
    for index, kind in enumerate(config.layer_types):
        p = f"model.layers.{index}"
        state[f"{p}.operator_norm.weight"] = norm(h)
        state[f"{p}.ffn_norm.weight"] = norm(h)
        state[f"{p}.feed_forward.w1.weight"] = mat(f, h)
        state[f"{p}.feed_forward.w3.weight"] = mat(f, h)
        state[f"{p}.feed_forward.w2.weight"] = mat(h, f)
        if kind == "conv":
            state[f"{p}.conv.in_proj.weight"] = mat(3 * h, h)
            state[f"{p}.conv.conv.weight"] = (0.3 * rng.standard_normal(
                (h, 1, config.conv_kernel_size), dtype=np.float32)).astype(np.float32)
            state[f"{p}.conv.out_proj.weight"] = mat(h, h)
        else:
            state[f"{p}.self_attn.q_proj.weight"] = mat(hq * d, h)
            state[f"{p}.self_attn.k_proj.weight"] = mat(hkv * d, h)
            state[f"{p}.self_attn.v_proj.weight"] = mat(hkv * d, h)
            state[f"{p}.self_attn.out_proj.weight"] = mat(h, hq * d)
            state[f"{p}.self_attn.q_layernorm.weight"] = norm(d)
            state[f"{p}.self_attn.k_layernorm.weight"] = norm(d)
    return state


def make_state_dict_streams(config: LFM2Config, seed: int = 0, *, std: float = 0.02,
                            untied_head: bool = False, workers: int | None = None) -> dict[str, np.ndarray]:
    """Same distributions as make_state_dict, but every tensor is drawn from its own PCG64 stream
    (seeded by ``(seed, position of the tensor)``) so the tensors can be generated on a thread pool:
    a 1.2 B-parameter checkpoint takes seconds per core instead of minutes on one. The values differ
    from make_state_dict's for the same seed; they are reproducible on any machine with numpy alone,
    which is what lets fixtures computed elsewhere be compared against an engine built here."""
    import os
    from concurrent.futures import ThreadPoolExecutor

    h, f, v = config.hidden_size, config.mlp_hidden_size, config.vocab_size
    d, hq, hkv = config.head_dim, config.num_attention_heads, config.num_key_value_heads
    plan: list[tuple[str, str, tuple]] = [("model.embed_tokens.weight", "mat", (v, h)),
                                          ("model.embedding_norm.weight", "norm", (h,))]
    if untied_head:
        plan.append(("model.lm_head.weight", "mat", (v, h)))
    for index, kind in enumerate(config.layer_types):
        p = f"model.layers.{index}"
        plan += [(f"{p}.operator_norm.weight", "norm", (h,)), (f"{p}.ffn_norm.weight", "norm", (h,)),
                 (f"{p}.feed_forward.w1.weight", "mat", (f, h)), (f"{p}.feed_forward.w3.weight", "mat", (f, h)),
                 (f"{p}.feed_forward.w2.weight", "mat", (h, f))]
        if kind == "conv":
            plan += [(f"{p}.conv.in_proj.weight", "mat", (3 * h, h)),
                     (f"{p}.conv.conv.weight", "taps", (h, 1, config.conv_kernel_size)),
                     (f"{p}.conv.out_proj.weight", "mat", (h, h))]
        else:
            plan += [(f"{p}.self_attn.q_proj.weight", "mat", (hq * d, h)),
                     (f"{p}.self_attn.k_proj.weight", "mat", (hkv * d, h)),
                     (f"{p}.self_attn.v_proj.weight", "mat", (hkv * d, h)),
                     (f"{p}.self_attn.out_proj.weight", "mat", (h, hq * d)),
                     (f"{p}.self_attn.q_layernorm.weight", "norm", (d,)),
                     (f"{p}.self_attn.k_layernorm.weight", "norm", (d,))]

    def draw(item):
        position, (name, kind, shape) = item
        rng = np.random.default_rng([int(seed), position])
        values = rng.standard_normal(shape, dtype=np.float32)
        if kind == "mat":
            values *= np.float32(std)
        elif kind == "norm":
            values = (1.0 + 0.1 * values).astype(np.float32)
        else:
            values *= np.float32(0.3)
        return name, values

    with ThreadPoolExecutor(workers or min(32, os.cpu_count() or 1)) as pool:
        return dict(pool.map(draw, enumerate(plan)))


def make_state_dict_on_device(config: LFM2Config, seed: int, device, dtype, *, std: float = 0.02,
                              untied_head: bool = False) -> dict:
    """Same distributions as make_state_dict, drawn with torch's generator directly on ``device``
    (benchmark-sized models: 1.2 B normals are drawn in a fraction of a second on the GPU)."""
    import torch

    gen = torch.Generator(device=device)
    gen.manual_seed(int(seed))
    h, f, v = config.hidden_size, config.mlp_hidden_size, config.vocab_size
    d, hq, hkv = config.head_dim, config.num_attention_heads, config.num_key_value_heads

    def mat(*shape):
        return (torch.randn(shape, generator=gen, device=device, dtype=torch.float32) * std).to(dtype)

    def norm(n):
        return (1.0 + 0.1 * torch.randn(n, generator=gen, device=device, dtype=torch.float32)).to(dtype)

    state = {"model.embed_tokens.weight": mat(v, h), "model.embedding_norm.weight": norm(h)}
    if untied_head:
        state["model.lm_head.weight"] = mat(v, h)
    for index, kind in enumerate(config.layer_types):
        p = f"model.layers.{index}"
        state[f"{p}.operator_norm.weight"] = norm(h)
        state[f"{p}.ffn_norm.weight"] = norm(h)
        state[f"{p}.feed_forward.w1.weight"] = mat(f, h)
        state[f"{p}.feed_forward.w3.weight"] = mat(f, h)
        state[f"{p}.feed_forward.w2.weight"] = mat(h, f)
        if kind == "conv":
            state[f"{p}.conv.in_proj.weight"] = mat(3 * h, h)
            state[f"{p}.conv.conv.weight"] = (0.3 * torch.randn((h, 1, config.conv_kernel_size), generator=gen,
                                                                device=device, dtype=torch.float32)).to(dtype)
            state[f"{p}.conv.out_proj.weight"] = mat(h, h)
        else:
            state[f"{p}.self_attn.q_proj.weight"] = mat(hq * d, h)
            state[f"{p}.self_attn.k_proj.weight"] = mat(hkv * d, h)
            state[f"{p}.self_attn.v_proj.weight"] = mat(hkv * d, h)
            state[f"{p}.self_attn.out_proj.weight"] = mat(h, hq * d)
            state[f"{p}.self_attn.q_layernorm.weight"] = norm(d)
            state[f"{p}.self_attn.k_layernorm.weight"] = norm(d)
    return state


def uniform_prompts(count: int, low: int, high: int, vocab: int, seed: int = 0,
                    *, first_id: int = 3) -> list[list[int]]:
    """``count`` prompts, lengths uniform in [low, high], ids uniform in [first_id, vocab)."""
    rng = np.random.default_rng(seed)
    lengths = rng.integers(low, high + 1, size=count)
    return [rng.integers(first_id, vocab, size=int(n)).tolist() for n in lengths]


def lognormal_prompts(count: int, median: float, sigma: float, low: int, high: int, vocab: int,
                      seed: int = 0, *, first_id: int = 3) -> list[list[int]]:
    """Prompt lengths clip(lognormal(ln median, sigma), low, high) (continuous-batching queue)."""
    rng = np.random.default_rng(seed)
    lengths = np.clip(np.exp(rng.normal(np.log(median), sigma, size=count)), low, high).astype(np.int64)
    return [rng.integers(first_id, vocab, size=int(n)).tolist() for n in lengths]


def geometric_lengths(count: int, mean: float, cap: int, seed: int = 0, *, low: int = 1) -> list[int]:
    """Output lengths from a constant per-token EOS hazard 1/mean, capped (stands in for EOS)."""
    rng = np.random.default_rng(seed)
    return np.clip(rng.geometric(1.0 / mean, size=count), low, cap).astype(np.int64).tolist()
