"""Seeded inputs shared by the golden-vector generator and the tests that replay them.

Everything is numpy (PCG64) and already rounded to bf16-representable fp32, so both the
reference kernels (generator side) and the oracle / CUDA kernels (test side) see the
same bits.
"""
from __future__ import annotations

import numpy as np


def _bf16(x):
    x = np.ascontiguousarray(x, dtype=np.float32)
    bits = x.view(np.uint32)
    lsb = (bits >> np.uint32(16)) & np.uint32(1)
    return ((bits + np.uint32(0x7FFF) + lsb) & np.uint32(0xFFFF0000)).view(np.float32)


def kernel_inputs() -> dict:
    rng = np.random.default_rng(11)
    rows, h, f = 3, 256, 384
    hq, hkv, d = 4, 2, 64
    out = dict(rows=rows, h=h, f=f, hq=hq, hkv=hkv, d=d, eps=1e-5)
    out["x"] = _bf16(rng.standard_normal((rows, h)))
    out["res"] = _bf16(rng.standard_normal((rows, h)))
    out["norm_w"] = _bf16(1 + 0.1 * rng.standard_normal(h))
    out["gate_up"] = _bf16(2.0 * rng.standard_normal((rows, 2 * f)))
    out["bcx"] = _bf16(rng.standard_normal((rows, 3 * h)))
    out["conv_w"] = _bf16(0.3 * rng.standard_normal((h, 3)))
    out["conv_state"] = _bf16(rng.standard_normal((5, h, 3)))  # 5 physical slots
    out["conv_active"] = np.array([True, False, True])
    out["conv_slots"] = np.array([4, 1, 0], dtype=np.int32)
    out["qkv"] = _bf16(rng.standard_normal((rows, (hq + 2 * hkv) * d)))
    out["q_norm_w"] = _bf16(1 + 0.1 * rng.standard_normal(d))
    out["k_norm_w"] = _bf16(1 + 0.1 * rng.standard_normal(d))
    out["positions"] = np.array([0, 17, 4093], dtype=np.int32)
    out["rope_theta"] = 1_000_000.0
    out["rope_len"] = 4096
    wide = _bf16(rng.standard_normal((rows, 512)) * np.array([[1.0], [30.0], [1e-3]]))
    wide[2, :] = 0.0  # an all-zero row exercises the 1e-12 scale floor
    out["quant_x"] = wide
    return out


def rope_tables(theta: float, length: int, dim: int):
    """fp32 cos/sin tables [length, dim/2], computed with torch on CPU exactly as the
    reference engine builds them (src/climbing_gym/inference/lfm25_engine.py:1004-1012)."""
    import torch

    inv = 1.0 / (theta ** (torch.arange(0, dim, 2, dtype=torch.float32) / dim))
    freqs = torch.einsum("i,j->ij", torch.arange(length, dtype=torch.float32), inv)
    return freqs.cos().numpy(), freqs.sin().numpy()
