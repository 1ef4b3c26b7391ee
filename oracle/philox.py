"""Philox-4x32-10 counter RNG for the sampler oracle (TEST INFRASTRUCTURE).

The reference sampler draws its uniforms from Triton's ``tl.rand(seed, offset)``
(src/climbing_gym/inference/lfm25_sampling.py:17-26), a dependency that is not part of
the reference tree (``triton>=3.6,<3.7``, pyproject.toml). This file restates the
published algorithm it implements: Philox-4x32 with 10 rounds (Salmon et al., "Parallel
Random Numbers: As Easy as 1, 2, 3", SC'11) keyed with the 64-bit seed split into two
32-bit key words, counter ``(offset, 0, 0, 0)``, first output word, mapped to [0, 1) by
folding the sign of the int32 reinterpretation and scaling by 2**-31.

Keying follows the reference call sites: batch mode uses key
``(seed + step * 0x9E3779B97F4A7C15) & (2**63 - 1)`` and offset ``row * V + col``
(lfm25_sampling.py:25,83); per-row mode uses the row's own seed and generated-token
position in the same formula and offset ``col`` (lfm25_sampling.py:19-21).
"""
from __future__ import annotations

import numpy as np

_MULT_A = np.uint64(0xD2511F53)
_MULT_B = np.uint64(0xCD9E8D57)
_KEY_A = np.uint32(0x9E3779B9)
_KEY_B = np.uint32(0xBB67AE85)
GOLDEN64 = 0x9E3779B97F4A7C15
MASK63 = 0x7FFFFFFFFFFFFFFF
UNIFORM_SCALE = np.float32(4.6566127342e-10)


def step_key(seed: int, step: int) -> int:
    return (int(seed) + int(step) * GOLDEN64) & MASK63


def philox4x32_10(c0: np.ndarray, key: int) -> np.ndarray:
    """First output word for counters (c0, 0, 0, 0) under a 64-bit key."""
    c0 = np.asarray(c0).astype(np.uint32)
    c1 = np.zeros_like(c0)
    c2 = np.zeros_like(c0)
    c3 = np.zeros_like(c0)
    k0 = np.uint32(key & 0xFFFFFFFF)
    k1 = np.uint32((key >> 32) & 0xFFFFFFFF)
    with np.errstate(over="ignore"):
        for _ in range(10):
            pa = c0.astype(np.uint64) * _MULT_A
            pb = c2.astype(np.uint64) * _MULT_B
            hi_a, lo_a = (pa >> np.uint64(32)).astype(np.uint32), pa.astype(np.uint32)
            hi_b, lo_b = (pb >> np.uint64(32)).astype(np.uint32), pb.astype(np.uint32)
            c0, c1, c2, c3 = hi_b ^ c1 ^ k0, lo_b, hi_a ^ c3 ^ k1, lo_a
            k0 = np.uint32((int(k0) + int(_KEY_A)) & 0xFFFFFFFF)
            k1 = np.uint32((int(k1) + int(_KEY_B)) & 0xFFFFFFFF)
    return c0


def uniform(offsets: np.ndarray, key: int) -> np.ndarray:
    """fp32 uniforms in [0, 1): int32 view, negative values folded by ``-x-1``, times 2**-31."""
    word = philox4x32_10(offsets, key).view(np.int32).astype(np.int64)
    folded = np.where(word < 0, -word - 1, word)
    return (folded.astype(np.float32) * UNIFORM_SCALE).astype(np.float32)
