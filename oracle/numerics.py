"""Rounding primitives for the CPU oracle (TEST INFRASTRUCTURE, never the product path).

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline legs may
import this package. It restates, in numpy, the rounding points of the reference's
LFM2.5 rollout engine so the CUDA path can be compared with it bit-for-bit where the
arithmetic is elementwise and within stated tolerances where a reduction order differs.

* bf16 rounding: IEEE round-to-nearest-even of an fp32 value to 8 mantissa bits, the
  conversion ``tensor.to(torch.bfloat16)`` performs at every point the reference's fused
  kernels cast (src/climbing_gym/inference/lfm25_cuda_kernels.py:39,42,64,84,92-95).
* e4m3 rounding: ``cvt.rn.satfinite.e4m3x2.f32`` semantics used by the reference's KV
  store (src/climbing_gym/inference/lfm25_fp8_kv.py:14-25) and, after the explicit
  clamp to +-448, by its row quantiser (src/climbing_gym/inference/lfm25_fp8.py:16-23).
"""
from __future__ import annotations

import numpy as np

E4M3_MAX = 448.0


def round_bf16(x: np.ndarray) -> np.ndarray:
    """fp32 -> nearest-even bf16 -> fp32 (NaN/Inf preserved)."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    bits = x.view(np.uint32)
    lsb = (bits >> np.uint32(16)) & np.uint32(1)
    rounded = (bits + np.uint32(0x7FFF) + lsb) & np.uint32(0xFFFF0000)
    nan = np.isnan(x)
    out = rounded.view(np.float32).copy()
    if nan.any():
        out[nan] = np.nan
    return out


def truncate_bf16(x: np.ndarray) -> np.ndarray:
    """fp32 -> bf16 by dropping the low 16 bits.

    NOT what the GPU does (PTX ``cvt.rn.bf16.f32`` rounds to nearest even). It is what
    Triton's CPU interpreter does for fp32->bf16 casts, so vectors produced by running the
    reference kernels under that interpreter are compared in this mode: it checks that the
    oracle casts at the same points, while ``round_bf16`` carries the real rounding mode.
    """
    x = np.ascontiguousarray(x, dtype=np.float32)
    return (x.view(np.uint32) & np.uint32(0xFFFF0000)).view(np.float32)


def bf16_bits(x: np.ndarray) -> np.ndarray:
    """Upper 16 bits of an already-bf16-representable fp32 array (for byte comparisons)."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    return (x.view(np.uint32) >> np.uint32(16)).astype(np.uint16)


def from_bf16_bits(bits: np.ndarray) -> np.ndarray:
    return (np.ascontiguousarray(bits).astype(np.uint32) << np.uint32(16)).view(np.float32)


def identity(x: np.ndarray) -> np.ndarray:
    return np.asarray(x, dtype=np.float32)


def rounder(dtype: str):
    """Return the cast the model dtype applies after each op ("fp32" -> none)."""
    if dtype in ("fp32", "float32"):
        return identity
    if dtype in ("bf16", "bfloat16"):
        return round_bf16
    raise ValueError(f"unsupported oracle dtype {dtype!r}")


def _e4m3_table() -> np.ndarray:
    """All 256 e4m3fn code points as fp32 (0x7F / 0xFF are NaN)."""
    codes = np.arange(256, dtype=np.uint32)
    sign = np.where(codes & 0x80, -1.0, 1.0)
    exp = (codes >> 3) & 0xF
    man = codes & 0x7
    value = np.where(exp == 0, man / 8.0 * 2.0 ** -6, (1.0 + man / 8.0) * 2.0 ** (exp.astype(np.float64) - 7))
    value = sign * value
    value[(codes & 0x7F) == 0x7F] = np.nan
    return value.astype(np.float32)


E4M3_VALUES = _e4m3_table()
_POS = E4M3_VALUES[:0x7F].astype(np.float64)  # 0 .. 448, ascending


def encode_e4m3_search(x: np.ndarray) -> np.ndarray:
    """fp32 -> e4m3fn code by searching the table of code points (slow; the definition the bit-wise
    encoder below is checked against)."""
    x = np.asarray(x, dtype=np.float32)
    mag = np.minimum(np.abs(x.astype(np.float64)), E4M3_MAX)
    hi = np.searchsorted(_POS, mag, side="left").clip(0, len(_POS) - 1)
    lo = (hi - 1).clip(0)
    d_hi = _POS[hi] - mag
    d_lo = mag - _POS[lo]
    pick_lo = (d_lo < d_hi) | ((d_lo == d_hi) & ((lo & 1) == 0))
    code = np.where(pick_lo, lo, hi).astype(np.uint8)
    code = np.where(np.signbit(x), code | 0x80, code).astype(np.uint8)
    return code


def encode_e4m3(x: np.ndarray) -> np.ndarray:
    """fp32 -> e4m3fn code (uint8), round-to-nearest-even, saturating to +-448.

    Bit-wise: above 2^-6 the fp32 mantissa is rounded to three bits (the carry runs into the exponent
    field, as it must) and the exponent re-biased from 127 to 7; below it the value is a multiple of
    2^-9, rounded half-to-even. Same codes as encode_e4m3_search, two orders of magnitude faster."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    mag = np.minimum(np.abs(x), np.float32(E4M3_MAX))
    bits = mag.view(np.uint32)
    lsb = (bits >> np.uint32(20)) & np.uint32(1)
    normal = ((bits + np.uint32(0x7FFFF) + lsb) >> np.uint32(20)).astype(np.int32) - np.int32(960)
    subnormal = np.rint(mag * np.float32(512.0)).astype(np.int32)
    code = np.where(mag < np.float32(2.0 ** -6), subnormal, normal).astype(np.uint8)
    return np.where(np.signbit(x), code | np.uint8(0x80), code).astype(np.uint8)


def decode_e4m3(code: np.ndarray) -> np.ndarray:
    return E4M3_VALUES[np.asarray(code, dtype=np.uint8)]


def quantize_rows_e4m3(x: np.ndarray) -> tuple[np.ndarray, np.ndarray]:
    """Per-row dynamic scale: scale = max(absmax/448, 1e-12); q = e4m3(clamp(x/scale)).

    Follows src/climbing_gym/inference/lfm25_fp8.py:16-23. Returns (codes uint8, scales fp32).
    Matrices of more than a few million elements are cut into row blocks that run on a thread pool
    (numpy releases the GIL inside its loops); rows are independent, so the result is the same.
    """
    x = np.asarray(x, dtype=np.float32)
    if x.ndim == 2 and x.size > (1 << 22):
        import os
        from concurrent.futures import ThreadPoolExecutor

        workers = min(32, os.cpu_count() or 1)
        bounds = np.linspace(0, x.shape[0], 4 * workers + 1).astype(int)
        blocks = [x[a:b] for a, b in zip(bounds[:-1], bounds[1:]) if b > a]
        with ThreadPoolExecutor(workers) as pool:
            parts = list(pool.map(_quantize_rows_block, blocks))
        return np.concatenate([p[0] for p in parts]), np.concatenate([p[1] for p in parts])
    return _quantize_rows_block(x)


def _quantize_rows_block(x: np.ndarray) -> tuple[np.ndarray, np.ndarray]:
    absmax = np.max(np.abs(x), axis=-1)
    scale = np.maximum(absmax / np.float32(448.0), np.float32(1.0e-12)).astype(np.float32)
    q = np.clip(x / scale[..., None], -448.0, 448.0).astype(np.float32)
    return encode_e4m3(q), scale
