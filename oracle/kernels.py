"""Per-kernel CPU restatements of the reference's fused decode kernels (TEST INFRASTRUCTURE).

Each function follows one Triton kernel of the reference and applies the model-dtype cast
(``rd``) at exactly the points that kernel does. Pinned bit-for-bit by
``tests/golden/kernels.json`` (the reference kernels run under Triton's CPU interpreter).
"""
from __future__ import annotations

import numpy as np

from .numerics import decode_e4m3, encode_e4m3, quantize_rows_e4m3, round_bf16


def rms_norm(x, w, eps, residual=None, rd=round_bf16):
    """lfm25_cuda_kernels.py:32-44: optional residual add rounded first and returned,
    fp32 mean square, normalised value rounded, then times weight and rounded on store."""
    x = np.asarray(x, np.float32)
    summed = x
    if residual is not None:
        summed = rd(x + np.asarray(residual, np.float32))
    var = np.sum(summed * summed, axis=-1, keepdims=True, dtype=np.float32) / np.float32(x.shape[-1])
    normalized = rd(summed * (np.float32(1.0) / np.sqrt(var + np.float32(eps))))
    return rd(normalized * w), summed


def swiglu(gate_up, rd=round_bf16):
    """lfm25_cuda_kernels.py:58-65: bf16(silu(gate)) * up."""
    f = gate_up.shape[-1] // 2
    gate, up = gate_up[..., :f], gate_up[..., f:]
    act = rd(gate / (np.float32(1.0) + np.exp(-gate, dtype=np.float32)))
    return rd(act * up)


def conv_update(bcx, w, state, active=None, slots=None, rd=round_bf16):
    """lfm25_cuda_kernels.py:75-100. ``state`` [slots, H, 3] is updated in place for active rows."""
    rows, h = bcx.shape[0], w.shape[0]
    y = np.empty((rows, h), np.float32)
    for row in range(rows):
        slot = max(int(slots[row]), 0) if slots is not None else row
        b, c, x = bcx[row, :h], bcx[row, h:2 * h], bcx[row, 2 * h:]
        bx = rd(b * x)
        s0, s1 = state[slot, :, 1].copy(), state[slot, :, 2].copy()
        conv = rd(rd(s0 * w[:, 0]) + rd(s1 * w[:, 1]) + rd(bx * w[:, 2]))
        if active is None or bool(active[row]):
            state[slot, :, 0], state[slot, :, 1], state[slot, :, 2] = s0, s1, bx
        y[row] = rd(c * conv)
    return y


def qkv_rope(qkv, q_w, k_w, cos, sin, positions, hq, hkv, d, eps, rd=round_bf16):
    """lfm25_cuda_kernels.py:113-140: per-head RMSNorm, weight, half-split RoPE, V copied."""
    rows = qkv.shape[0]
    heads = qkv.reshape(rows, hq + 2 * hkv, d)
    out = []
    for lo, hi, w in ((0, hq, q_w), (hq, hq + hkv, k_w)):
        x = heads[:, lo:hi]
        ms = np.sum(x * x, -1, keepdims=True, dtype=np.float32) / np.float32(d)
        n = rd(x * (np.float32(1.0) / np.sqrt(ms + np.float32(eps))))
        n = rd(n * w)
        other = np.concatenate([n[..., d // 2:], n[..., :d // 2]], -1)
        c = rd(np.concatenate([cos[positions], cos[positions]], -1))[:, None, :]
        s = rd(np.concatenate([sin[positions], sin[positions]], -1))[:, None, :]
        left, right = rd(n * c), rd(other * s)
        sign = np.where(np.arange(d) < d // 2, -1.0, 1.0).astype(np.float32)
        out.append(rd(left + sign * right))
    return out[0], out[1], heads[:, hq + hkv:].copy()


def quantize_rows(x):
    """lfm25_fp8.py:16-23 -> (e4m3 codes uint8, fp32 scales)."""
    return quantize_rows_e4m3(x)


def rms_quantize(x, w, eps, residual=None, rd=round_bf16):
    """lfm25_fp8.py:26-41: RMSNorm output rounded to the model dtype, then row-quantised."""
    y, summed = rms_norm(x, w, eps, residual, rd)
    codes, scales = quantize_rows_e4m3(y)
    return codes, scales, summed


def swiglu_quantize(gate_up, rd=round_bf16):
    """lfm25_fp8.py:44-54."""
    return quantize_rows_e4m3(swiglu(gate_up, rd))


def fp8_matmul(a_codes, a_scales, w_codes, w_scales, rd=round_bf16):
    """lfm25_fp8.py:76-93: exact e4m3 products, fp32 accumulate, x a_scale[m] then x w_scale[n]."""
    acc = decode_e4m3(a_codes).astype(np.float32) @ decode_e4m3(w_codes).astype(np.float32).T
    acc = acc * np.asarray(a_scales, np.float32)[:, None]
    acc = acc * np.asarray(w_scales, np.float32)[None, :]
    return rd(acc)


def store_kv_e4m3(k):
    """lfm25_fp8_kv.py:47-55: per (token, head) scale, cvt.rn.satfinite of k/scale."""
    k = np.asarray(k, np.float32)
    scale = np.maximum(np.max(np.abs(k), -1) / np.float32(448.0), np.float32(1e-12)).astype(np.float32)
    return encode_e4m3(k / scale[..., None]), scale


def record_sample(sampled, logp, st, *, eos, vocab):
    """lfm25_session.py:34-56, in place on the dict of per-slot arrays ``st``.

    Keys: tokens [S,CAP], logprobs, lengths, limits, reasons, alive, pending, input,
    stop_states, stop_offsets, stop_table (flat), ignore_eos, rng_positions.
    """
    for row in range(len(sampled)):
        if not st["alive"][row]:
            continue
        token, length = int(sampled[row]), int(st["lengths"][row])
        st["tokens"][row, length] = token
        st["logprobs"][row, length] = logp[row]
        value = int(st["stop_table"][int(st["stop_offsets"][row]) + int(st["stop_states"][row]) * vocab + token])
        st["stop_states"][row] = value & 65535
        if token == eos and not st["ignore_eos"][row]:
            reason = 1
        elif value >= 65536:
            reason = 2
        elif length + 1 >= int(st["limits"][row]):
            reason = 3
        else:
            reason = 0
        st["lengths"][row] = length + 1
        st["rng_positions"][row] += 1
        st["reasons"][row] = reason
        st["alive"][row] = reason == 0
        st["pending"][row] = reason == 0
        st["input"][row] = token


def behavior_head(logits, selected, logp, k):
    """lfm25_sampling.py:127-149: the k largest logits of every row (descending; torch.topk leaves the
    order of equal values open, this restatement takes the lowest ids first) and their log-probs
    against the partition function the sampler already produced: log Z = logit[selected] - logp."""
    logits = np.asarray(logits, np.float32)
    if not 0 < k <= min(logits.shape[1], 128):
        raise ValueError("Behavior head exceeds the vocabulary or supported size")
    ids = np.stack([np.lexsort((np.arange(row.size), -row))[:k] for row in logits]).astype(np.int32)
    values = np.take_along_axis(logits, ids, 1)
    log_z = logits[np.arange(len(logits)), np.asarray(selected)] - np.asarray(logp, np.float32)
    return ids, (values - log_z[:, None]).astype(np.float32)


def record_head(ids, probs, out_ids, out_probs, lengths, alive):
    """lfm25_session.py:20-30: live rows store their head at [row, lengths[row]] (before record_sample
    advances the length)."""
    for row in range(len(ids)):
        if alive[row]:
            out_ids[row, int(lengths[row])] = ids[row]
            out_probs[row, int(lengths[row])] = probs[row]


def apply_repetition_penalty(logits, seen, penalty):
    """lfm25_engine.py:1777-1791: fp32 logits of seen tokens are multiplied by the penalty when negative
    and divided by it otherwise."""
    logits = np.asarray(logits, np.float32)
    if seen is None or penalty == 1.0:
        return logits
    if penalty <= 0.0:
        raise ValueError("repetition penalty must be > 0")
    p = np.float32(penalty)
    return np.where(np.asarray(seen, bool), np.where(logits < 0, logits * p, logits / p), logits).astype(np.float32)
