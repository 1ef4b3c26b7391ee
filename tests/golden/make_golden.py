"""Regenerate tests/golden/*.json by running the reference implementation on CPU.

Run from the repository root in a container where the reference checkout is mounted:

    python tests/golden/make_golden.py --reference <reference checkout>/src

The reference is imported read-only and executed as-is: its eager ``LFM25Engine`` for the
model-level vectors, and its Triton kernels under Triton's CPU interpreter
(``TRITON_INTERPRET=1``) for the kernel-level vectors. Inputs come from
``climbing_gym_b200.synthetic`` (numpy PCG64) so tests rebuild them without the
reference. Only the outputs are stored.
"""
from __future__ import annotations

import argparse
import json
import os
import sys
from pathlib import Path

os.environ.setdefault("TRITON_INTERPRET", "1")
os.environ.setdefault("CUDA_VISIBLE_DEVICES", "")

import numpy as np
import torch

ROOT = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(ROOT))

from climbing_gym_b200 import synthetic  # noqa: E402

OUT = Path(__file__).resolve().parent


def ref_engine(ref, cfg, state, dtype, max_model_len=256):
    from climbing_gym.models.lfm2 import LFM2Config
    from climbing_gym.inference.lfm25_engine import LFM25Engine, LFM25PackedWeights

    rcfg = LFM2Config.from_dict({**cfg.to_dict(), "attn_backend": "eager"})
    tensors = {k: torch.from_numpy(v) for k, v in state.items()}
    weights = LFM25PackedWeights.from_state_dict(rcfg, tensors, device=torch.device("cpu"), dtype=dtype)
    return LFM25Engine(weights, max_model_len=max_model_len)


def force_eos(engine, force_at, eos):
    """Replace row r's token with EOS at generated position force_at[r] (sampler wrap,
    the reference tests' own technique: tests/test_text_stops.py:122-126)."""
    original = engine._sample
    state = {"step": 0, "alive": list(range(len(force_at)))}

    def wrapped(logits, sampling, **kwargs):
        tokens, raw, smp = original(logits, sampling, **kwargs)
        rows = state["alive"]
        assert len(rows) == logits.size(0)
        tokens = tokens.clone()
        for j, row in enumerate(rows):
            if force_at[row] == state["step"]:
                tokens[j] = eos
        lf = logits.float()
        raw = lf.gather(1, tokens[:, None]).squeeze(1) - torch.logsumexp(lf, dim=-1)
        state["alive"] = [row for j, row in enumerate(rows) if int(tokens[j]) != eos]
        state["step"] += 1
        return tokens, raw, raw

    engine._sample = wrapped


def generate_case(name, cfg, state, dtype, prompts, n_new, force_at=None, repeats=1):
    from climbing_gym.inference.lfm25_engine import LFM25SamplingConfig, flatten_token_batches

    engine = ref_engine(None, cfg, state, dtype)
    if force_at is not None:
        force_eos(engine, force_at, cfg.eos_token_id)
    out = engine.generate(*flatten_token_batches(prompts), repeats=repeats,
                          sampling=LFM25SamplingConfig(temperature=0.0, max_new_tokens=n_new))
    return dict(name=name, token_ids=out.token_ids.tolist(), lengths=out.lengths.tolist(),
                finish_reasons=out.finish_reasons.tolist(),
                logprobs=[[[round(float(x), 6) for x in r] for r in p] for p in out.logprobs.tolist()])


def model_vectors():
    from climbing_gym.inference.lfm25_engine import flatten_token_batches

    result = {}
    for tag, untied in (("untied", True), ("tied", False)):
        cfg = synthetic.tiny_config()
        state = synthetic.make_state_dict(cfg, seed=0, untied_head=untied)
        prompts = synthetic.uniform_prompts(8, 8, 64, cfg.vocab_size, seed=0)
        force_at = np.random.default_rng(1).integers(8, 33, size=8).tolist()
        for dname, dtype in (("fp32", torch.float32), ("bf16", torch.bfloat16)):
            result[f"generate_{tag}_{dname}"] = generate_case(f"{tag}_{dname}", cfg, state, dtype, prompts, 32)
            result[f"generate_eos_{tag}_{dname}"] = dict(
                generate_case(f"eos_{tag}_{dname}", cfg, state, dtype, prompts, 32, force_at=force_at),
                force_eos_at=force_at)
        # prefill logits (fp32): argmax, a slice of the row and its logsumexp
        engine = ref_engine(None, cfg, state, torch.float32)
        prefix = engine.prefill(*flatten_token_batches(prompts[:4]))
        logits = prefix.next_token_logits.float()
        result[f"prefill_{tag}_fp32"] = dict(
            argmax=logits.argmax(-1).tolist(), head=[[round(float(x), 6) for x in row[:16]] for row in logits],
            lse=[round(float(x), 6) for x in torch.logsumexp(logits, -1)])
        # repeats > 1 share one prompt prefill
        result[f"generate_repeats_{tag}_fp32"] = generate_case("repeats", cfg, state, torch.float32, prompts[:3], 8, repeats=2)
        completions = synthetic.uniform_prompts(4, 3, 12, cfg.vocab_size, seed=5)
        scores = engine.score_completions(prompts[:4], completions)
        result[f"score_{tag}_fp32"] = [[round(float(x), 6) for x in row] for row in scores]
    return result


def sampler_vectors():
    """Reference Triton sampler kernels, executed by Triton's CPU interpreter."""
    from climbing_gym.inference import lfm25_sampling as ref

    rng = np.random.default_rng(7)
    batch, vocab = 5, 9000  # three 4096-wide tiles, the last one ragged
    logits = torch.from_numpy((rng.standard_normal((batch, vocab)) * 2.0).astype(np.float32))
    logits[1, 17] = logits[1, 4500] = 9.0  # tie across tiles: lowest index wins
    logits[2, :4096] = -float("inf")  # one fully masked tile
    parts = -(-vocab // 4096)
    out = {"batch": batch, "vocab": vocab, "cases": []}

    def run(per_row, temperature, seed, step, seeds=None, steps=None, temps=None):
        scores = torch.empty((batch, parts)); indices = torch.empty((batch, parts), dtype=torch.int32)
        maxima = torch.empty_like(scores); totals = torch.empty_like(scores)
        tokens = torch.empty(batch, dtype=torch.long); logp = torch.empty(batch)
        if per_row:
            ref._partial_sample[(batch, parts)](logits, scores, indices, maxima, totals, seeds, vocab, parts,
                                               1., True, 4096, steps, temps, True)
        else:
            key = (int(seed) + int(step) * 0x9E3779B97F4A7C15) & 0x7FFFFFFFFFFFFFFF
            ref._partial_sample[(batch, parts)](logits, scores, indices, maxima, totals, key, vocab, parts,
                                               temperature, True, 4096)
        ref._finish_sample[(batch,)](logits, scores, indices, maxima, totals, tokens, logp, vocab, parts, True, 4)
        return tokens.tolist(), [round(float(x), 6) for x in logp]

    for temperature, seed, step in ((0.0, 0, 0), (1.0, 0, 0), (1.0, 0, 1), (0.7, 1234567, 5), (1.0, 2 ** 40 + 3, 300)):
        tokens, logp = run(False, temperature, seed, step)
        out["cases"].append(dict(mode="batch", temperature=temperature, seed=seed, step=step, tokens=tokens, logprobs=logp))
    seeds = torch.tensor([1, 2, 3, 2 ** 50 + 11, 5], dtype=torch.int64)
    steps = torch.tensor([0, 1, 2, 3, 400], dtype=torch.int64)
    temps = torch.tensor([1.0, 0.0, 0.5, 1.0, 1.3], dtype=torch.float32)
    tokens, logp = run(True, 1.0, 0, 0, seeds, steps, temps)
    out["cases"].append(dict(mode="per_row", seeds=seeds.tolist(), steps=steps.tolist(),
                             temperatures=[round(float(x), 6) for x in temps], tokens=tokens, logprobs=logp))
    return out


def kernel_vectors():
    """Rounding-point vectors from the reference's fused decode kernels (interpreter, bf16).

    Outputs are stored as raw bf16 / e4m3 bit patterns so the comparison is bit-exact.
    """
    from climbing_gym.inference import lfm25_cuda_kernels as ck
    from climbing_gym.inference import lfm25_fp8 as f8
    from climbing_gym.inference import lfm25_session as ss

    sys.path.insert(0, str(OUT))
    from inputs import kernel_inputs, rope_tables

    inp = kernel_inputs()
    rows, h, f, hq, hkv, d, eps = (inp[k] for k in ("rows", "h", "f", "hq", "hkv", "d", "eps"))
    out = {}

    def bf(x):
        return torch.from_numpy(np.asarray(x, dtype=np.float32)).to(torch.bfloat16)

    def bits(t):
        if t.dtype == torch.bfloat16:
            return t.contiguous().view(torch.int16).numpy().astype(np.uint16).tolist()
        if t.dtype == torch.float8_e4m3fn:
            return t.contiguous().view(torch.uint8).numpy().tolist()
        if t.dtype == torch.float32:
            return t.numpy().view(np.uint32).tolist()
        return t.tolist()

    x, r, w = bf(inp["x"]), bf(inp["res"]), bf(inp["norm_w"])
    y, s = torch.empty_like(x), torch.empty_like(x)
    ck._rms_kernel[(rows,)](x, w, r, y, s, h, eps, True, 256)
    out["rms_add"] = dict(y=bits(y), sum=bits(s))
    y2 = torch.empty_like(x)
    ck._rms_kernel[(rows,)](x, w, x, y2, x, h, eps, False, 256)
    out["rms"] = dict(y=bits(y2))

    gu = bf(inp["gate_up"])
    act = torch.empty((rows, f), dtype=torch.bfloat16)
    ck._swiglu_kernel[(rows, -(-f // 256))](gu, act, f, 256)
    out["swiglu"] = dict(y=bits(act))

    bcx, cw = bf(inp["bcx"]), bf(inp["conv_w"])
    state = bf(inp["conv_state"]).clone()
    active = torch.from_numpy(inp["conv_active"])
    slots = torch.from_numpy(inp["conv_slots"])
    cy = torch.empty((rows, h), dtype=torch.bfloat16)
    ck._conv_kernel[(rows, -(-h // 256))](bcx, cw, state, cy, active, h, 256, True, slots, True)
    out["conv_indexed_masked"] = dict(y=bits(cy), state=bits(state))
    state2 = bf(inp["conv_state"]).clone()
    cy2 = torch.empty((rows, h), dtype=torch.bfloat16)
    ck._conv_kernel[(rows, -(-h // 256))](bcx, cw, state2, cy2, None, h, 256, False, None, False)
    out["conv_plain"] = dict(y=bits(cy2), state=bits(state2))

    cos, sin = (torch.from_numpy(t) for t in rope_tables(inp["rope_theta"], inp["rope_len"], d))
    qkv = bf(inp["qkv"])
    q = torch.empty((rows, 1, hq, d), dtype=torch.bfloat16)
    k = torch.empty((rows, 1, hkv, d), dtype=torch.bfloat16)
    v = torch.empty_like(k)
    ck._qkv_kernel[(rows, hq + hkv)](qkv, bf(inp["q_norm_w"]), bf(inp["k_norm_w"]), cos, sin,
                                     torch.from_numpy(inp["positions"]), q, k, v, hq, hkv, d, eps)
    out["qkv_rope"] = dict(q=bits(q), k=bits(k), v=bits(v))

    qx = bf(inp["quant_x"])
    qq = torch.empty(qx.shape, dtype=torch.float8_e4m3fn)
    qs = torch.empty(rows, dtype=torch.float32)
    f8._quantize_rows[(rows,)](qx, qq, qs, qx.size(1), 512)
    out["quantize_rows"] = dict(q=bits(qq), scales=bits(qs))
    rq = torch.empty((rows, h), dtype=torch.float8_e4m3fn)
    rs, rsum = torch.empty(rows, dtype=torch.float32), torch.empty_like(x)
    f8._rms_quantize[(rows,)](x, w, r, rq, rs, rsum, h, eps, True, 256)
    out["rms_quantize"] = dict(q=bits(rq), scales=bits(rs), sum=bits(rsum))
    sq = torch.empty((rows, f), dtype=torch.float8_e4m3fn)
    sscale = torch.empty(rows, dtype=torch.float32)
    f8._swiglu_quantize[(rows,)](gu, sq, sscale, f, 512)
    out["swiglu_quantize"] = dict(q=bits(sq), scales=bits(sscale))

    # W8A8 matmul with per-token x per-channel epilogue scaling (fp32 accumulate)
    rng = np.random.default_rng(12)
    wmat = bf(rng.standard_normal((64, 512)) * 0.05)
    wq = torch.empty(wmat.shape, dtype=torch.float8_e4m3fn)
    ws = torch.empty(64, dtype=torch.float32)
    f8._quantize_rows[(64,)](wmat, wq, ws, 512, 512)
    yo = torch.empty((rows, 64), dtype=torch.bfloat16)
    f8._matmul[(1, 1, 1)](qq, wq, qs, ws, yo, rows, 64, 512, 16, 64, 128, 1)
    out["fp8_matmul"] = dict(seed=12, w_q=bits(wq), w_s=bits(ws), y=bits(yo))

    # session bookkeeping kernel: EOS > stop-table > length priority, pending/input hand-off
    n, cap, vocab, eos = 6, 4, 16, 2
    sampled = torch.tensor([5, 2, 9, 2, 7, 3], dtype=torch.long)
    logp = torch.tensor([-1.0, -2.0, -3.0, -4.0, -5.0, -6.0])
    tokens = torch.zeros((n, cap), dtype=torch.long); logprobs = torch.zeros((n, cap))
    lengths = torch.tensor([0, 1, 3, 2, 0, 1], dtype=torch.int32)
    limits = torch.tensor([4, 4, 4, 4, 4, 4], dtype=torch.int32)
    reasons = torch.zeros(n, dtype=torch.int8)
    alive = torch.tensor([True, True, True, True, False, True])
    pending = torch.zeros(n, dtype=torch.bool); inputs = torch.zeros(n, dtype=torch.long)
    stop_states = torch.zeros(n, dtype=torch.int64)
    stop_offsets = torch.tensor([0, 0, 0, 0, 0, vocab], dtype=torch.int64)
    table = torch.zeros(2 * vocab, dtype=torch.int32); table[vocab + 3] = 65536
    ignore = torch.tensor([False, False, False, True, False, False])
    rngpos = torch.tensor([0, 1, 3, 2, 0, 1], dtype=torch.int64)
    ss._record_sample[(n,)](sampled, logp, tokens, logprobs, lengths, limits, reasons, alive, pending,
                            inputs, stop_states, stop_offsets, table, ignore, rngpos, eos, vocab, cap)
    out["record_sample"] = dict(tokens=tokens.tolist(), logprobs=logprobs.tolist(), lengths=lengths.tolist(),
                                reasons=reasons.tolist(), alive=alive.tolist(), pending=pending.tolist(),
                                input=inputs.tolist(), rng_positions=rngpos.tolist(), stop_states=stop_states.tolist())
    return out


def head_vectors():
    """Reference behaviour head (torch.topk + its Triton log-prob kernel) and the session's head recorder,
    fed by the reference sampler's own tokens and log-probs. Rows of distinct logits, so that the order
    torch.topk returns is determined."""
    from climbing_gym.inference import lfm25_sampling as ref
    from climbing_gym.inference import lfm25_session as ss

    rng = np.random.default_rng(8)
    batch, vocab = 5, 9000
    logits = torch.from_numpy((rng.standard_normal((batch, vocab)) * 2.0).astype(np.float32))
    parts = -(-vocab // 4096)
    scores = torch.empty((batch, parts)); indices = torch.empty((batch, parts), dtype=torch.int32)
    maxima = torch.empty_like(scores); totals = torch.empty_like(scores)
    tokens = torch.empty(batch, dtype=torch.long); logp = torch.empty(batch)
    key = (21 + 3 * 0x9E3779B97F4A7C15) & 0x7FFFFFFFFFFFFFFF
    ref._partial_sample[(batch, parts)](logits, scores, indices, maxima, totals, key, vocab, parts, 1.0, True, 4096)
    ref._finish_sample[(batch,)](logits, scores, indices, maxima, totals, tokens, logp, vocab, parts, True, 4)
    out = {"batch": batch, "vocab": vocab, "seed": 21, "step": 3, "tokens": tokens.tolist(),
           "logprobs": [round(float(x), 6) for x in logp], "heads": []}
    for k in (1, 5, 128):
        ids, probs = ref.behavior_topk(logits, tokens, logp, k)
        out["heads"].append(dict(k=k, ids=ids.tolist(), logprobs=[[round(float(x), 6) for x in row] for row in probs]))
    k, cap = 5, 4
    ids, probs = ref.behavior_topk(logits, tokens, logp, k)
    lengths = torch.tensor([0, 3, 1, 2, 0], dtype=torch.int32)
    alive = torch.tensor([True, True, False, True, True])
    out_ids = torch.zeros((batch, cap, k), dtype=torch.int32); out_probs = torch.zeros((batch, cap, k))
    ss._record_head[(batch,)](ids.to(torch.int32), probs, out_ids, out_probs, lengths, alive, k, cap, 8)
    out["record_head"] = dict(k=k, capacity=cap, lengths=lengths.tolist(), alive=alive.tolist(), ids=out_ids.tolist(),
                              logprobs=[[[round(float(x), 6) for x in r] for r in slot] for slot in out_probs])
    return out


def penalty_vectors():
    """Reference repetition penalty: the elementwise rule on random logits, and greedy generation of the
    tiny model under a penalty (the reference's eager CPU engine; prompt tokens count as seen)."""
    from climbing_gym.inference import lfm25_engine as ref

    rng = np.random.default_rng(9)
    logits = torch.from_numpy((rng.standard_normal((4, 512)) * 2.0).astype(np.float32))
    seen = torch.from_numpy(rng.random((4, 512)) < 0.3)
    out = {"rule": []}
    for penalty in (1.3, 0.8):
        y = ref._apply_repetition_penalty(logits.clone(), seen_token_mask=seen, penalty=penalty)
        out["rule"].append(dict(penalty=penalty, bits=y.view(torch.int32).tolist()))
    cfg = synthetic.tiny_config()
    state = synthetic.make_state_dict(cfg, seed=0, untied_head=True)
    prompts = synthetic.uniform_prompts(8, 8, 64, cfg.vocab_size, seed=0)[:4]
    engine = ref_engine(None, cfg, state, torch.float32)
    for penalty in (1.3, 0.8):
        got = engine.generate(*ref.flatten_token_batches(prompts), repeats=2,
                              sampling=ref.LFM25SamplingConfig(temperature=0.0, max_new_tokens=24,
                                                               repetition_penalty=penalty, ignore_eos=True))
        out[f"generate_fp32_{penalty}"] = dict(
            penalty=penalty, token_ids=got.token_ids.tolist(),
            logprobs=[[[round(float(x), 6) for x in r] for r in p] for p in got.logprobs.tolist()])
    return out


FULL_SIZE_PROMPT_SEED = 21


def full_size_inputs():
    """Seeded inputs of the 1.2B-size cases; tests rebuild them from here (numpy only)."""
    cfg = synthetic.lfm25_1p2b_config()
    prompts = synthetic.uniform_prompts(8, 64, 256, cfg.vocab_size, seed=FULL_SIZE_PROMPT_SEED)
    score_prompts = synthetic.uniform_prompts(6, 32, 128, cfg.vocab_size, seed=FULL_SIZE_PROMPT_SEED + 1)
    completions = synthetic.uniform_prompts(6, 8, 24, cfg.vocab_size, seed=FULL_SIZE_PROMPT_SEED + 2)
    long_prompt = synthetic.uniform_prompts(1, 9300, 9300, cfg.vocab_size, seed=FULL_SIZE_PROMPT_SEED + 3)[0]
    return cfg, prompts, score_prompts, completions, long_prompt


def full_size_vectors():
    """The reference's eager CPU engine on the LFM2.5-1.2B architecture in bf16 (the benchmarked size):
    greedy generation, completion scoring and the next-token logits of one 9300-token prompt (prefilled
    in one piece; the engine under test chunks it). Weights: synthetic.make_state_dict_streams(seed 0).
    Takes tens of minutes on a handful of cores."""
    import time
    from climbing_gym.inference.lfm25_engine import LFM25SamplingConfig, flatten_token_batches

    cfg, prompts, score_prompts, completions, long_prompt = full_size_inputs()
    state = synthetic.make_state_dict_streams(cfg, seed=0)
    engine = ref_engine(None, cfg, state, torch.bfloat16, max_model_len=9344)
    del state
    out, t0 = {}, time.time()
    got = engine.generate(*flatten_token_batches(prompts), repeats=1,
                          sampling=LFM25SamplingConfig(temperature=0.0, max_new_tokens=32, ignore_eos=True))
    out["generate_bf16"] = dict(token_ids=got.token_ids[:, 0].tolist(),
                                logprobs=[[round(float(x), 6) for x in row] for row in got.logprobs[:, 0].tolist()])
    print("generate", round(time.time() - t0, 1), flush=True)
    scores = engine.score_completions(score_prompts, completions)
    out["score_bf16"] = [[round(float(x), 6) for x in row] for row in scores]
    print("score", round(time.time() - t0, 1), flush=True)
    prefix = engine.prefill(*flatten_token_batches([long_prompt]))
    logits = prefix.next_token_logits.float()[0]
    top = torch.topk(logits, 8)
    out["long_prefill_bf16"] = dict(length=len(long_prompt), lse=round(float(torch.logsumexp(logits, -1)), 6),
                                    top_ids=top.indices.tolist(), top_logits=[round(float(x), 6) for x in top.values],
                                    every_256th=[round(float(x), 6) for x in logits[::256]])
    print("long prefill", round(time.time() - t0, 1), flush=True)
    return out


def main():
    parser = argparse.ArgumentParser()
    parser.add_argument("--reference", required=True, help="the src/ directory of a reference checkout")
    parser.add_argument("--only", default="")
    args = parser.parse_args()
    sys.path.insert(0, args.reference)
    jobs = dict(model=model_vectors, sampler=sampler_vectors, kernels=kernel_vectors, head=head_vectors,
                penalty=penalty_vectors, model_1p2b=full_size_vectors)
    for name, fn in jobs.items():
        if (args.only and name not in args.only.split(",")) or (name == "model_1p2b" and not args.only):
            continue  # the full-size vectors take tens of minutes: only on request (--only model_1p2b)
        payload = fn()
        (OUT / f"{name}.json").write_text(json.dumps(payload, separators=(",", ":")) + "\n")
        print("wrote", name)


if __name__ == "__main__":
    main()
