"""CPU restatement of the reference LFM2.5 rollout engine (TEST INFRASTRUCTURE ONLY).

This is the checker for the CUDA path, never the product path: only ``tests/``,
``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline legs may import it.

It restates in numpy what ``src/climbing_gym/inference/lfm25_engine.py`` (eager engine),
``lfm25_cuda.py`` (fused decode step and generate loop), ``lfm25_cuda_kernels.py``,
``lfm25_fp8.py`` and ``lfm25_fp8_kv.py`` compute, with the model dtype's rounding applied
at the same points as the reference's kernels ("bf16" mode) or not at all ("fp32" mode,
the reference's CPU-runnable configuration). Parity is pinned by
``tests/golden/*.json``, produced by running the reference itself on CPU
(``tests/golden/make_golden.py``).

Reference anchors (file:line within the reference project):
  RMSNorm ............ lfm25_engine.py:1741-1746, lfm25_cuda_kernels.py:32-44
  RoPE ............... lfm25_engine.py:1004-1012,1749-1756, lfm25_cuda_kernels.py:113-140
  attention prefill .. lfm25_engine.py:1364-1394
  attention decode ... lfm25_engine.py:1306-1362,1533-1572; lfm25_fp8_kv.py:72-120
  conv prefill ....... lfm25_engine.py:1451-1476
  conv decode ........ lfm25_engine.py:1424-1449; lfm25_cuda_kernels.py:75-100
  MLP ................ lfm25_engine.py:1042-1044,1300-1304; lfm25_cuda_kernels.py:58-65
  FP8 W8A8 MLP ....... lfm25_fp8.py:16-54,76-93; lfm25_cuda.py:173-177
  generate loop ...... lfm25_cuda.py:269-380, lfm25_engine.py:741-865
  sampler ............ lfm25_sampling.py:10-58
  scoring ............ lfm25_engine.py:1108-1163
"""
from __future__ import annotations

from dataclasses import dataclass, field
from typing import Sequence

import numpy as np

from . import philox
from .numerics import decode_e4m3, encode_e4m3, quantize_rows_e4m3, rounder

LOG2E = np.float32(1.4426950408889634)


@dataclass(frozen=True)
class OracleConfig:
    vocab_size: int = 65536
    hidden_size: int = 2048
    mlp_hidden_size: int = 8192
    num_attention_heads: int = 32
    num_key_value_heads: int = 8
    layer_types: tuple = ()
    rope_theta: float = 1_000_000.0
    norm_eps: float = 1e-5
    conv_kernel_size: int = 3
    eos_token_id: int = 7

    @property
    def head_dim(self) -> int:
        return self.hidden_size // self.num_attention_heads


@dataclass
class OracleSampling:
    """Mirror of LFM25SamplingConfig's fields used on the hot path (lfm25_engine.py:22-35)."""

    temperature: float = 1.0
    max_new_tokens: int = 256
    stop_token_ids: tuple = ()
    seed: int = 0
    ignore_eos: bool = False
    # test hook: generated position at which each flat row's token is replaced by EOS
    force_eos_at: tuple | None = None
    repetition_penalty: float = 1.0


@dataclass
class SeqState:
    """One sequence's hybrid cache: KV per attention layer, conv history per conv layer."""

    k: list  # per attention layer: list of [Hkv, D] rows (fp32 values or e4m3 codes)
    v: list
    ks: list  # per attention layer: list of [Hkv] scales (fp8 KV only)
    vs: list
    conv: np.ndarray  # [n_conv, H, 3], newest last
    length: int = 0

    def clone(self) -> "SeqState":
        return SeqState([list(x) for x in self.k], [list(x) for x in self.v],
                        [list(x) for x in self.ks], [list(x) for x in self.vs],
                        self.conv.copy(), self.length)


class OracleEngine:
    """Numpy engine with the reference's numerics contract.

    ``dtype`` is "fp32" or "bf16". ``fp8_mlp`` / ``fp8_kv`` switch on the reference's
    decode-time FP8 paths (prefill always uses the model dtype, lfm25_fp8.py:4-5).
    """

    def __init__(self, cfg: OracleConfig, state_dict: dict, *, dtype: str = "fp32",
                 max_model_len: int = 4096, fp8_mlp: bool = False, fp8_kv: bool = False,
                 weights_exact: bool = False, fp8_lm_head: bool = False):
        """``weights_exact``: the arrays of ``state_dict`` are already representable in the model
        dtype (e.g. copied from a bf16 checkpoint), so the load-time cast is skipped: at 1.2 B
        parameters the numpy cast alone takes minutes."""
        self.cfg, self.dtype = cfg, dtype
        self.rd = rounder(dtype)
        self.fp8_mlp, self.fp8_kv, self.fp8_lm_head = bool(fp8_mlp), bool(fp8_kv), bool(fp8_lm_head)
        self.max_model_len = int(max_model_len)
        rd = (lambda a: a) if weights_exact else self.rd

        def t(key):
            return rd(np.asarray(state_dict[key], dtype=np.float32))

        self.embed = t("model.embed_tokens.weight")
        self.head = t("model.lm_head.weight") if "model.lm_head.weight" in state_dict else self.embed
        self.final_norm = t("model.embedding_norm.weight")
        self.layers = []
        n_attn = n_conv = 0
        for i, kind in enumerate(cfg.layer_types):
            p = f"model.layers.{i}"
            layer = dict(kind=kind, op_norm=t(f"{p}.operator_norm.weight"), ffn_norm=t(f"{p}.ffn_norm.weight"),
                         w13=np.concatenate([t(f"{p}.feed_forward.w1.weight"), t(f"{p}.feed_forward.w3.weight")], 0),
                         w2=t(f"{p}.feed_forward.w2.weight"))
            if kind == "full_attention":
                layer.update(qkv=np.concatenate([t(f"{p}.self_attn.q_proj.weight"), t(f"{p}.self_attn.k_proj.weight"),
                                                 t(f"{p}.self_attn.v_proj.weight")], 0),
                             out=t(f"{p}.self_attn.out_proj.weight"), q_norm=t(f"{p}.self_attn.q_layernorm.weight"),
                             k_norm=t(f"{p}.self_attn.k_layernorm.weight"), cache_index=n_attn)
                n_attn += 1
            else:
                layer.update(conv_in=t(f"{p}.conv.in_proj.weight"), conv_w=t(f"{p}.conv.conv.weight")[:, 0, :],
                             conv_out=t(f"{p}.conv.out_proj.weight"), cache_index=n_conv)
                n_conv += 1
            self.layers.append(layer)
        if self.fp8_mlp:
            self.prepare_fp8()
        if self.fp8_lm_head:  # the vocabulary head joins the FP8 copies (lfm25_cuda.py:103-105)
            codes, self.head_s = quantize_rows_e4m3(self.head)
            self.head_q = decode_e4m3(codes)
        self.n_attn, self.n_conv = n_attn, n_conv
        half = cfg.head_dim // 2
        inv_freq = (1.0 / (np.float32(cfg.rope_theta) ** (np.arange(0, cfg.head_dim, 2, dtype=np.float32)
                                                           / np.float32(cfg.head_dim)))).astype(np.float32)
        freqs = np.arange(self.max_model_len, dtype=np.float32)[:, None] * inv_freq[None, :]
        self.rope_cos, self.rope_sin = np.cos(freqs).astype(np.float32), np.sin(freqs).astype(np.float32)
        assert self.rope_cos.shape[1] == half

    def prepare_fp8(self) -> None:
        """FP8 copies of w13 / w2: per-output-channel row quantisation (PackedFP8Weight.from_weight,
        lfm25_fp8.py:127-131). Idempotent, so one engine can serve bf16 and FP8 runs by switching
        ``fp8_mlp`` / ``fp8_kv`` between them."""
        for layer in self.layers:
            for name in ("w13", "w2"):
                if name + "_q" not in layer:
                    codes, scales = quantize_rows_e4m3(layer[name])
                    layer[name + "_q"], layer[name + "_s"] = decode_e4m3(codes), scales

    # ------------------------------------------------------------------ primitives
    def linear(self, x, w):
        return self.rd(x.astype(np.float32) @ w.T)

    def rms_norm(self, x, w):
        x = x.astype(np.float32)
        var = np.mean(x * x, axis=-1, keepdims=True, dtype=np.float32)
        normalized = self.rd(x * (np.float32(1.0) / np.sqrt(var + np.float32(self.cfg.norm_eps))))
        return self.rd(normalized * w)

    def rope(self, x, positions):
        """x [T, heads, D]; half-split rotation with dtype-rounded coefficients and products."""
        rd, half = self.rd, self.cfg.head_dim // 2
        cos = rd(self.rope_cos[positions])[:, None, :]
        sin = rd(self.rope_sin[positions])[:, None, :]
        x1, x2 = x[..., :half], x[..., half:]
        y1 = rd(rd(x1 * cos) - rd(x2 * sin))
        y2 = rd(rd(x2 * cos) + rd(x1 * sin))
        return np.concatenate([y1, y2], -1)

    def swiglu(self, gate_up):
        f = self.cfg.mlp_hidden_size
        gate, up = gate_up[..., :f], gate_up[..., f:]
        act = self.rd(gate / (np.float32(1.0) + np.exp(-gate, dtype=np.float32)))
        return self.rd(act * up)

    def mlp(self, layer, hidden_normed, *, decode: bool):
        if self.fp8_mlp and decode:
            codes, a_s = quantize_rows_e4m3(hidden_normed)
            acc = decode_e4m3(codes) @ layer["w13_q"].T
            gate_up = self.rd(acc * a_s[:, None] * layer["w13_s"][None, :])
            codes, a_s = quantize_rows_e4m3(self.swiglu(gate_up))
            acc = decode_e4m3(codes) @ layer["w2_q"].T
            return self.rd(acc * a_s[:, None] * layer["w2_s"][None, :])
        return self.linear(self.swiglu(self.linear(hidden_normed, layer["w13"])), layer["w2"])

    def new_state(self) -> SeqState:
        cfg = self.cfg
        return SeqState([[] for _ in range(self.n_attn)], [[] for _ in range(self.n_attn)],
                        [[] for _ in range(self.n_attn)], [[] for _ in range(self.n_attn)],
                        np.zeros((self.n_conv, cfg.hidden_size, cfg.conv_kernel_size), np.float32), 0)

    def _store_kv(self, state: SeqState, idx: int, k, v):
        """Append rows k, v [T, Hkv, D] to one attention layer's history."""
        if not self.fp8_kv:
            state.k[idx].extend(k)
            state.v[idx].extend(v)
            return
        for row_k, row_v in zip(k, v):
            ck, sk = quantize_rows_e4m3(row_k)  # per (token, head) scale, lfm25_fp8_kv.py:47-55
            cv, sv = quantize_rows_e4m3(row_v)
            state.k[idx].append(decode_e4m3(ck))
            state.v[idx].append(decode_e4m3(cv))
            state.ks[idx].append(sk)
            state.vs[idx].append(sv)

    def _attend_history(self, state: SeqState, idx: int, q):
        """One query token q [Hq, D] over the whole stored history (already includes itself)."""
        cfg, rd = self.cfg, self.rd
        g = cfg.num_attention_heads // cfg.num_key_value_heads
        k = np.stack(state.k[idx])  # [T, Hkv, D]
        v = np.stack(state.v[idx])
        qg = q.reshape(cfg.num_key_value_heads, g, cfg.head_dim)
        scores = np.einsum("hgd,thd->hgt", qg, k).astype(np.float32) * np.float32(cfg.head_dim ** -0.5)
        if self.fp8_kv:
            scores = scores * np.stack(state.ks[idx]).T[:, None, :]
        scores = scores - scores.max(-1, keepdims=True)
        p = np.exp(scores, dtype=np.float32)
        total = p.sum(-1, keepdims=True, dtype=np.float32)
        if self.fp8_kv:
            # un-normalised P scaled by the V scale and rounded, normalised afterwards (lfm25_fp8_kv.py:103-112)
            pv = rd(p * np.stack(state.vs[idx]).T[:, None, :])
            out = np.einsum("hgt,thd->hgd", pv, v).astype(np.float32) / total
        else:
            out = np.einsum("hgt,thd->hgd", rd(p / total), v).astype(np.float32)
        return rd(out).reshape(-1)

    # ------------------------------------------------------------------ prefill
    def prefill(self, tokens: Sequence[int], state: SeqState | None = None, *, return_hidden: bool = False):
        """Run tokens through the model appending to ``state`` (chunk continuation allowed).

        Returns (state, last-token logits [V]) or, with return_hidden, the final-normed
        hidden states [T, H] (for completion scoring, lfm25_engine.py:1097-1098).
        """
        cfg, rd = self.cfg, self.rd
        state = self.new_state() if state is None else state
        tokens = np.asarray(tokens, dtype=np.int64)
        n, start = len(tokens), state.length
        positions = np.arange(start, start + n)
        hidden = self.embed[tokens]
        hq, hkv, d = cfg.num_attention_heads, cfg.num_key_value_heads, cfg.head_dim
        g = hq // hkv
        for layer in self.layers:
            x = self.rms_norm(hidden, layer["op_norm"])
            if layer["kind"] == "full_attention":
                idx = layer["cache_index"]
                qkv = self.linear(x, layer["qkv"])
                q = qkv[:, :hq * d].reshape(n, hq, d)
                k = qkv[:, hq * d:(hq + hkv) * d].reshape(n, hkv, d)
                v = qkv[:, (hq + hkv) * d:].reshape(n, hkv, d)
                q = self.rope(self.rms_norm(q, layer["q_norm"]), positions)
                k = self.rope(self.rms_norm(k, layer["k_norm"]), positions)
                # history before this chunk (as stored, i.e. dequantised codes when fp8_kv)
                if start:
                    pk, pv = np.stack(state.k[idx]), np.stack(state.v[idx])
                    if self.fp8_kv:
                        pk = pk * np.stack(state.ks[idx])[..., None]
                        pv = pv * np.stack(state.vs[idx])[..., None]
                    kk, vv = np.concatenate([pk, k]), np.concatenate([pv, v])
                else:
                    kk, vv = k, v
                self._store_kv(state, idx, k, v)
                qg = q.reshape(n, hkv, g, d)
                scores = np.einsum("thgd,shd->hgts", qg, kk).astype(np.float32) * np.float32(d ** -0.5)
                mask = np.arange(start + n)[None, :] > positions[:, None]
                scores = np.where(mask[None, None], -np.inf, scores)
                scores = scores - scores.max(-1, keepdims=True)
                p = np.exp(scores, dtype=np.float32)
                p = rd(p / p.sum(-1, keepdims=True, dtype=np.float32))
                att = rd(np.einsum("hgts,shd->thgd", p, vv).astype(np.float32)).reshape(n, hq * d)
                op = self.linear(att, layer["out"])
            else:
                idx = layer["cache_index"]
                bcx = self.linear(x, layer["conv_in"])
                h = cfg.hidden_size
                b, c, xx = bcx[:, :h], bcx[:, h:2 * h], bcx[:, 2 * h:]
                bx = rd(b * xx)
                # causal depthwise conv, left context = the two newest carried rows (zeros when
                # fresh); exact products, fp32 sum, one rounding (F.conv1d, lfm25_engine.py:1464-1469)
                full = np.concatenate([state.conv[idx].T, bx])  # rows: 3 carried + n new
                hist = full[1:]
                w = layer["conv_w"]
                conv = rd(hist[:-2] * w[:, 0] + hist[1:-1] * w[:, 1] + hist[2:] * w[:, 2])
                state.conv[idx] = full[-3:].T.copy()
                op = self.linear(rd(c * conv), layer["conv_out"])
            hidden = rd(hidden + op)
            y = self.rms_norm(hidden, layer["ffn_norm"])
            hidden = rd(hidden + self.mlp(layer, y, decode=False))
        state.length = start + n
        if return_hidden:
            return state, self.rms_norm(hidden, self.final_norm)
        return state, self.linear(self.rms_norm(hidden[-1:], self.final_norm), self.head)[0]

    # ------------------------------------------------------------------ decode
    def decode(self, states: Sequence[SeqState], tokens: Sequence[int]) -> np.ndarray:
        """One fused decode step for a batch (lfm25_cuda.py:128-192). Returns logits [B, V]."""
        cfg, rd = self.cfg, self.rd
        tokens = np.asarray(tokens, dtype=np.int64)
        bsz = len(tokens)
        positions = np.array([s.length for s in states])
        hq, hkv, d, h = cfg.num_attention_heads, cfg.num_key_value_heads, cfg.head_dim, cfg.hidden_size
        hidden = self.embed[tokens]
        for layer in self.layers:
            x = self.rms_norm(hidden, layer["op_norm"])
            if layer["kind"] == "full_attention":
                idx = layer["cache_index"]
                qkv = self.linear(x, layer["qkv"])
                q = self.rope(self.rms_norm(qkv[:, :hq * d].reshape(bsz, hq, d), layer["q_norm"]), positions)
                k = self.rope(self.rms_norm(qkv[:, hq * d:(hq + hkv) * d].reshape(bsz, hkv, d), layer["k_norm"]), positions)
                v = qkv[:, (hq + hkv) * d:].reshape(bsz, hkv, d)
                att = np.empty((bsz, hq * d), np.float32)
                for i, s in enumerate(states):
                    self._store_kv(s, idx, k[i:i + 1], v[i:i + 1])
                    att[i] = self._attend_history(s, idx, q[i])
                op = self.linear(att, layer["out"])
            else:
                idx = layer["cache_index"]
                bcx = self.linear(x, layer["conv_in"])
                b, c, xx = bcx[:, :h], bcx[:, h:2 * h], bcx[:, 2 * h:]
                bx = rd(b * xx)
                w = layer["conv_w"]
                conv = np.empty((bsz, h), np.float32)
                for i, s in enumerate(states):
                    st = s.conv[idx]
                    st[:, 0], st[:, 1], st[:, 2] = st[:, 1].copy(), st[:, 2].copy(), bx[i]
                    # products rounded individually, fp32 sum, one more rounding (lfm25_cuda_kernels.py:92-95)
                    conv[i] = rd(rd(st[:, 0] * w[:, 0]) + rd(st[:, 1] * w[:, 1]) + rd(st[:, 2] * w[:, 2]))
                op = self.linear(rd(c * conv), layer["conv_out"])
            hidden = rd(hidden + op)
            y = self.rms_norm(hidden, layer["ffn_norm"])
            hidden = rd(hidden + self.mlp(layer, y, decode=True))
        for s in states:
            s.length += 1
        final = self.rms_norm(hidden, self.final_norm)
        if self.fp8_lm_head:  # decode-time FP8 head: quantised final norm output (lfm25_cuda.py:181-191)
            codes, a_s = quantize_rows_e4m3(final)
            return rd((decode_e4m3(codes) @ self.head_q.T) * a_s[:, None] * self.head_s[None, :])
        return self.linear(final, self.head)

    # ------------------------------------------------------------------ sampler
    def sample(self, logits, *, temperature: float, seed: int, step: int, rows=None):
        """Gumbel-max / greedy with untempered sampled-token logprob (lfm25_sampling.py:10-58).

        Batch keying: key(seed, step), offset row*V+col. ``rows`` gives each logits row's
        batch index (defaults to 0..B-1).
        """
        logits = np.asarray(logits, dtype=np.float32)
        bsz, vocab = logits.shape
        rows = np.arange(bsz) if rows is None else np.asarray(rows)
        if temperature > 0:
            key = philox.step_key(seed, step)
            offsets = (rows[:, None].astype(np.int64) * vocab + np.arange(vocab)[None, :]) & 0xFFFFFFFF
            u = np.maximum(philox.uniform(offsets, key), np.float32(1.0e-30))
            score = logits / np.float32(temperature) - np.log(-np.log(u, dtype=np.float32), dtype=np.float32)
        else:
            score = logits
        tokens = np.argmax(score, axis=-1)  # numpy argmax returns the lowest index on ties
        return tokens, OracleEngine.logprob_of(logits, tokens)

    def sample_per_row(self, logits, seeds, positions, temperatures):
        """Per-request RNG streams (RowSampler, lfm25_sampling.py:17-23,95-123): offset = col."""
        logits = np.asarray(logits, dtype=np.float32)
        bsz, vocab = logits.shape
        tokens = np.empty(bsz, np.int64)
        for i in range(bsz):
            if temperatures[i] > 0:
                key = philox.step_key(int(seeds[i]) & philox.MASK63, int(positions[i]))
                u = np.maximum(philox.uniform(np.arange(vocab), key), np.float32(1.0e-30))
                score = logits[i] / np.maximum(np.float32(temperatures[i]), np.float32(1e-30)) \
                    - np.log(-np.log(u, dtype=np.float32), dtype=np.float32)
            else:
                score = logits[i]
            tokens[i] = int(np.argmax(score))
        return tokens, OracleEngine.logprob_of(logits, tokens)

    @staticmethod
    def logprob_of(logits, tokens):
        m = logits.max(-1)
        lse = m + np.log(np.exp(logits - m[:, None], dtype=np.float32).sum(-1, dtype=np.float32), dtype=np.float32)
        return (logits[np.arange(len(tokens)), tokens] - lse).astype(np.float32)

    # ------------------------------------------------------------------ generate
    def generate(self, prompts: Sequence[Sequence[int]], repeats: int, sampling: OracleSampling):
        """Batch generate with the reference's loop semantics (lfm25_cuda.py:269-380).

        Returns dict(token_ids [P,R,N] int64, lengths [P,R] int32, logprobs [P,R,N] f32,
        finish_reasons [P,R] int8). Dead rows write token 0 / logprob 0; unfinished rows get
        reason 3; the first token comes from the prefill logits.
        """
        n_new, eos = sampling.max_new_tokens, self.cfg.eos_token_id
        states, first = [], []
        for prompt in prompts:
            st, logits = self.prefill(prompt)
            for _ in range(repeats):
                states.append(st.clone())
                first.append(logits)
        bsz = len(states)
        # seen-token mask of the repetition penalty: the prompt's tokens, then every sampled token
        # (lfm25_engine.py:933-958, lfm25_cuda.py:336-337)
        seen = None
        if sampling.repetition_penalty != 1.0:
            from .kernels import apply_repetition_penalty
            seen = np.zeros((bsz, self.cfg.vocab_size), bool)
            for p, prompt in enumerate(prompts):
                seen[p * repeats:(p + 1) * repeats, list(prompt)] = True
        logits = np.stack(first)
        tokens = np.zeros((bsz, n_new), np.int64)
        logprobs = np.zeros((bsz, n_new), np.float32)
        lengths = np.zeros(bsz, np.int32)
        reasons = np.zeros(bsz, np.int8)
        alive = np.ones(bsz, bool)
        fixed = sampling.ignore_eos and not sampling.stop_token_ids
        for step in range(n_new):
            if seen is not None:  # the draw and its log-prob both come from the penalised fp32 logits
                logits = apply_repetition_penalty(logits, seen, sampling.repetition_penalty)
            sampled, lp = self.sample(logits, temperature=sampling.temperature, seed=sampling.seed, step=step)
            if seen is not None:
                seen[np.arange(bsz), sampled] = True
            if sampling.force_eos_at is not None:
                forced = np.asarray(sampling.force_eos_at) == step
                if forced.any():
                    sampled = np.where(forced, eos, sampled)
                    lp = self.logprob_of(np.asarray(logits, np.float32), sampled)
            tokens[:, step] = sampled if fixed else np.where(alive, sampled, 0)
            logprobs[:, step] = lp if fixed else np.where(alive, lp, 0)
            if not fixed:
                lengths += alive
                cur = np.zeros(bsz, np.int8)
                if not sampling.ignore_eos:
                    cur[sampled == eos] = 1
                for stop in sampling.stop_token_ids:
                    cur[(cur == 0) & (sampled == stop)] = 2
                reasons = np.where(alive, cur, reasons).astype(np.int8)
                alive &= cur == 0
                if not alive.any():
                    break
            if step + 1 < n_new:
                live = np.nonzero(alive)[0] if not fixed else np.arange(bsz)
                new_logits = self.decode([states[i] for i in live], sampled[live])
                logits = np.array(logits, copy=True)
                logits[live] = new_logits
        if fixed:
            lengths[:] = n_new
        reasons[reasons == 0] = 3
        shape = (len(prompts), repeats)
        return dict(token_ids=tokens.reshape(*shape, n_new), lengths=lengths.reshape(shape),
                    logprobs=logprobs.reshape(*shape, n_new), finish_reasons=reasons.reshape(shape))

    # ------------------------------------------------------------------ teacher forcing
    def teacher_forced(self, prompts: Sequence[Sequence[int]], tokens, *, probe=None) -> dict:
        """Decode a GIVEN continuation and report what this engine thinks of every token of it.

        ``tokens`` [B, N] are the continuations another implementation produced for ``prompts`` (greedy or
        sampled). Row b is prefilled with prompts[b]; step s scores tokens[b, s] against this engine's
        logits for that position and then feeds it as the next decode input, exactly like the generate
        loop (lfm25_cuda.py:315-372), so every step is comparable even after the two implementations
        would have chosen different tokens. Returns fp32 arrays [B, N]: ``logprobs`` of the given tokens,
        this engine's greedy choice ``argmax``, its top logit ``top_logit`` and the given token's logit
        ``given_logit`` (top_logit - given_logit is the margin by which this engine prefers its own
        choice; 0 where the choices agree). ``probe`` [B, N] (optional) names one more token per step
        whose logit is reported as ``probe_logit`` (e.g. a third implementation's choice)."""
        tokens = np.asarray(tokens, dtype=np.int64)
        bsz, n_new = tokens.shape
        states, first = [], []
        for prompt in prompts:
            st, logits = self.prefill(prompt)
            states.append(st)
            first.append(logits)
        logits = np.stack(first).astype(np.float32)
        out = dict(logprobs=np.zeros((bsz, n_new), np.float32), argmax=np.zeros((bsz, n_new), np.int64),
                   top_logit=np.zeros((bsz, n_new), np.float32), given_logit=np.zeros((bsz, n_new), np.float32),
                   probe_logit=np.zeros((bsz, n_new), np.float32))
        rows = np.arange(bsz)
        for step in range(n_new):
            given = tokens[:, step]
            out["logprobs"][:, step] = self.logprob_of(logits, given)
            out["argmax"][:, step] = np.argmax(logits, axis=-1)
            out["top_logit"][:, step] = logits.max(-1)
            out["given_logit"][:, step] = logits[rows, given]
            if probe is not None:
                out["probe_logit"][:, step] = logits[rows, np.asarray(probe, dtype=np.int64)[:, step]]
            if step + 1 < n_new:
                logits = self.decode(states, given).astype(np.float32)
        return out

    # ------------------------------------------------------------------ scoring
    def score_completions(self, prompts, completions):
        """Raw completion log-probs, every completion token included (lfm25_engine.py:1108-1163)."""
        out = []
        for prompt, completion in zip(prompts, completions):
            seq = list(prompt) + list(completion)
            _, hidden = self.prefill(seq, return_hidden=True)
            sel = hidden[len(prompt) - 1:len(seq) - 1]
            logits = self.linear(sel, self.head).astype(np.float32)
            out.append(tuple(float(x) for x in self.logprob_of(logits, np.asarray(completion))))
        return out
