"""Kernel launch sequences of the LFM2.5 forward pass (decode step and packed prefill chunk).

The decode sequence mirrors the reference's fused step
(src/climbing_gym/inference/lfm25_cuda.py:128-192): the residual stream is carried un-summed
between kernels, every RMSNorm fuses the pending residual add, attention layers run
qkv GEMM -> QK-norm/RoPE/KV-append -> paged attention -> out GEMM, conv layers run
in GEMM -> short-conv state update -> out GEMM, then (fused-quant) RMSNorm -> w13 GEMM ->
SwiGLU -> w2 GEMM. The prefill sequence runs the same kernels over packed rows
(reference: lfm25_engine.py:1050-1106, which pads instead of packing).

Everything here only enqueues kernels on the current stream through the C ABI, writes into
buffers allocated once per row capacity, and reads shapes from Python ints, so one call can be
captured into a CUDA graph and replayed.
"""
from __future__ import annotations

import torch

from . import _native as nv
from .paged import PagedHybridCache
from .weights import LFM25PackedWeights, PackedFP8Weight


class ForwardBuffers:
    """Activation scratch for up to ``rows`` rows (addresses stay fixed for graph replay)."""

    def __init__(self, weights: LFM25PackedWeights, rows: int, *, fp8: bool, attn_splits: int = 1):
        cfg, dev, dt = weights.config, weights.device, weights.dtype
        h, f, d = cfg.hidden_size, cfg.mlp_hidden_size, cfg.head_dim
        hq, hkv = cfg.num_attention_heads, cfg.num_key_value_heads
        self.rows = rows

        def buf(width, dtype=dt):
            return torch.empty((rows, width), device=dev, dtype=dtype)

        self.embed, self.branch, self.residual, self.normed = buf(h), buf(h), buf(h), buf(h)
        self.qkv, self.q, self.attended = buf((hq + 2 * hkv) * d), buf(hq * d), buf(hq * d)
        self.bcx, self.conv_out = buf(3 * h), buf(h)
        self.gate_up, self.activated = buf(2 * f), buf(f)
        self.final = buf(h)
        if fp8:
            self.normed_q, self.activated_q = buf(h, torch.uint8), buf(f, torch.uint8)
            self.normed_s = torch.empty(rows, device=dev, dtype=torch.float32)
            self.activated_s = torch.empty(rows, device=dev, dtype=torch.float32)
        self.attn_splits = attn_splits
        self.attn_ws = (torch.empty(rows * hq * attn_splits * (d + 2), device=dev, dtype=torch.float32)
                        if attn_splits > 1 else None)
        # split-K partial tiles of the decode GEMMs: at most 2 x 148 resident CTAs, each parking one
        # [token tile][128] fp32 tile (token tile = 32 / 64 / 128 rows); larger row counts do not split
        token_tile = 32 if rows <= 32 else 64 if rows <= 64 else 128
        self.gemm_ws = torch.empty(2 * 148 * token_tile * 128 * 4, device=dev, dtype=torch.uint8)


class LFM25Runner:
    def __init__(self, weights: LFM25PackedWeights, rope_cos: torch.Tensor, rope_sin: torch.Tensor,
                 *, fp8_mlp: bool = False, fp8_lm_head: bool = False, gemm_impl: int = 0):
        self.weights, self.cfg = weights, weights.config
        self.rope_cos, self.rope_sin = rope_cos, rope_sin
        self.dt = nv.dtype_code(weights.dtype)
        self.fp8_mlp, self.fp8_lm_head = bool(fp8_mlp), bool(fp8_lm_head)
        self.gemm_impl = gemm_impl
        self.attn_impl = 0  # 0 auto, 1 CUDA-core kernel, 2 tensor-core kernel (see cgym_paged_attention)
        self.fp8_weights: dict[int, PackedFP8Weight] = {}
        self.packed_weights: dict = {}  # id(weight) -> PackedBF16Weight, used by single-row steps only
        self.scale = float(self.cfg.head_dim ** -0.5)
        if (fp8_mlp or fp8_lm_head) and weights.dtype != torch.bfloat16:
            raise ValueError("FP8 projections require bfloat16 weights")

    # ---- FP8 copies (reference: lfm25_cuda.py:97-106) ------------------------------------------
    def prepare_fp8(self) -> None:
        if self.fp8_weights or not (self.fp8_mlp or self.fp8_lm_head):
            return
        matrices = ([w for layer in self.weights.layers for w in (layer.w13_weight, layer.w2_weight)]
                    if self.fp8_mlp else [])
        if self.fp8_lm_head:
            matrices.append(self.weights.lm_head_weight)
        self.fp8_weights = {id(w): PackedFP8Weight(w) for w in matrices}

    def refresh_fp8(self) -> None:
        for packed in self.fp8_weights.values():
            packed.refresh()

    # ---- single kernels --------------------------------------------------------------------------
    def _gemm(self, y, x, w, rows, bufs, status, row_mask=None, row_map=None):
        n, k = w.shape
        packed = self.packed_weights.get(id(w)) if rows == 1 and row_map is None else None
        if packed is not None:  # single-request decode: the 12-bit weight stream (lfm25_cuda.py:124-126)
            packed.linear(x[:1], out=y[:1], row_mask=row_mask)
            return
        nv.call("cgym_gemm_scatter", nv.ptr(y), nv.ptr(x), nv.ptr(w), nv.ptr(row_mask), nv.ptr(row_map), rows, n, k,
                self.dt, self.gemm_impl, nv.ptr(bufs.gemm_ws), bufs.gemm_ws.numel(), nv.ptr(status),
                nv.stream_ptr(w.device))

    def _gemm_fp8(self, y, xq, xs, packed, rows, bufs, status, row_mask=None, row_map=None):
        n, k = packed.values.shape
        nv.call("cgym_gemm_fp8_scatter", nv.ptr(y), nv.ptr(xq), nv.ptr(xs), nv.ptr(packed.values),
                nv.ptr(packed.scales), nv.ptr(row_mask), nv.ptr(row_map), rows, n, k, self.gemm_impl,
                nv.ptr(bufs.gemm_ws), bufs.gemm_ws.numel(), nv.ptr(status), nv.stream_ptr(y.device))

    def _rmsnorm(self, y, x, w, rows, residual=None, sum_out=None):
        nv.call("cgym_rmsnorm", nv.ptr(y), nv.ptr(sum_out), nv.ptr(x), nv.ptr(residual), nv.ptr(w), rows,
                self.cfg.hidden_size, float(self.cfg.norm_eps), self.dt, nv.stream_ptr(x.device))

    def _rmsnorm_quant(self, q, s, x, w, rows, residual=None, sum_out=None):
        nv.call("cgym_rmsnorm_quant", nv.ptr(q), nv.ptr(s), nv.ptr(sum_out), nv.ptr(x), nv.ptr(residual), nv.ptr(w),
                rows, self.cfg.hidden_size, float(self.cfg.norm_eps), nv.stream_ptr(x.device))

    # ---- the layer stack ---------------------------------------------------------------------------
    def _layers(self, bufs: ForwardBuffers, cache: PagedHybridCache, rows: int, *, decode: bool,
                positions, slots, active, kv_lens, cu_seqlens=None, seq_slots=None, seq_starts=None, n_seqs=0,
                tiles=None):
        """Runs every layer over bufs.embed[:rows]; returns (branch, residual) for the final norm."""
        cfg, dev = self.cfg, self.weights.device
        stream = nv.stream_ptr(dev)
        status = cache.status
        hq, f, h = cfg.num_attention_heads, cfg.mlp_hidden_size, cfg.hidden_size
        use_fp8 = self.fp8_mlp and decode
        x, residual = bufs.embed, None
        for layer in self.weights.layers:
            # operator norm; the first layer has nothing to add and its residual is the embedding
            if residual is None:
                self._rmsnorm(bufs.normed, x, layer.operator_norm_weight, rows)
                residual = x
            else:
                self._rmsnorm(bufs.normed, x, layer.operator_norm_weight, rows, residual, bufs.residual)
                residual = bufs.residual
            if layer.attention is not None:
                a = layer.attention
                self._gemm(bufs.qkv, bufs.normed, a.qkv_weight, rows, bufs, status)
                nv.call("cgym_qk_norm_rope_append", nv.ptr(bufs.q), None, None, nv.ptr(bufs.qkv),
                        nv.ptr(a.q_norm_weight), nv.ptr(a.k_norm_weight), nv.ptr(self.rope_cos), nv.ptr(self.rope_sin),
                        nv.ptr(positions), nv.ptr(slots), nv.ptr(active), cache.kv, a.cache_index, rows, hq,
                        float(cfg.norm_eps), self.dt, nv.ptr(status), stream)
                if tiles is not None:
                    row0, ntok, tslot, pos0, n_tiles = tiles
                    nv.call("cgym_prefill_attention", nv.ptr(bufs.attended), nv.ptr(bufs.q), nv.ptr(row0), nv.ptr(ntok),
                            nv.ptr(tslot), nv.ptr(pos0), cache.kv, a.cache_index, n_tiles, hq, self.scale, self.dt,
                            nv.ptr(status), stream)
                else:
                    nv.call("cgym_paged_attention", nv.ptr(bufs.attended), nv.ptr(bufs.q), nv.ptr(kv_lens),
                            nv.ptr(slots), nv.ptr(active), cache.kv, a.cache_index, rows, hq, self.scale,
                            bufs.attn_splits if decode else 1, nv.ptr(bufs.attn_ws), self.dt, self.attn_impl,
                            nv.ptr(status), stream)
                self._gemm(bufs.branch, bufs.attended, a.out_weight, rows, bufs, status)
            else:
                c = layer.conv
                self._gemm(bufs.bcx, bufs.normed, c.in_weight, rows, bufs, status)
                state = cache.conv_layer(c.cache_index)
                if decode:
                    nv.call("cgym_conv_update", nv.ptr(bufs.conv_out), nv.ptr(state), nv.ptr(bufs.bcx),
                            nv.ptr(c.conv_weight), nv.ptr(active), nv.ptr(slots), rows, h, self.dt, stream)
                else:
                    nv.call("cgym_conv_prefill", nv.ptr(bufs.conv_out), nv.ptr(state), nv.ptr(bufs.bcx),
                            nv.ptr(c.conv_weight), nv.ptr(cu_seqlens), nv.ptr(seq_slots), nv.ptr(seq_starts), n_seqs,
                            rows, h, self.dt, stream)
                self._gemm(bufs.branch, bufs.conv_out, c.out_weight, rows, bufs, status)
            # ffn norm fuses (residual + operator output); the sum becomes the new residual
            sum_out = bufs.residual
            if use_fp8:
                self._rmsnorm_quant(bufs.normed_q, bufs.normed_s, bufs.branch, layer.ffn_norm_weight, rows, residual, sum_out)
                self._gemm_fp8(bufs.gate_up, bufs.normed_q, bufs.normed_s, self.fp8_weights[id(layer.w13_weight)], rows, bufs, status)
                nv.call("cgym_swiglu_quant", nv.ptr(bufs.activated_q), nv.ptr(bufs.activated_s), nv.ptr(bufs.gate_up),
                        rows, f, stream)
                self._gemm_fp8(bufs.branch, bufs.activated_q, bufs.activated_s, self.fp8_weights[id(layer.w2_weight)], rows, bufs, status)
            else:
                self._rmsnorm(bufs.normed, bufs.branch, layer.ffn_norm_weight, rows, residual, sum_out)
                self._gemm(bufs.gate_up, bufs.normed, layer.w13_weight, rows, bufs, status)
                nv.call("cgym_swiglu", nv.ptr(bufs.activated), nv.ptr(bufs.gate_up), rows, f, self.dt, stream)
                self._gemm(bufs.branch, bufs.activated, layer.w2_weight, rows, bufs, status)
            residual = sum_out
            x = bufs.branch
        return x, residual

    def _embed(self, bufs, tokens, rows):
        cfg = self.cfg
        nv.call("cgym_embedding", nv.ptr(bufs.embed), nv.ptr(self.weights.embed_tokens), nv.ptr(tokens), rows,
                cfg.hidden_size, cfg.vocab_size, self.dt, nv.stream_ptr(self.weights.device))

    def _head(self, bufs, logits, hidden_rows, rows, status, row_mask=None, row_map=None):
        if self.fp8_lm_head:
            packed = self.fp8_weights[id(self.weights.lm_head_weight)]
            self._gemm_fp8(logits, bufs.normed_q, bufs.normed_s, packed, rows, bufs, status, row_mask, row_map)
        else:
            self._gemm(logits, hidden_rows, self.weights.lm_head_weight, rows, bufs, status, row_mask, row_map)

    # ---- public sequences ------------------------------------------------------------------------------
    def decode_step(self, bufs: ForwardBuffers, cache: PagedHybridCache, tokens, active, logits, *, slots=None,
                    rows: int | None = None, kv_lens=None, positions=None, logits_rows=None) -> None:
        """One token per row. Rows with active == 0 leave KV, conv taps and their logits row untouched.
        positions are the slots' current seq_lens (pass them when the caller already holds them per row, e.g.
        a contiguous range of slots); the caller advances seq_lens afterwards.
        kv_lens: the per-row attention lengths cgym_step_begin wrote (seq_lens + 1); computed here with
        a torch op when the caller did not ask step_begin for them.
        logits_rows (int32 per row, optional): row r's logits go to logits[logits_rows[r]] (negative: nowhere);
        a step over a compacted set of rows writes each row's logits into its slot's row this way."""
        rows = tokens.numel() if rows is None else rows
        self._embed(bufs, tokens, rows)
        # a decode row at cache length L writes position L and then attends to L + 1 tokens
        if positions is None:
            positions = cache.seq_lens if slots is None else bufs_positions(cache, slots)
        if kv_lens is None:
            kv_lens = self._kv_lens_plus_one(cache, positions)
        x, residual = self._layers(bufs, cache, rows, decode=True, positions=positions, slots=slots, active=active,
                                   kv_lens=kv_lens)
        if self.fp8_lm_head:
            self._rmsnorm_quant(bufs.normed_q, bufs.normed_s, x, self.weights.embedding_norm_weight, rows, residual, bufs.residual)
        else:
            self._rmsnorm(bufs.final, x, self.weights.embedding_norm_weight, rows, residual, bufs.residual)
        self._head(bufs, logits, bufs.final, rows, cache.status, row_mask=active, row_map=logits_rows)

    @staticmethod
    def kv_lens_buffer(cache) -> torch.Tensor:
        """int32 [slots] scratch for the per-row attention lengths of a decode step."""
        if not hasattr(cache, "_kv_lens"):
            cache._kv_lens = torch.empty_like(cache.seq_lens)
        return cache._kv_lens

    def _kv_lens_plus_one(self, cache, positions):
        # torch op on a tiny int32 vector (capturable); keeps the attention ABI "attend to [0, kv_len)"
        out = self.kv_lens_buffer(cache)
        torch.add(positions, 1, out=out[:positions.numel()])
        return out

    def prefill_chunk(self, bufs: ForwardBuffers, cache: PagedHybridCache, tokens, positions, token_slots, kv_lens,
                      cu_seqlens, seq_slots, seq_starts, n_seqs: int, rows: int, *, last_rows=None, logits=None,
                      return_hidden: bool = False, tiles=None):
        """Packed rows of one or more sequences (or chunks of them). Pages must be reserved by the caller.

        last_rows (int64 row indices) selects the rows whose logits are wanted (written to ``logits``);
        with return_hidden the final-normed hidden states of all rows are returned instead."""
        self._embed(bufs, tokens, rows)
        x, residual = self._layers(bufs, cache, rows, decode=False, positions=positions, slots=token_slots,
                                   active=None, kv_lens=kv_lens, cu_seqlens=cu_seqlens, seq_slots=seq_slots,
                                   seq_starts=seq_starts, n_seqs=n_seqs,
                                   tiles=tiles if self.attn_impl != 1 else None)
        if return_hidden:
            self._rmsnorm(bufs.final, x, self.weights.embedding_norm_weight, rows, residual, bufs.residual)
            return bufs.final[:rows]
        if last_rows is None:
            return None
        # only the selected rows go through the final norm and the LM head
        n = last_rows.numel()
        picked_x = x.index_select(0, last_rows)
        picked_r = residual.index_select(0, last_rows)
        final = torch.empty_like(picked_x)
        summed = torch.empty_like(picked_x)
        self._rmsnorm(final, picked_x, self.weights.embedding_norm_weight, n, picked_r, summed)
        nk = self.weights.lm_head_weight.shape
        nv.call("cgym_gemm", nv.ptr(logits), nv.ptr(final), nv.ptr(self.weights.lm_head_weight), None, n, nk[0], nk[1],
                self.dt, self.gemm_impl, nv.ptr(bufs.gemm_ws), bufs.gemm_ws.numel(), nv.ptr(cache.status),
                nv.stream_ptr(self.weights.device))
        return logits


def bufs_positions(cache: PagedHybridCache, slots: torch.Tensor) -> torch.Tensor:
    """Cache lengths of the rows' slots (padding rows, slot < 0, read slot 0 and are masked later)."""
    return cache.seq_lens.index_select(0, slots.clamp_min(0).long())
