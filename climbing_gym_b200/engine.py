"""LFM25Engine: the token-level rollout engine, B200-native.

Public surface and error behaviour follow the reference engine
(src/climbing_gym/inference/lfm25_engine.py:479-1163): ``from_pretrained / from_model``,
``prefill``, ``fork``, ``decode_step``, ``generate``, ``score_completions``,
``enable_cuda_graphs / disable_cuda_graphs``, ``generation_session``, ``sync_from_model``,
``release_inference_buffers``. Differences are under the API:

* every tensor op on the path is one of this package's sm_100a kernels behind the C ABI; the
  engine refuses to run without them (no eager PyTorch or CPU path);
* the cache is paged (``PagedHybridCache``) and prompts are prefetched as packed variable-length
  rows, split at ``max_prefill_tokens`` even inside one prompt (chunked prefill), instead of
  padded groups of whole prompts (reference grouping rule: lfm25_engine.py:646-665);
* ``generate`` always runs through the captured step graph; ``enable_cuda_graphs`` only selects
  its options (FP8 MLP / KV / head, prefill budget), so calling ``generate`` first enables the
  default configuration.
"""
from __future__ import annotations

import json
import math
from pathlib import Path
from typing import Any, Sequence

import numpy as np
import torch

from . import _native as nv
from .config import LFM2Config, LFM25SamplingConfig
from .model import ForwardBuffers
from .paged import PagedHybridCache
from .types import LFM25DecodeBatch, LFM25GenerationOutput, LFM25PrefixBatch, LFM25StepOutput
from .weights import LFM25PackedWeights


def _resolve_dtype(dtype, *, device: torch.device) -> torch.dtype:
    if isinstance(dtype, torch.dtype):
        return dtype
    if dtype is None or str(dtype).lower() == "auto":
        return torch.bfloat16 if device.type == "cuda" else torch.float32
    names = {"bf16": torch.bfloat16, "bfloat16": torch.bfloat16, "fp16": torch.float16, "float16": torch.float16,
             "fp32": torch.float32, "float32": torch.float32}
    try:
        return names[str(dtype).strip().lower()]
    except KeyError as exc:
        raise ValueError(f"Unsupported dtype: {dtype!r}") from exc


def flatten_token_batches(input_ids: Sequence[Sequence[int]], *, device=None):
    """Python batch of token ids -> (flat int64 ids, int32 cu_seqlens, max length)."""
    if not input_ids:
        raise ValueError("input_ids must contain at least one prompt")
    lengths = [len(item) for item in input_ids]
    if any(length <= 0 for length in lengths):
        raise ValueError("empty prompts are not supported")
    dev = torch.device(device or "cpu")
    flat = torch.tensor([token for item in input_ids for token in item], device=dev, dtype=torch.long)
    cu = torch.zeros(len(lengths) + 1, device=dev, dtype=torch.int32)
    cu[1:] = torch.tensor(lengths, device=dev, dtype=torch.int32).cumsum(0)
    return flat, cu, max(lengths)


class LFM25Engine:
    def __init__(self, weights: LFM25PackedWeights, *, max_model_len: int | None = None):
        self.weights = weights
        self.config = weights.config
        self.device = weights.device
        self.dtype = weights.dtype
        if self.device.type != "cuda":
            raise RuntimeError("climbing_gym_b200 runs on a CUDA device only (B200, sm_100a); there is no CPU path")
        nv.load()  # fail loudly now if the kernels are not built
        self.max_model_len = int(max_model_len or min(int(self.config.max_position_embeddings), 32768))
        if self.max_model_len <= 0:
            raise ValueError("max_model_len must be > 0")
        if self.max_model_len > int(self.config.max_position_embeddings):
            raise ValueError("max_model_len cannot exceed config.max_position_embeddings")
        self._cuda_decoder = None
        self.policy_version = 0
        self._prefill_bufs: ForwardBuffers | None = None
        self._build_rope_cache()

    # ---- construction ------------------------------------------------------------------------------
    @classmethod
    def from_pretrained(cls, model_dir, *, device=None, dtype=None, max_model_len=None) -> "LFM25Engine":
        metadata_path = Path(model_dir) / "config.json"
        if metadata_path.exists() and json.loads(metadata_path.read_text()).get("model_type") == "lfm3":
            raise ValueError("LFM3 checkpoints are not supported by the B200 engine")
        dev = torch.device(device or "cuda")
        weights = LFM25PackedWeights.from_pretrained(model_dir, device=dev, dtype=_resolve_dtype(dtype, device=dev))
        return cls(weights, max_model_len=max_model_len)

    @classmethod
    def from_model(cls, model: Any, *, device=None, dtype=None, max_model_len=None) -> "LFM25Engine":
        first = next(model.parameters())
        dev = torch.device(device or first.device)
        weights = LFM25PackedWeights.from_model(model, device=dev, dtype=_resolve_dtype(dtype or first.dtype, device=dev))
        return cls(weights, max_model_len=max_model_len)

    @classmethod
    def from_state_dict(cls, config: LFM2Config, state_dict, *, device="cuda", dtype=torch.bfloat16,
                        max_model_len=None) -> "LFM25Engine":
        weights = LFM25PackedWeights.from_state_dict(config, state_dict, device=torch.device(device), dtype=dtype)
        return cls(weights, max_model_len=max_model_len)

    def _build_rope_cache(self) -> None:
        d = self.config.head_dim
        inv = 1.0 / (self.config.rope_theta ** (torch.arange(0, d, 2, dtype=torch.float32, device=self.device) / d))
        positions = torch.arange(self.max_model_len, dtype=torch.float32, device=self.device)
        freqs = torch.einsum("i,j->ij", positions, inv)
        self._rope_cos, self._rope_sin = freqs.cos().contiguous(), freqs.sin().contiguous()

    # ---- weight sync / lifecycle ------------------------------------------------------------------------
    @torch.inference_mode()
    def sync_from_model(self, model: Any, *, drain_timeout: int | float = 300) -> "LFM25Engine":
        timeout = float(drain_timeout)
        if not math.isfinite(timeout) or timeout < 0.0:
            raise ValueError("drain_timeout must be finite and >= 0")
        if self._cuda_decoder is not None and self._cuda_decoder._active_session is not None:
            raise RuntimeError("Close the native generation session before synchronizing weights")
        self.weights.copy_from_model_(model)
        if self._cuda_decoder is not None:
            self._cuda_decoder.refresh_weights()
        self.policy_version += 1
        return self

    def weights_updated(self) -> None:
        """Call after the packed buffers were overwritten in place by something other than
        sync_from_model (e.g. the NCCL weight broadcast): re-quantises FP8 copies, bumps the version."""
        if self._cuda_decoder is not None:
            if self._cuda_decoder._active_session is not None:
                raise RuntimeError("Close the native generation session before synchronizing weights")
            self._cuda_decoder.refresh_weights()
        self.policy_version += 1

    def release_inference_buffers(self) -> None:
        decoder = self._cuda_decoder
        if decoder is None:
            return
        if decoder._active_session is not None:
            raise RuntimeError("Close the native generation session before releasing inference buffers")
        if not (decoder.graphs or decoder.packed_weights or decoder.fp8_weights):
            return
        torch.cuda.synchronize(self.device)
        decoder.clear()
        self._prefill_bufs = None
        torch.cuda.empty_cache()

    def enable_cuda_graphs(self, *, max_graphs: int = 2, bf16_weight_packing: bool = True,
                           max_prefill_tokens: int = 4096, fp8_mlp: bool = False, fp8_kv: bool = False,
                           adaptive_batching: bool = False, fp8_lm_head: bool = False, **extra) -> None:
        from .decoder import B200Decoder

        if self._cuda_decoder is not None and self._cuda_decoder._active_session is not None:
            raise RuntimeError("Close the native generation session before reconfiguring CUDA graphs")
        self._cuda_decoder = B200Decoder(self, max_graphs=max_graphs, bf16_weight_packing=bf16_weight_packing,
                                         max_prefill_tokens=max_prefill_tokens, fp8_mlp=fp8_mlp, fp8_kv=fp8_kv,
                                         adaptive_batching=adaptive_batching, fp8_lm_head=fp8_lm_head, **extra)
        self._prefill_bufs = None

    def disable_cuda_graphs(self) -> None:
        if self._cuda_decoder is not None:
            self._cuda_decoder.clear()
        self._cuda_decoder = None

    def _decoder(self):
        if self._cuda_decoder is None:
            self.enable_cuda_graphs()
        return self._cuda_decoder

    def generation_session(self, *, max_batch_size: int, max_new_tokens: int, cache_len: int | None = None,
                           behavior_topk: int = 0, profile_timings: bool = False, queue_capacity: int = 0):
        """``queue_capacity`` > 0 opens the session with a device-side admission queue of that many parked
        prompts (``session.enqueue``): finished requests are then evicted and queued ones admitted inside the
        decode graph, without a host round-trip between polls."""
        if self._cuda_decoder is None:
            raise RuntimeError("generation_session requires enable_cuda_graphs()")
        from .session import LFM25GenerationSession

        return LFM25GenerationSession(self._cuda_decoder, max_batch_size=max_batch_size, max_new_tokens=max_new_tokens,
                                      cache_len=cache_len, behavior_topk=behavior_topk, profile_timings=profile_timings,
                                      queue_capacity=queue_capacity)

    # ---- cache ------------------------------------------------------------------------------------------
    def _empty_cache(self, *, max_slots: int, max_seq_len: int, fp8_kv: bool = False, page_size: int = 64,
                     n_pages: int | None = None, spare_rows: int = 0) -> PagedHybridCache:
        if max_slots <= 0:
            raise ValueError("max_slots must be > 0")
        if max_seq_len <= 0:
            raise ValueError("max_seq_len must be > 0")
        if max_seq_len > self.max_model_len:
            raise ValueError(f"max_seq_len={max_seq_len} exceeds engine max_model_len={self.max_model_len}")
        cfg = self.config
        return PagedHybridCache(n_attn_layers=self.weights.num_attention_layers, n_conv_layers=self.weights.num_conv_layers,
                                n_slots=max_slots, max_seq_len=max_seq_len, n_kv_heads=cfg.num_key_value_heads,
                                head_dim=cfg.head_dim, hidden_size=cfg.hidden_size, dtype=self.dtype,
                                device=self.device, page_size=page_size, n_pages=n_pages, fp8_kv=fp8_kv,
                                spare_rows=spare_rows)

    # ---- prefill ----------------------------------------------------------------------------------------
    def _split_prompts(self, input_ids, cu_seqlens, max_seqlen) -> list[list[int]]:
        ids = torch.as_tensor(input_ids).reshape(-1).to("cpu", torch.long)
        cu = torch.as_tensor(cu_seqlens).reshape(-1).to("cpu", torch.long)
        if cu.numel() < 2:
            raise ValueError("cu_seqlens must contain at least [0, total_tokens]")
        if int(cu[0]) != 0:
            raise ValueError("cu_seqlens must start at 0")
        if int(cu[-1]) != int(ids.numel()):
            raise ValueError("cu_seqlens[-1] must equal input_ids.numel()")
        lengths = cu[1:] - cu[:-1]
        if bool((lengths <= 0).any()):
            raise ValueError("empty prompts are not supported")
        if int(lengths.max()) > int(max_seqlen):
            raise ValueError("max_seqlen is smaller than at least one prompt")
        flat, bounds = ids.tolist(), cu.tolist()
        return [flat[bounds[i]:bounds[i + 1]] for i in range(len(bounds) - 1)]

    def _prefill_buffers(self, rows: int) -> ForwardBuffers:
        if self._prefill_bufs is None or self._prefill_bufs.rows < rows:
            self._prefill_bufs = ForwardBuffers(self.weights, rows, fp8=False)
        return self._prefill_bufs

    def _runner(self):
        return self._decoder().runner

    @torch.inference_mode()
    def _prefill_packed(self, cache: PagedHybridCache, slots: Sequence[int], prompts, starts: Sequence[int],
                        logits: torch.Tensor | None, max_prefill_tokens: int | None, *,
                        flat_tokens: torch.Tensor | None = None, return_hidden: bool = False,
                        logits_rows: Sequence[int] | None = None):
        """Run prompt tokens (or continuation tokens starting at cache position ``starts[i]``) into
        ``slots``. ``prompts`` is a list of token lists, or a list of lengths when ``flat_tokens``
        (int64, on the device, all sequences back to back) carries the ids. Rows are packed back to
        back and cut every ``max_prefill_tokens`` rows, also in the middle of a prompt; a cut prompt
        continues from its cached prefix and conv taps in the next chunk. The last token's logits of
        sequence i land in ``logits[slots[i]]`` (``logits[logits_rows[i]]`` when given). Returns [(pieces, hidden)] when return_hidden, where
        a piece is (slot, n_rows, start_position, is_last_piece_of_its_sequence)."""
        budget = int(max_prefill_tokens or 4096)
        if budget <= 0:
            raise ValueError("max_prefill_tokens must be positive")
        dev = self.device
        if flat_tokens is None:
            lengths = [len(p) for p in prompts]
            host = np.fromiter((t for p in prompts for t in p), dtype=np.int64, count=sum(lengths))
            flat_tokens = torch.from_numpy(host).to(dev, non_blocking=True)
        else:
            lengths = [int(n) for n in prompts]
        for length, start in zip(lengths, starts):
            if length <= 0:
                raise ValueError("empty prompts are not supported")
            if start + length > cache.max_seq_len:
                raise RuntimeError("cache capacity exceeded")
            if start + length > self.max_model_len:
                raise RuntimeError("position exceeds engine max_model_len")
        runner = self._runner()
        # cut the work into chunks of at most `budget` rows; a chunk is a contiguous range of flat_tokens
        chunks, current, used = [], [], 0
        for slot, length, start in zip(slots, lengths, starts):
            offset = 0
            while offset < length:
                take = min(length - offset, budget - used)
                current.append((slot, take, start + offset, offset + take == length))
                used += take
                offset += take
                if used == budget:
                    chunks.append(current)
                    current, used = [], 0
        if current:
            chunks.append(current)
        hidden_parts, consumed = [], 0
        group = self.config.num_attention_heads // self.config.num_key_value_heads
        use_tiles = (self.dtype == torch.bfloat16 and cache.page_size == 64 and self.config.head_dim == 64
                     and group <= 16)
        tile_tokens = max(1, 128 // group)
        for chunk in chunks:
            counts = [piece[1] for piece in chunk]
            rows, n = sum(counts), len(chunk)
            bufs = self._prefill_buffers(rows)
            positions = np.concatenate([np.arange(piece[2], piece[2] + piece[1], dtype=np.int32) for piece in chunk])
            token_slots = np.repeat(np.asarray([piece[0] for piece in chunk], dtype=np.int32), counts)
            cu = np.zeros(n + 1, dtype=np.int32)
            cu[1:] = np.cumsum(counts)
            seq_slots = np.asarray([piece[0] for piece in chunk], dtype=np.int32)
            seq_starts = np.asarray([piece[2] for piece in chunk], dtype=np.int32)
            seq_ends = seq_starts + np.asarray(counts, dtype=np.int32)
            # query tiles of the tensor-core prefill attention: <= 128 / group consecutive tokens of one piece
            tile_fields, n_tiles = [np.zeros(0, np.int32)] * 4, 0
            if use_tiles:
                starts_t = [np.arange(0, c, tile_tokens, dtype=np.int32) for c in counts]
                per_piece = [len(s) for s in starts_t]
                offs = np.concatenate(starts_t)
                base = np.repeat(cu[:-1], per_piece)
                remaining = np.repeat(np.asarray(counts, dtype=np.int32), per_piece) - offs
                tile_fields = [base + offs, np.minimum(remaining, tile_tokens).astype(np.int32),
                               np.repeat(seq_slots, per_piece), np.repeat(seq_starts, per_piece) + offs]
                n_tiles = len(offs)
            meta = np.concatenate([positions, token_slots, positions + 1, cu, seq_slots, seq_starts, seq_ends,
                                   *tile_fields]).astype(np.int32)
            meta_dev = torch.from_numpy(meta).to(dev, non_blocking=True)
            tokens_dev = flat_tokens[consumed:consumed + rows]
            consumed += rows
            views, o = [], 0
            for size in (rows, rows, rows, n + 1, n, n, n, n_tiles, n_tiles, n_tiles, n_tiles):
                views.append(meta_dev[o:o + size])
                o += size
            positions_d, slots_d, kv_lens_d, cu_d, seq_slots_d, seq_starts_d, seq_ends_d = views[:7]
            tiles = (*views[7:], n_tiles) if use_tiles else None
            cache.reserve(seq_slots_d, seq_ends_d)
            finished = [i for i, piece in enumerate(chunk) if piece[3]]
            if return_hidden:
                hidden = runner.prefill_chunk(bufs, cache, tokens_dev, positions_d, slots_d, kv_lens_d, cu_d,
                                              seq_slots_d, seq_starts_d, n, rows, return_hidden=True, tiles=tiles)
                hidden_parts.append((chunk, hidden.clone()))
            elif finished and logits is not None:
                last_rows = torch.from_numpy(cu[1:][finished].astype(np.int64) - 1).to(dev, non_blocking=True)
                out = torch.empty((len(finished), self.config.vocab_size), device=dev, dtype=self.dtype)
                runner.prefill_chunk(bufs, cache, tokens_dev, positions_d, slots_d, kv_lens_d, cu_d, seq_slots_d,
                                     seq_starts_d, n, rows, last_rows=last_rows, logits=out, tiles=tiles)
                dest = seq_slots[finished].astype(np.int64)
                if logits_rows is not None:
                    row_of = dict(zip(slots, logits_rows))
                    dest = np.asarray([row_of[int(s)] for s in dest], dtype=np.int64)
                dest = torch.from_numpy(dest).to(dev, non_blocking=True)
                logits.index_copy_(0, dest, out)
            else:
                runner.prefill_chunk(bufs, cache, tokens_dev, positions_d, slots_d, kv_lens_d, cu_d, seq_slots_d,
                                     seq_starts_d, n, rows, tiles=tiles)
            cache.row_lens.index_copy_(0, seq_slots_d.long(), seq_ends_d)
        return hidden_parts

    def _split_lengths(self, input_ids, cu_seqlens, max_seqlen):
        """(flat int64 ids on the device, host list of prompt lengths); only cu_seqlens visits the host."""
        ids = torch.as_tensor(input_ids).reshape(-1)
        cu = torch.as_tensor(cu_seqlens).reshape(-1).to("cpu", torch.long)
        if cu.numel() < 2:
            raise ValueError("cu_seqlens must contain at least [0, total_tokens]")
        if int(cu[0]) != 0:
            raise ValueError("cu_seqlens must start at 0")
        if int(cu[-1]) != int(ids.numel()):
            raise ValueError("cu_seqlens[-1] must equal input_ids.numel()")
        lengths = (cu[1:] - cu[:-1]).tolist()
        if min(lengths) <= 0:
            raise ValueError("empty prompts are not supported")
        if max(lengths) > int(max_seqlen):
            raise ValueError("max_seqlen is smaller than at least one prompt")
        return ids.to(device=self.device, dtype=torch.long, non_blocking=True), lengths

    @torch.inference_mode()
    def prefill(self, input_ids, cu_seqlens, max_seqlen: int, *, max_cache_len: int | None = None,
                cache: PagedHybridCache | None = None, max_prefill_tokens: int | None = None,
                logits_buffer: torch.Tensor | None = None, slots: Sequence[int] | None = None) -> LFM25PrefixBatch:
        flat_ids, lengths = self._split_lengths(input_ids, cu_seqlens, max_seqlen)
        n = len(lengths)
        cache_len = int(max_cache_len or max_seqlen)
        if cache is None:
            cache = self._empty_cache(max_slots=n, max_seq_len=cache_len)
        elif cache.max_seq_len < cache_len or (slots is None and cache.max_slots < n):
            raise ValueError("destination cache does not fit the prompt batch")
        if max_prefill_tokens is not None and max_prefill_tokens <= 0:
            raise ValueError("max_prefill_tokens must be positive")
        slots = list(range(n)) if slots is None else list(slots)
        shape = (cache.max_slots, self.config.vocab_size)
        if logits_buffer is None:
            logits_buffer = torch.empty(shape, device=self.device, dtype=self.dtype)
        elif tuple(logits_buffer.shape) != shape or logits_buffer.dtype != self.dtype or logits_buffer.device != self.device:
            raise ValueError("logits buffer must match the prompt batch, vocabulary, device, and model dtype")
        self._prefill_packed(cache, slots, lengths, [0] * n, logits_buffer,
                             max_prefill_tokens or self._decoder().max_prefill_tokens, flat_tokens=flat_ids)
        slot_index = torch.tensor(slots, device=self.device, dtype=torch.int64)
        return LFM25PrefixBatch(cache=cache, next_token_logits=logits_buffer.index_select(0, slot_index),
                                prompt_lengths=torch.tensor(lengths, device=self.device, dtype=torch.int32),
                                input_ids=flat_ids, slots=slot_index)

    # ---- generate / score -----------------------------------------------------------------------------------
    @torch.inference_mode()
    def generate(self, input_ids, cu_seqlens, max_seqlen: int, repeats: int,
                 sampling: LFM25SamplingConfig | None = None) -> LFM25GenerationOutput:
        return self._decoder().generate(input_ids, cu_seqlens, max_seqlen, repeats, sampling or LFM25SamplingConfig())

    @torch.inference_mode()
    def score_completions(self, prompts, completions, *, max_prefill_tokens: int = 4096,
                          head_chunk_size: int = 256) -> list[tuple]:
        """Raw, untempered log-probs of every completion token given its prompt; packed varlen
        scoring prefill, LM head and log-softmax evaluated ``head_chunk_size`` rows at a time."""
        if len(prompts) != len(completions):
            raise ValueError("prompts and completions must have equal lengths")
        if max_prefill_tokens <= 0 or head_chunk_size <= 0:
            raise ValueError("scoring chunk sizes must be positive")
        if any(not p or not c for p, c in zip(prompts, completions)):
            raise ValueError("scoring requires nonempty prompts and completions")
        sequences = [list(p) + list(c) for p, c in zip(prompts, completions)]
        if any(len(s) > self.max_model_len for s in sequences):
            raise ValueError("scored sequence exceeds max_model_len")
        runner, dev = self._runner(), self.device
        result: list[tuple] = [()] * len(sequences)
        order = sorted(range(len(sequences)), key=lambda i: len(sequences[i]))
        start = 0
        while start < len(order):
            # as many whole sequences as fit the token budget share one scratch cache
            end, total = start, 0
            while end < len(order) and (end == start or total + len(sequences[order[end]]) <= max_prefill_tokens):
                total += len(sequences[order[end]])
                end += 1
            group = order[start:end]
            longest = max(len(sequences[i]) for i in group)
            cache = self._empty_cache(max_slots=len(group), max_seq_len=longest)
            parts = self._prefill_packed(cache, list(range(len(group))), [sequences[i] for i in group],
                                         [0] * len(group), None, max_prefill_tokens, return_hidden=True)
            # stitch per-sequence hidden rows back together (a long sequence may span chunks)
            per_slot: dict[int, list] = {s: [] for s in range(len(group))}
            for chunk, hidden in parts:
                offset = 0
                for slot, count, _, _ in chunk:
                    per_slot[slot].append(hidden[offset:offset + count])
                    offset += count
            selected, targets = [], []
            for slot, i in enumerate(group):
                rows = torch.cat(per_slot[slot])
                selected.append(rows[len(prompts[i]) - 1:len(sequences[i]) - 1])
                targets.extend(completions[i])
            selected = torch.cat(selected).contiguous()
            target_ids = torch.tensor(targets, device=dev, dtype=torch.int64)
            scores = torch.empty(selected.size(0), device=dev, dtype=torch.float32)
            head = self.weights.lm_head_weight
            status = cache.status
            for offset in range(0, selected.size(0), head_chunk_size):
                rows = min(head_chunk_size, selected.size(0) - offset)
                chunk_logits = torch.empty((rows, head.size(0)), device=dev, dtype=self.dtype)
                bufs = self._prefill_buffers(1)
                nv.call("cgym_gemm", nv.ptr(chunk_logits), nv.ptr(selected[offset:offset + rows]), nv.ptr(head), None,
                        rows, head.size(0), head.size(1), runner.dt, runner.gemm_impl, nv.ptr(bufs.gemm_ws),
                        bufs.gemm_ws.numel(), nv.ptr(status), nv.stream_ptr(dev))
                nv.call("cgym_target_logprobs", nv.ptr(scores[offset:offset + rows]), nv.ptr(chunk_logits),
                        nv.ptr(target_ids[offset:offset + rows]), rows, head.size(0), runner.dt, nv.stream_ptr(dev))
            flat = scores.cpu().tolist()
            cursor = 0
            for i in group:
                size = len(completions[i])
                result[i] = tuple(flat[cursor:cursor + size])
                cursor += size
            cache.check_status()
            start = end
        return result

    # ---- step-level API (kept for callers that drive the engine token by token) -----------------------------
    @torch.inference_mode()
    def fork(self, prefix: LFM25PrefixBatch, repeats: int, *, max_cache_len: int | None = None) -> LFM25DecodeBatch:
        if repeats <= 0:
            raise ValueError("repeats must be > 0")
        n = prefix.batch_size
        total = n * int(repeats)
        cache_len = int(max_cache_len or prefix.cache.max_seq_len)
        if cache_len < prefix.cache.max_seq_len:
            raise ValueError("max_cache_len cannot be smaller than the prefix cache")
        source = prefix.cache
        if repeats == 1 and cache_len == source.max_seq_len and source.max_slots == n:
            cache = source
        else:
            cache = self._fork_into_new_cache(prefix, int(repeats), cache_len)
        dev = self.device
        return LFM25DecodeBatch(cache=cache, active_slot_ids=torch.arange(total, device=dev),
                                prompt_indices=torch.arange(n, device=dev).repeat_interleave(repeats),
                                repeat_indices=torch.arange(repeats, device=dev).repeat(n),
                                alive=torch.ones(total, device=dev, dtype=torch.bool))

    def _fork_into_new_cache(self, prefix: LFM25PrefixBatch, repeats: int, cache_len: int) -> PagedHybridCache:
        """A cache of ``batch x repeats`` slots whose slot ``p * repeats + r`` continues prompt ``p``: the
        prefix pages are copied page by page into the first sample of each group (two caches never share a
        pool), the other samples of the group then share them by reference (reference: the dense
        repeat_interleave copy of lfm25_engine.py:735-790)."""
        source, dev, n = prefix.cache, self.device, prefix.batch_size
        rows = (prefix.slots if prefix.slots is not None else torch.arange(n, device=dev)).long()
        cache = self._empty_cache(max_slots=n * repeats, max_seq_len=cache_len, fp8_kv=source.fp8_kv,
                                  page_size=source.page_size)
        lens = source.seq_lens.index_select(0, rows)
        first = torch.arange(n, device=dev, dtype=torch.int32) * repeats
        cache.reserve(first, lens)
        held = torch.arange(source.max_blocks, device=dev)[None, :] * source.page_size < lens[:, None]
        src_pages = source.block_table.index_select(0, rows)[held].long()
        dst_pages = cache.block_table.index_select(0, first.long())[:, :source.max_blocks][held].long()
        cache.kv_pool[:, dst_pages] = source.kv_pool[:, src_pages]
        if cache.kv_scales is not None:
            cache.kv_scales[:, dst_pages] = source.kv_scales[:, src_pages]
        cache.conv_state[:, first.long()] = source.conv_state[:, rows]
        cache.row_lens.index_copy_(0, first.long(), lens)
        if repeats > 1:
            src = first.repeat_interleave(repeats - 1)
            dst = (first[:, None] + torch.arange(1, repeats, device=dev, dtype=torch.int32)[None, :]).reshape(-1)
            cache.fork(src, dst.contiguous(), lens.repeat_interleave(repeats - 1).contiguous())
        cache.check_status()
        return cache

    @torch.inference_mode()
    def decode_step(self, state: LFM25DecodeBatch, input_tokens: torch.Tensor,
                    sampling: LFM25SamplingConfig | None = None) -> LFM25StepOutput:
        """Append one token to every slot in ``state.active_slot_ids`` (one input token each, in that order)
        and sample the next one; other slots of the cache are not touched. Outputs are indexed like
        ``active_slot_ids`` (reference: src/climbing_gym/inference/lfm25_engine.py:715-738). Top-k / top-p are
        applied through the device threshold kernel; a repetition penalty needs the generate loop's seen-token
        mask and is refused here."""
        sampling = sampling or LFM25SamplingConfig()
        cache, dev = state.cache, self.device
        slots = state.active_slot_ids.to(device=dev, dtype=torch.int32).reshape(-1)
        tokens = input_tokens.to(device=dev, dtype=torch.long).reshape(-1).contiguous()
        n = int(slots.numel())
        if tokens.numel() != n:
            raise ValueError("input_tokens must have one token per active slot")
        if float(sampling.repetition_penalty) != 1.0:
            raise ValueError("decode_step does not apply a repetition penalty: use generate, which tracks the seen tokens")
        if n == 0:
            raise ValueError("decode_step needs at least one active slot")
        rows = slots.long()
        if bool((slots < 0).any()) or bool((slots >= cache.max_slots).any()) or rows.unique().numel() != n:
            raise ValueError("active_slot_ids must be distinct slots of the cache")
        if bool((cache.seq_lens.index_select(0, rows) >= cache.max_seq_len).any()):
            raise RuntimeError("cache capacity exceeded")
        runner = self._runner()
        vocab = self.config.vocab_size
        bufs = ForwardBuffers(self.weights, n, fp8=runner.fp8_mlp or runner.fp8_lm_head)
        active = torch.ones(n, device=dev, dtype=torch.uint8)
        logits = torch.empty((n, vocab), device=dev, dtype=self.dtype)
        kv_lens = torch.empty(n, device=dev, dtype=torch.int32)
        stream = nv.stream_ptr(dev)
        nv.call("cgym_step_begin", cache.pool, nv.ptr(cache.seq_lens), None, None, nv.ptr(active), nv.ptr(slots),
                nv.ptr(kv_lens), n, nv.ptr(cache.status), stream)
        runner.decode_step(bufs, cache, tokens, active, logits, slots=slots, rows=n, kv_lens=kv_lens)
        cache.seq_lens.index_add_(0, rows, torch.ones(n, device=dev, dtype=torch.int32))
        out_tokens = torch.empty(n, device=dev, dtype=torch.int64)
        out_logp = torch.empty(n, device=dev, dtype=torch.float32)
        seeds = torch.full((n,), int(sampling.seed) & 0x7FFFFFFFFFFFFFFF, device=dev, dtype=torch.int64)
        steps = torch.zeros(n, device=dev, dtype=torch.int64)
        temps = torch.full((n,), float(sampling.temperature), device=dev, dtype=torch.float32)
        offsets = torch.arange(n, device=dev, dtype=torch.int64) * vocab
        filtered = sampling.temperature > 0.0 and (0 < sampling.top_k < vocab or sampling.top_p < 1.0)
        if filtered:
            # same kernels as the generate loop: a per-row value threshold, then the sampler restricted to it
            from .decoder import SlotState

            scratch = SlotState(n, 1, vocab, int(self.config.eos_token_id), torch.zeros(n, device=dev, dtype=torch.int32))
            scratch.configure(list(range(n)), limits=2, seeds=int(sampling.seed) & 0x7FFFFFFFFFFFFFFF,
                              temperatures=float(sampling.temperature), ignore_eos=1, stop_offsets=0,
                              rng_offsets=[row * vocab for row in range(n)])
            scratch.top_k.fill_(int(sampling.top_k))
            scratch.top_p.fill_(float(sampling.top_p))
            dt = nv.dtype_code(self.dtype)
            nv.call("cgym_filter_thresholds", nv.ptr(scratch.min_logits), nv.ptr(logits), nv.ptr(scratch.temperatures),
                    nv.ptr(scratch.top_k), nv.ptr(scratch.top_p), nv.ptr(scratch.alive), n, vocab, dt, stream)
            import ctypes as C

            nv.call("cgym_sample_record", nv.ptr(logits), C.byref(scratch.struct_filtered), None, nv.ptr(out_tokens),
                    nv.ptr(out_logp), n, vocab, dt, nv.ptr(scratch.sample_ws), stream)
        else:
            nv.call("cgym_sample", nv.ptr(out_tokens), nv.ptr(out_logp), nv.ptr(logits), nv.ptr(seeds), nv.ptr(steps),
                    nv.ptr(temps), nv.ptr(offsets), n, vocab, nv.dtype_code(self.dtype), None, stream)
        reasons = torch.zeros(n, device=dev, dtype=torch.int8)
        if not sampling.ignore_eos:
            reasons[out_tokens == int(self.config.eos_token_id)] = 1
        for stop in sampling.stop_token_ids:
            reasons[(reasons == 0) & (out_tokens == int(stop))] = 2
        cache.check_status()
        return LFM25StepOutput(token_ids=out_tokens, raw_logprobs=out_logp if sampling.return_logprobs else None,
                               sampling_logprobs=out_logp if sampling.return_logprobs else None,
                               finished=reasons != 0, finish_reasons=reasons, logits=logits)
