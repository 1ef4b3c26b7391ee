"""CUDA-graph decode engine over the paged cache (drop-in for the reference's LFM25CUDADecoder).

Reference: src/climbing_gym/inference/lfm25_cuda.py. Same role and attribute contract
(``generate``, ``graphs`` keyed ``(batch, capacity, masked)``, ``_get_graph``, ``refresh_weights``,
``clear``, ``_active_session`` ...), different machinery: one captured graph per entry holds the
WHOLE step - page allocation for rows that cross a page boundary, the 16-layer forward, the LM
head, the fused sampler and the per-slot bookkeeping - so a decode step is one graph replay with
no host logic between tokens. Rows are the physical slots of a paged cache; finished or empty
rows are masked inside the kernels instead of being compacted on the host.
"""
from __future__ import annotations

import contextlib
import ctypes as C
import gc
from collections import OrderedDict
from dataclasses import dataclass, field

import torch

from . import _native as nv
from .config import LFM25SamplingConfig
from .model import ForwardBuffers, LFM25Runner
from .paged import PagedHybridCache
from .text_stops import build_token_sequence_table, product_stop_table
from .types import LFM25GenerationOutput


@contextlib.contextmanager
def _quiet_collector():
    """Stream capture must not see the cyclic garbage collector at work: a decode graph that was evicted from
    the cache (or belonged to an engine that is gone) and is only kept alive by a reference cycle would be
    destroyed whenever the collector happens to run, and destroying a CUDA graph while another one is being
    captured is an operation the capture does not permit (it is invalidated: "operation not permitted when
    stream is capturing"). Collect what is garbage now, outside the capture, and hold the collector until it ends."""
    gc.collect()
    enabled = gc.isenabled()
    gc.disable()
    try:
        yield
    finally:
        if enabled:
            gc.enable()


class SlotState:
    """Per-slot request state on the device (the reference session's row tensors,
    src/climbing_gym/inference/lfm25_session.py:147-167) plus the struct the sampler kernel reads."""

    def __init__(self, n_slots: int, capacity: int, vocab: int, eos: int, seq_lens: torch.Tensor,
                 *, stop_states: int = 32):
        dev = seq_lens.device
        self.n_slots, self.capacity, self.vocab = n_slots, capacity, vocab

        def rows(dtype, value=0):
            return torch.full((n_slots,), value, device=dev, dtype=dtype)

        self.tokens = torch.zeros((n_slots, capacity), device=dev, dtype=torch.int64)
        self.logprobs = torch.zeros((n_slots, capacity), device=dev, dtype=torch.float32)
        self.lengths, self.limits = rows(torch.int32), rows(torch.int32)
        self.reasons = rows(torch.int8)
        self.alive, self.pending, self.ignore_eos = rows(torch.uint8), rows(torch.uint8), rows(torch.uint8)
        self.input_tokens = rows(torch.int64)
        self.stop_states, self.stop_offsets = rows(torch.int64), rows(torch.int64)
        self.rng_positions, self.seeds, self.rng_offsets = rows(torch.int64), rows(torch.int64), rows(torch.int64)
        self.temperatures = rows(torch.float32)
        self.force_eos_at = rows(torch.int32, -1)
        self.active = rows(torch.uint8)  # snapshot of `pending` taken at the start of each step
        # stop-table arena: table 0 is all zeros (no stops); more tables are appended in place
        self.stop_table = torch.zeros(stop_states * vocab, device=dev, dtype=torch.int32)
        self.stop_table_used = vocab
        self.seq_lens = seq_lens
        # sampler scratch: per-(row, slice) partial picks + one arrival counter per row, kept at zero
        self.sample_ws = torch.zeros(int(nv.load().cgym_sample_workspace_bytes(n_slots)) // 4, device=dev,
                                     dtype=torch.float32)
        # top-k / top-p per slot and the value thresholds cgym_filter_thresholds derives from them each step
        self.top_k, self.top_p = rows(torch.int32), rows(torch.float32, 1.0)
        self.min_logits = rows(torch.float32, float("-inf"))

        self.eos = eos
        self.queue = None  # device-resident admission queue (allocate_queue)
        self.noise = None  # [n_slots][vocab] fp32 Gumbel noise of the current step (allocate_noise)
        self._build_structs()
        self.head_k, self.head_ids, self.head_logprobs = 0, None, None
        self.penalties, self.seen, self.penalised = None, None, None

    def _build_structs(self) -> None:
        out_rows = self.queue["out_rows"] if self.queue is not None else None

        def struct(min_logits):
            return nv.SlotState(
                nv.ptr(self.tokens), nv.ptr(self.logprobs), nv.ptr(self.lengths), nv.ptr(self.limits),
                nv.ptr(self.reasons), nv.ptr(self.alive), nv.ptr(self.pending), nv.ptr(self.input_tokens),
                nv.ptr(self.stop_states), nv.ptr(self.stop_offsets), nv.ptr(self.stop_table), nv.ptr(self.ignore_eos),
                nv.ptr(self.rng_positions), nv.ptr(self.seeds), nv.ptr(self.temperatures), nv.ptr(self.rng_offsets),
                nv.ptr(self.force_eos_at), nv.ptr(self.seq_lens), nv.ptr(min_logits), nv.ptr(self.noise),
                nv.ptr(out_rows), self.capacity, self.eos)

        self.struct = struct(None)                      # full-support sampling
        self.struct_filtered = struct(self.min_logits)  # draws restricted to logits >= min_logits[slot]

    def allocate_noise(self) -> None:
        """Buffer for the step's Gumbel noise, drawn beside the layers (cgym_gumbel_noise)."""
        self.noise = torch.zeros((self.n_slots, self.vocab), device=self.lengths.device, dtype=torch.float32)
        self._build_structs()

    def allocate_queue(self, queue_capacity: int, result_capacity: int, n_rows: int, logits_dtype) -> None:
        """Device-resident admission queue and per-request result rows (cgym_admit_queue): parked prompts wait
        in ``queue_capacity`` entries, and a request's tokens / log-probs live in row ``request id %
        result_capacity`` of the arenas from its admission until the host has read them, whichever slot ran it."""
        dev, n = self.lengths.device, self.n_slots
        self.tokens = torch.zeros((result_capacity, self.capacity), device=dev, dtype=torch.int64)
        self.logprobs = torch.zeros((result_capacity, self.capacity), device=dev, dtype=torch.float32)

        def entries(dtype, value=0):
            return torch.full((queue_capacity,), value, device=dev, dtype=dtype)

        q = dict(rows=entries(torch.int32, -1), requests=entries(torch.int32, -1), limits=entries(torch.int32),
                 seeds=entries(torch.int64), temperatures=entries(torch.float32), ignore_eos=entries(torch.uint8),
                 stop_offsets=entries(torch.int64),
                 logits=torch.zeros((queue_capacity, self.vocab), device=dev, dtype=logits_dtype),
                 head=torch.zeros(1, device=dev, dtype=torch.int32), tail=torch.zeros(1, device=dev, dtype=torch.int32),
                 result_lengths=torch.zeros(result_capacity, device=dev, dtype=torch.int32),
                 result_reasons=torch.zeros(result_capacity, device=dev, dtype=torch.int8),
                 slot_requests=torch.full((n,), -1, device=dev, dtype=torch.int32),
                 out_rows=torch.zeros(n, device=dev, dtype=torch.int32),
                 adopt_rows=torch.full((n,), -1, device=dev, dtype=torch.int32),
                 adopt_entries=torch.full((n,), -1, device=dev, dtype=torch.int32),
                 release_mask=torch.zeros(n_rows, device=dev, dtype=torch.uint8))
        q["capacity"], q["result_capacity"] = queue_capacity, result_capacity
        self.queue = q
        self.queue_struct = nv.AdmitQueue(
            nv.ptr(q["rows"]), nv.ptr(q["requests"]), nv.ptr(q["limits"]), nv.ptr(q["seeds"]), nv.ptr(q["temperatures"]),
            nv.ptr(q["ignore_eos"]), nv.ptr(q["stop_offsets"]), nv.ptr(q["logits"]), nv.ptr(q["head"]), nv.ptr(q["tail"]),
            queue_capacity, result_capacity, nv.ptr(q["result_lengths"]), nv.ptr(q["result_reasons"]),
            nv.ptr(q["slot_requests"]), nv.ptr(q["out_rows"]), nv.ptr(q["adopt_rows"]), nv.ptr(q["adopt_entries"]),
            nv.ptr(q["release_mask"]))
        self._build_structs()

    def allocate_penalty(self) -> None:
        """Repetition-penalty buffers: per-slot factor, one seen byte per (slot, token) and the penalised
        fp32 copy of the step's logits that the sampler reads (cgym_repetition_penalty)."""
        dev = self.lengths.device
        self.penalties = torch.ones(self.n_slots, device=dev, dtype=torch.float32)
        self.seen = torch.zeros((self.n_slots, self.vocab), device=dev, dtype=torch.uint8)
        self.penalised = torch.zeros((self.n_slots, self.vocab), device=dev, dtype=torch.float32)

    def allocate_heads(self, k: int, positions: int) -> None:
        """Behaviour head buffers [slots][positions][k] (ids int32, log-probs fp32), filled by cgym_topk_head;
        ``positions`` bounds the tokens one request generates, not its context."""
        dev = self.lengths.device
        self.head_k, self.head_positions = k, positions
        self.head_ids = torch.zeros((self.n_slots, positions, k), device=dev, dtype=torch.int32)
        self.head_logprobs = torch.zeros((self.n_slots, positions, k), device=dev, dtype=torch.float32)

    def reset(self) -> None:
        for t in (self.lengths, self.limits, self.reasons, self.alive, self.pending, self.ignore_eos,
                  self.input_tokens, self.stop_states, self.stop_offsets, self.rng_positions, self.seeds,
                  self.rng_offsets, self.temperatures, self.active, self.tokens, self.logprobs):
            t.zero_()
        self.force_eos_at.fill_(-1)
        self.stop_table_used = self.vocab
        if self.queue is not None:
            for name in ("head", "tail", "result_lengths", "result_reasons", "out_rows", "release_mask"):
                self.queue[name].zero_()
            for name in ("rows", "requests", "slot_requests", "adopt_rows", "adopt_entries"):
                self.queue[name].fill_(-1)
        if self.head_k:
            self.head_ids.zero_()
            self.head_logprobs.zero_()
        if self.penalties is not None:
            self.penalties.fill_(1.0)
            self.seen.zero_()

    def add_stop_table(self, table: torch.Tensor) -> int:
        """Append a [states, vocab] int32 table to the arena; returns its element offset."""
        flat = table.reshape(-1).to(device=self.stop_table.device, dtype=torch.int32)
        offset = self.stop_table_used
        if offset + flat.numel() > self.stop_table.numel():
            states = self.stop_table.numel() // self.vocab
            raise ValueError(f"stop tables exceed the reserved stop-state arena ({states} states, one per proper prefix "
                             "of every stop string): raise enable_cuda_graphs(stop_states=...)")
        self.stop_table[offset:offset + flat.numel()].copy_(flat)
        self.stop_table_used = offset + flat.numel()
        return offset

    def configure(self, slots, *, limits, seeds, temperatures, ignore_eos, stop_offsets, rng_offsets,
                  rng_positions=None, stop_states=None, force_eos_at=None) -> None:
        """Arm rows for a new request: one small scatter per field, no per-slot host writes."""
        dev = self.lengths.device
        index = torch.as_tensor(slots, dtype=torch.int64, device=dev)
        n = index.numel()

        def put(dst, values, dtype):
            if isinstance(values, (list, tuple)):
                src = torch.tensor(values, dtype=dtype, device=dev)
            else:
                src = torch.full((n,), values, dtype=dtype, device=dev)
            dst.index_copy_(0, index, src)

        put(self.lengths, 0, torch.int32)
        put(self.reasons, 0, torch.int8)
        put(self.limits, limits, torch.int32)
        put(self.seeds, seeds, torch.int64)
        put(self.temperatures, temperatures, torch.float32)
        put(self.ignore_eos, ignore_eos, torch.uint8)
        put(self.stop_offsets, stop_offsets, torch.int64)
        put(self.rng_offsets, rng_offsets, torch.int64)
        put(self.rng_positions, 0 if rng_positions is None else rng_positions, torch.int64)
        put(self.stop_states, 0 if stop_states is None else stop_states, torch.int64)
        put(self.force_eos_at, -1 if force_eos_at is None else force_eos_at, torch.int32)
        put(self.alive, 1, torch.uint8)
        put(self.pending, 0, torch.uint8)


@dataclass
class _DecodeGraph:
    cache: PagedHybridCache
    input_tokens: torch.Tensor
    logits: torch.Tensor
    graph: object
    active: torch.Tensor
    state: SlotState
    bufs: ForwardBuffers
    compact_graphs: dict = field(default_factory=dict)
    filtered: bool = False  # the step derives top-k / top-p thresholds before it samples


@dataclass
class _CompactGraph:
    """A captured step over ``slots.numel()`` rows that stand for an arbitrary subset of a session's slots
    (the reference's CompactDecodeGraph, src/climbing_gym/inference/lfm25_batching.py:73-120). The rows
    reach the shared paged cache, conv taps and request state through ``slots``; nothing is copied."""

    graph: object
    slots: torch.Tensor          # int32 [rows], -1 = padding row
    buffers: tuple               # row-indexed inputs the graph reads (kept alive with it)
    mapped_slots: tuple = ()

    def set_slots(self, slots) -> None:
        mapping = tuple(slots)
        if mapping != self.mapped_slots:
            values = mapping + (-1,) * (self.slots.numel() - len(mapping))
            self.slots.copy_(torch.tensor(values, dtype=torch.int32), non_blocking=False)
            self.mapped_slots = mapping


class B200Decoder:
    supported_conv_kernel_sizes = (3,)

    def __init__(self, engine, *, max_graphs: int = 2, bf16_weight_packing: bool = True,
                 max_prefill_tokens: int = 4096, finish_check_interval: int = 32,
                 skip_finished_attention: bool = True, fp8_mlp: bool = False, fp8_kv: bool = False,
                 adaptive_batching: bool = False, fp8_lm_head: bool = False, page_size: int = 64,
                 snapshot_rows: int = 32, snapshot_pages: int | None = None, stop_states: int = 256):
        if engine.device.type != "cuda" or engine.dtype not in (torch.bfloat16, torch.float32):
            raise ValueError("LFM2.5 CUDA graphs require CUDA and bfloat16 (or float32) weights")
        cfg = engine.config
        if cfg.conv_kernel_size not in self.supported_conv_kernel_sizes or cfg.conv_bias:
            raise ValueError(f"Native CUDA graphs require bias-free convolutions of width {self.supported_conv_kernel_sizes}")
        if cfg.head_dim not in (32, 64, 128, 256):
            raise ValueError("LFM2.5 CUDA graphs require head_dim in {32, 64, 128, 256}")
        if max_graphs <= 0:
            raise ValueError("max_graphs must be > 0")
        if max_prefill_tokens <= 0:
            raise ValueError("max_prefill_tokens must be positive")
        if type(finish_check_interval) is not int or finish_check_interval <= 0:
            raise ValueError("finish_check_interval must be a positive integer")
        if (fp8_mlp or fp8_kv or fp8_lm_head) and engine.dtype != torch.bfloat16:
            raise ValueError("Native FP8 paths require bfloat16 weights")
        if not nv.load().cgym_device_supported():
            raise ValueError("The cgym_b200 kernels require an NVIDIA B200 (compute capability 10.x)")
        self.engine = engine
        self.max_graphs = max_graphs
        self.max_prefill_tokens = max_prefill_tokens
        self.finish_check_interval = finish_check_interval
        # Accepted for the reference's constructor contract and always in force here: a finished row is inactive
        # in every kernel of the step (no KV append, no attention over its history), which is what the
        # reference's flag switches on by zeroing the row's length (src/climbing_gym/inference/lfm25_cuda.py:361-365).
        self.skip_finished_attention = bool(skip_finished_attention)
        self.bf16_weight_packing = bool(bf16_weight_packing) and engine.dtype == torch.bfloat16
        self.fp8_mlp, self.fp8_kv = bool(fp8_mlp), bool(fp8_kv)
        self.adaptive_batching, self.fp8_lm_head = bool(adaptive_batching), bool(fp8_lm_head)
        self.page_size = page_size
        if snapshot_rows < 0 or (snapshot_pages is not None and snapshot_pages < 0):
            raise ValueError("snapshot_rows and snapshot_pages must be >= 0")
        # session caches park prefix snapshots in spare rows of the paged cache; the page reserve defaults to
        # eight full-length prefixes plus one private tail page per snapshot
        self.snapshot_rows, self.snapshot_pages = int(snapshot_rows), snapshot_pages
        # Stop tables live in one device arena of `stop_states` x vocab int32 entries per graph entry (state 0
        # is the shared "no stops" table): one state per proper prefix of every stop string in use. 256 states
        # cost 64 MB at a 65,536-token vocabulary. The reference concatenates tables without a limit
        # (src/climbing_gym/inference/lfm25_session.py:228-241); here the arena is fixed because the captured
        # graph holds its address, so its size is an option and tables no slot refers to are recycled.
        if type(stop_states) is not int or stop_states < 2:
            raise ValueError("stop_states must be an integer >= 2")
        self.stop_states = stop_states
        # the step's kernels are chained with programmatic dependent launches while a graph is captured
        self.use_pdl = True
        self.runner = LFM25Runner(engine.weights, engine._rope_cos, engine._rope_sin, fp8_mlp=self.fp8_mlp,
                                  fp8_lm_head=self.fp8_lm_head)
        self.graphs: OrderedDict = OrderedDict()
        self._active_session = None
        # the step's own kernels go first wherever both streams have work ready
        self._capture_stream = torch.cuda.Stream(device=engine.device, priority=-1)
        self._noise_stream = torch.cuda.Stream(device=engine.device)
        self.debug_force_eos_at = None  # test hook: per-row generated position forced to EOS
        # when set, generate() brackets its decode-graph replays with CUDA events on the launching
        # stream and appends (start, end, replays) here; resolved by the caller after a synchronize
        self.profile_decode = False
        self.decode_profile: list = []

    @property
    def fp8_weights(self) -> dict:
        return self.runner.fp8_weights

    @property
    def packed_weights(self) -> dict:
        """Lossless 12-bit bf16 streams of the matrices a single-request step reads (PackedBF16Weight)."""
        return self.runner.packed_weights

    def _prepare_weights(self) -> None:
        """Encoded copies of the vocabulary head and the MLP matrices for batch-1 graphs (reference:
        src/climbing_gym/inference/lfm25_cuda.py:108-122): they dominate single-request decode traffic."""
        if not self.bf16_weight_packing or self.runner.packed_weights:
            return
        from .weights import PackedBF16Weight

        weights = self.engine.weights
        matrices = [] if self.fp8_lm_head else [weights.lm_head_weight]
        if not self.fp8_mlp:
            for layer in weights.layers:
                matrices.extend((layer.w13_weight, layer.w2_weight))
        self.runner.packed_weights = {id(w): PackedBF16Weight.from_weight(w) for w in matrices
                                      if w.size(1) % 2 == 0 and w.size(1) <= 16384}

    def clear(self) -> None:
        if self._active_session is not None:
            self._active_session.close()
        self.graphs.clear()
        self.runner.packed_weights.clear()
        self.runner.fp8_weights.clear()

    def refresh_weights(self) -> None:
        for packed in self.runner.packed_weights.values():
            packed.refresh()
        self.runner.refresh_fp8()

    # ---- graph entries ------------------------------------------------------------------------------
    def _step(self, entry: _DecodeGraph) -> None:
        """The whole decode step for every slot of the entry (what the graph captures)."""
        cache, state = entry.cache, entry.state
        n = cache.n_slots
        stream = nv.stream_ptr(self.engine.device)
        kv_lens = self.runner.kv_lens_buffer(cache)
        if state.queue is not None:
            self._turnover(entry)
        nv.call("cgym_step_begin", cache.pool, nv.ptr(cache.seq_lens), nv.ptr(state.pending), nv.ptr(state.active),
                None, None, nv.ptr(kv_lens), n, nv.ptr(cache.status), stream)
        self._launch_noise(entry)
        self.runner.decode_step(entry.bufs, cache, state.input_tokens, state.active, entry.logits, kv_lens=kv_lens)
        self._join_noise(entry)
        self._sample(entry, nv.ptr(state.active), stream)

    def _launch_noise(self, entry: _DecodeGraph) -> None:
        """The step's Gumbel noise depends on the slot state alone (seed, position, temperature), not on the
        logits: draw it now on a side stream, beside the layers, and let the sampler subtract it. The ten
        Philox rounds per logit otherwise sit on the critical path after the LM head (0.1 ms at 256 rows)."""
        state = entry.state
        if state.noise is None:
            return
        main = torch.cuda.current_stream(self.engine.device)
        self._noise_stream.wait_stream(main)
        with torch.cuda.stream(self._noise_stream):
            nv.call("cgym_gumbel_noise", nv.ptr(state.noise), C.byref(state.struct), state.n_slots, state.vocab,
                    nv.stream_ptr(self.engine.device))

    def _join_noise(self, entry: _DecodeGraph) -> None:
        if entry.state.noise is not None:
            torch.cuda.current_stream(self.engine.device).wait_stream(self._noise_stream)

    def _turnover(self, entry: _DecodeGraph) -> None:
        """Evict finished requests and admit parked ones, on the device (cgym_slot_turnover)."""
        cache, state, cfg = entry.cache, entry.state, self.engine.config
        nv.call("cgym_slot_turnover", cache.pool_rows, cache.n_slots, C.byref(state.struct), C.byref(state.queue_struct),
                nv.ptr(entry.logits), nv.ptr(cache.conv_state), nv.ptr(cache.row_lens), cache.n_conv_layers,
                cfg.hidden_size, cfg.vocab_size, nv.dtype_code(entry.logits.dtype), nv.stream_ptr(self.engine.device))

    def _sample(self, entry: _DecodeGraph, advance, stream) -> None:
        """Sampler + bookkeeping of one step; filtered entries first turn each row's top-k / top-p into
        a value threshold (the reference leaves its fused sampler for torch sort / multinomial here,
        src/climbing_gym/inference/lfm25_cuda.py:311-324)."""
        state, n, vocab = entry.state, entry.cache.n_slots, self.engine.config.vocab_size
        logits, dtype = entry.logits, nv.dtype_code(entry.logits.dtype)
        if state.head_k:  # behaviour head of the unfiltered distribution, recorded at the row's current length
            nv.call("cgym_topk_head", nv.ptr(state.head_ids), nv.ptr(state.head_logprobs), nv.ptr(logits),
                    nv.ptr(state.alive), nv.ptr(state.lengths), n, vocab, state.head_positions, state.head_k, dtype, stream)
        if state.penalties is not None:  # everything after this reads the penalised fp32 copy of the logits
            nv.call("cgym_repetition_penalty", nv.ptr(state.penalised), nv.ptr(logits), nv.ptr(state.seen),
                    nv.ptr(state.tokens), nv.ptr(state.lengths), nv.ptr(state.alive), nv.ptr(state.penalties), n, vocab,
                    state.capacity, dtype, stream)
            logits, dtype = state.penalised, nv.F32
        if entry.filtered:
            nv.call("cgym_filter_thresholds", nv.ptr(state.min_logits), nv.ptr(logits), nv.ptr(state.temperatures),
                    nv.ptr(state.top_k), nv.ptr(state.top_p), nv.ptr(state.alive), n, vocab, dtype, stream)
        struct = state.struct_filtered if entry.filtered else state.struct
        nv.call("cgym_sample_record", nv.ptr(logits), C.byref(struct), advance, None, None, n, vocab, dtype,
                nv.ptr(state.sample_ws), stream)

    def _sample_only(self, entry: _DecodeGraph) -> None:
        """First token of freshly prefetched rows: sample from the prefill logits, no forward."""
        self._launch_noise(entry)
        self._join_noise(entry)
        self._sample(entry, None, nv.stream_ptr(self.engine.device))

    @torch.inference_mode()
    def _get_graph(self, batch_size: int, cache_len: int, *, masked: bool = False, filtered: bool = False,
                   head_k: int = 0, head_positions: int = 0, penalised: bool = False,
                   queue_capacity: int = 0) -> _DecodeGraph:
        engine = self.engine
        alignment = 32 if batch_size >= 64 else 128
        alignment = max(alignment, self.page_size)
        capacity = min(engine.max_model_len, -(-cache_len // alignment) * alignment)
        head_positions = min(capacity, -(-head_positions // 64) * 64) if head_k else 0
        key = (batch_size, capacity, masked) + (("filtered",) if filtered else ())
        key += (f"head{head_k}x{head_positions}",) if head_k else ()
        key += ("penalised",) if penalised else ()
        key += (f"queue{queue_capacity}",) if queue_capacity else ()
        if key in self.graphs:
            self.graphs.move_to_end(key)
            return self.graphs[key]
        if len(self.graphs) >= self.max_graphs:
            self.graphs.popitem(last=False)
        self.runner.prepare_fp8()
        if batch_size == 1:
            self._prepare_weights()
        elif not any(existing[0] == 1 for existing in self.graphs):
            self.runner.packed_weights.clear()  # no surviving graph uses the single-request copies
        spare, n_pages = (self.snapshot_rows if masked else 0), None
        spare += queue_capacity  # one parked row per queue entry
        if spare:
            blocks = -(-capacity // self.page_size)
            reserve = self.snapshot_pages if self.snapshot_pages is not None else 8 * blocks + spare
            # parked prompts hold pages of their own until a slot adopts them
            n_pages = batch_size * blocks + reserve + queue_capacity * blocks
        cache = engine._empty_cache(max_slots=batch_size, max_seq_len=capacity, fp8_kv=self.fp8_kv,
                                    page_size=self.page_size, n_pages=n_pages, spare_rows=spare)
        state = SlotState(batch_size, capacity, engine.config.vocab_size, int(engine.config.eos_token_id), cache.seq_lens,
                          stop_states=self.stop_states)
        if head_k:
            state.allocate_heads(head_k, head_positions)
        if penalised:
            state.allocate_penalty()
        if engine.config.vocab_size >= 4096:  # smaller vocabularies: the sampler draws the noise itself
            state.allocate_noise()
        if queue_capacity:
            # results stay addressable until the host has read them: room for every request that can be
            # parked or running at once, twice over (finished requests wait for the next poll)
            state.allocate_queue(queue_capacity, 2 * (batch_size + queue_capacity), cache.n_rows, engine.dtype)
        logits = torch.zeros((batch_size, engine.config.vocab_size), device=engine.device, dtype=engine.dtype)
        bufs = self._forward_buffers(batch_size)
        entry = _DecodeGraph(cache, state.input_tokens, logits, None, state.active, state, bufs, filtered=filtered)
        # All rows are dead (alive = pending = 0) while warming up and capturing, so neither run
        # touches KV pages, conv taps, logits or bookkeeping.
        stream, current = self._capture_stream, torch.cuda.current_stream(engine.device)
        stream.wait_stream(current)
        lib = nv.load()
        # the step's kernels are chained with programmatic dependent launches (see cgym_set_pdl)
        previous_pdl = lib.cgym_set_pdl(1 if self.use_pdl else 0)
        try:
            with torch.cuda.stream(stream):
                for _ in range(2):
                    self._step(entry)
            current.wait_stream(stream)
            torch.cuda.synchronize(engine.device)
            graph = torch.cuda.CUDAGraph()
            before = lib.cgym_launch_count()
            with _quiet_collector(), torch.cuda.graph(graph, stream=stream):
                self._step(entry)
            current.wait_stream(stream)
            entry.graph = _StepGraph(graph, int(lib.cgym_launch_count() - before))
        finally:
            lib.cgym_set_pdl(previous_pdl)
        self.graphs[key] = entry
        return entry

    def _forward_buffers(self, rows: int) -> ForwardBuffers:
        """Activation scratch of a step over ``rows`` rows; decode attention is split along the context
        when rows x kv_heads alone would leave SMs idle."""
        heads = self.engine.config.num_key_value_heads
        splits = min(16, max(1, -(-148 // (rows * heads)))) if rows * heads < 148 else 1
        return ForwardBuffers(self.engine.weights, rows, fp8=self.fp8_mlp or self.fp8_lm_head, attn_splits=splits)

    def _select_graph(self, entry, live_slots):
        """The graph to replay for the live rows and its compute batch. With adaptive batching, the
        smallest bucket 16 * 2^k that holds them (the reference's rule,
        src/climbing_gym/inference/lfm25_cuda.py:194-209); every variant works on the same physical cache."""
        maximum = entry.input_tokens.numel()
        if not self.adaptive_batching or maximum <= 16:
            return entry.graph, maximum
        size = 16
        while size < len(live_slots):
            size *= 2
        if size >= maximum:
            return entry.graph, maximum
        if size not in entry.compact_graphs:
            entry.compact_graphs[size] = self._capture_compact(entry, size)
        compact = entry.compact_graphs[size]
        compact.set_slots(live_slots)
        return compact.graph, size

    def _compact_step(self, entry: _DecodeGraph, rows: int, slots, tokens, positions, active, kv_lens, bufs,
                      *, sample: bool) -> None:
        cache, state = entry.cache, entry.state
        stream = nv.stream_ptr(self.engine.device)
        nv.call("cgym_step_begin_rows", cache.pool, nv.ptr(cache.seq_lens), nv.ptr(state.pending),
                nv.ptr(state.input_tokens), nv.ptr(slots), nv.ptr(active), nv.ptr(state.active), nv.ptr(tokens),
                nv.ptr(positions), nv.ptr(kv_lens), rows, cache.n_slots, nv.ptr(cache.status), stream)
        if sample:
            self._launch_noise(entry)
        self.runner.decode_step(bufs, cache, tokens, active, entry.logits, slots=slots, rows=rows, kv_lens=kv_lens,
                                positions=positions, logits_rows=slots)
        if sample:
            self._join_noise(entry)
            self._sample(entry, nv.ptr(state.active), stream)

    @torch.inference_mode()
    def _capture_compact(self, entry: _DecodeGraph, rows: int) -> _CompactGraph:
        """Capture a step over ``rows`` compacted rows without disturbing resident requests: while
        warming up and capturing every row is a padding row (slot -1), so no KV page, conv tap or logits
        row is written, and the warm-up leaves the sampler out (its bookkeeping would advance live rows)."""
        engine, dev = self.engine, self.engine.device
        slots = torch.full((rows,), -1, device=dev, dtype=torch.int32)
        tokens = torch.zeros(rows, device=dev, dtype=torch.int64)
        positions = torch.zeros(rows, device=dev, dtype=torch.int32)
        active = torch.zeros(rows, device=dev, dtype=torch.uint8)
        kv_lens = torch.zeros(rows, device=dev, dtype=torch.int32)
        bufs = self._forward_buffers(rows)
        stream, current = self._capture_stream, torch.cuda.current_stream(dev)
        stream.wait_stream(current)
        lib = nv.load()
        previous_pdl = lib.cgym_set_pdl(1 if self.use_pdl else 0)
        try:
            with torch.cuda.stream(stream):
                for _ in range(2):
                    self._compact_step(entry, rows, slots, tokens, positions, active, kv_lens, bufs, sample=False)
            current.wait_stream(stream)
            torch.cuda.synchronize(dev)
            graph = torch.cuda.CUDAGraph()
            before = lib.cgym_launch_count()
            with _quiet_collector(), torch.cuda.graph(graph, stream=stream):
                self._compact_step(entry, rows, slots, tokens, positions, active, kv_lens, bufs, sample=True)
            current.wait_stream(stream)
            step = _StepGraph(graph, int(lib.cgym_launch_count() - before))
        finally:
            lib.cgym_set_pdl(previous_pdl)
        return _CompactGraph(step, slots, (tokens, positions, active, kv_lens, bufs))

    # ---- batch generate -------------------------------------------------------------------------------
    @torch.inference_mode()
    def generate(self, input_ids, cu_seqlens, max_seqlen: int, repeats: int, sampling: LFM25SamplingConfig):
        if self._active_session is not None:
            raise RuntimeError("Close the native generation session before calling generate")
        if repeats <= 0:
            raise ValueError("repeats must be > 0")
        engine = self.engine
        cache_len = int(max_seqlen) + sampling.max_new_tokens
        if cache_len > engine.max_model_len:
            raise ValueError(f"max_seq_len={cache_len} exceeds engine max_model_len={engine.max_model_len}")
        penalised = float(sampling.repetition_penalty) != 1.0
        filtered = sampling.temperature > 0.0 and (0 < sampling.top_k < engine.config.vocab_size or sampling.top_p < 1.0)
        head_k = sampling.behavior_topk
        if head_k > engine.config.vocab_size:
            raise ValueError("Behavior head exceeds the vocabulary")
        flat_ids, prompt_lengths = engine._split_lengths(input_ids, cu_seqlens, max_seqlen)
        n_prompts, batch = len(prompt_lengths), len(prompt_lengths) * repeats
        entry = self._get_graph(batch, cache_len, masked=self.adaptive_batching, filtered=filtered, head_k=head_k,
                                head_positions=sampling.max_new_tokens, penalised=penalised)
        cache, state, dev = entry.cache, entry.state, engine.device
        cache.release(torch.ones(batch, device=dev, dtype=torch.uint8))
        cache.conv_state.zero_()
        state.reset()
        sources = [p * repeats for p in range(n_prompts)]
        engine._prefill_packed(cache, sources, prompt_lengths, [0] * n_prompts, entry.logits, self.max_prefill_tokens,
                               flat_tokens=flat_ids)
        if repeats > 1:
            src = torch.tensor([p * repeats for p in range(n_prompts) for _ in range(repeats - 1)], device=dev, dtype=torch.int32)
            dst = torch.tensor([p * repeats + r for p in range(n_prompts) for r in range(1, repeats)], device=dev, dtype=torch.int32)
            lens = torch.tensor([prompt_lengths[p] for p in range(n_prompts) for _ in range(repeats - 1)], device=dev, dtype=torch.int32)
            cache.fork(src, dst, lens)
            entry.logits[dst.long()] = entry.logits[src.long()]
        stop_offset = 0
        if sampling.stop_table is not None or sampling.stop_token_ids or sampling.stop_token_sequences:
            stop_offset = state.add_stop_table(build_token_stop_table(sampling, engine.config.vocab_size, dev))
        vocab = engine.config.vocab_size
        state.configure(list(range(batch)), limits=sampling.max_new_tokens, seeds=int(sampling.seed) & 0x7FFFFFFFFFFFFFFF,
                        temperatures=float(sampling.temperature), ignore_eos=int(sampling.ignore_eos),
                        stop_offsets=stop_offset, rng_offsets=[row * vocab for row in range(batch)],
                        force_eos_at=self.debug_force_eos_at)
        if filtered:
            state.top_k.fill_(int(sampling.top_k))
            state.top_p.fill_(float(sampling.top_p))
        if penalised:
            # every sample of a prompt starts out having seen the prompt's tokens
            # (reference: src/climbing_gym/inference/lfm25_engine.py:933-958)
            state.penalties.fill_(float(sampling.repetition_penalty))
            first_rows = torch.arange(n_prompts, device=dev) * repeats
            token_rows = torch.repeat_interleave(first_rows, torch.tensor(prompt_lengths, device=dev))
            state.seen.index_put_((token_rows, flat_ids), torch.ones((), device=dev, dtype=torch.uint8))
            if repeats > 1:
                state.seen[dst.long()] = state.seen[src.long()]
        fixed_length = (sampling.ignore_eos and not sampling.stop_token_ids and not sampling.stop_token_sequences
                        and sampling.stop_table is None)
        interval = self.finish_check_interval if batch >= 16 else 1
        self._sample_only(entry)
        timing = self.profile_decode
        if timing:
            start_event, end_event = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            start_event.record()
        replays = 0
        graph = entry.graph
        for step in range(1, sampling.max_new_tokens):
            if not fixed_length and step % interval == 0:
                if self.adaptive_batching:
                    # rows that finished leave the compute batch: the live ones are compacted into the
                    # smallest graph bucket that holds them (src/climbing_gym/inference/lfm25_cuda.py:350-357)
                    live = torch.nonzero(state.alive).flatten().cpu().tolist()
                    if not live:
                        break
                    graph, _ = self._select_graph(entry, live)
                elif not bool(state.alive.any().item()):
                    break
            graph.replay()
            replays += 1
        if timing:
            end_event.record()
            self.decode_profile.append((start_event, end_event, replays))
        cache.check_status()
        n_new = sampling.max_new_tokens
        shape = (n_prompts, repeats)
        reasons = state.reasons.clone()
        reasons.masked_fill_(reasons == 0, 3)
        return LFM25GenerationOutput(
            token_ids=state.tokens[:, :n_new].reshape(*shape, n_new).clone(),
            lengths=state.lengths.reshape(shape).clone(),
            logprobs=state.logprobs[:, :n_new].reshape(*shape, n_new).clone() if sampling.return_logprobs else None,
            finish_reasons=reasons.reshape(shape),
            topk_token_ids=state.head_ids[:, :n_new].reshape(*shape, n_new, head_k).clone() if head_k else None,
            topk_logprobs=state.head_logprobs[:, :n_new].reshape(*shape, n_new, head_k).clone() if head_k else None)


class _StepGraph:
    """A captured step plus the number of this library's kernels inside it (for launch accounting)."""

    def __init__(self, graph, kernels: int):
        self.graph, self.kernels = graph, kernels

    def replay(self) -> None:
        self.graph.replay()
        nv.note_graph_replay(self.kernels)


def build_token_stop_table(sampling: LFM25SamplingConfig, vocab: int, device) -> torch.Tensor:
    """Stop ids folded into a (copy of the) stop table as ``matched`` entries, as the reference
    session does (src/climbing_gym/inference/lfm25_session.py:228-241)."""
    if sampling.stop_table is not None:
        table = sampling.stop_table.to(device).clone()
        if sampling.stop_token_sequences:  # both kinds of stop: their product automaton
            table = product_stop_table(table, build_token_sequence_table(sampling.stop_token_sequences, vocab))
    elif sampling.stop_token_sequences:  # suffix match on the generated ids, as an automaton over token ids
        table = build_token_sequence_table(sampling.stop_token_sequences, vocab).to(device)
    else:
        table = torch.zeros((1, vocab), dtype=torch.int32, device=device)
    if sampling.stop_token_ids:
        table[:, list(sampling.stop_token_ids)] = 65536
    return table
