"""Resumable fixed-slot generation with continuous request admission.

API, result types, validation messages and statistics keys follow the reference session
(src/climbing_gym/inference/lfm25_session.py:59-533): ``admit`` takes the lowest free slots,
``poll(steps)`` advances every live row at most ``steps`` tokens and returns the rows that
finished, ``resume`` continues a finished row from its exact cached prefix (its last sampled
token is still "pending", i.e. not yet in the cache), ``release`` frees the slot.

What differs underneath:
* a poll step is one replay of the decoder's step graph - page allocation, forward, LM head,
  sampler and bookkeeping all run on the device; the host touches nothing per token;
* ``release`` returns the slot's pages to the device-side pool (eviction), ``admit`` prefetches
  packed variable-length prompt rows straight into freshly reserved pages;
* ``resume`` feeds the pending token plus the new suffix through one packed prefill chunk that
  continues from the cached prefix, instead of one decode-graph replay per token.
"""
from __future__ import annotations

from contextlib import contextmanager
from dataclasses import dataclass
from typing import Sequence

import torch

from .config import LFM25SamplingConfig
from .decoder import build_token_stop_table
from .types import BehaviorTopK


@dataclass(frozen=True, slots=True)
class LFM25ContinuationHandle:
    """A single-use lease on one session slot; invalid after release/close."""

    session: object
    slot: int
    version: int
    prefix_token_ids: tuple


@dataclass(frozen=True, slots=True)
class LFM25SessionResult:
    handle: LFM25ContinuationHandle | None  # None: the request ran through the device-side queue (no continuation)
    prompt_token_ids: tuple
    token_ids: tuple
    logprobs: tuple | None
    finish_reason: int
    behavior_topk: BehaviorTopK | None = None
    request_id: int | None = None  # set for requests submitted with ``enqueue``


@dataclass(frozen=True, slots=True)
class LFM25PrefixSnapshot:
    """Opaque immutable lease on a cached prefix; its pages belong to the creating session."""

    session: object
    identity: int
    policy_version: int
    prefix_token_ids: tuple


@dataclass
class _SnapshotState:
    lease: LFM25PrefixSnapshot
    row: int                 # spare row of the session's paged cache that holds the prefix
    length: int              # cached tokens (= len(prefix_token_ids))
    logits: torch.Tensor     # [1, vocab] next-token logits after the prefix
    seed: int
    rng_position: int
    stop_state: int


@dataclass
class _Request:
    prompt: tuple
    sampling: LFM25SamplingConfig
    version: int
    delivered: bool = False
    handle: LFM25ContinuationHandle | None = None


class LFM25GenerationSession:
    @torch.inference_mode()
    def __init__(self, decoder, *, max_batch_size: int, max_new_tokens: int, cache_len: int | None = None,
                 behavior_topk: int = 0, profile_timings: bool = False, queue_capacity: int = 0):
        if decoder._active_session is not None:
            raise RuntimeError("A native generation session is already open")
        if type(max_batch_size) is not int or max_batch_size <= 0:
            raise ValueError("max_batch_size must be a positive integer")
        if type(max_new_tokens) is not int or max_new_tokens <= 0:
            raise ValueError("max_new_tokens must be a positive integer")
        self.decoder, self.engine = decoder, decoder.engine
        self.batch_size, self.max_new_tokens = max_batch_size, max_new_tokens
        if type(behavior_topk) is not int or not 0 <= behavior_topk <= min(128, self.engine.config.vocab_size):
            raise ValueError("behavior_topk must be an integer between 0 and min(vocab, 128)")
        self.behavior_topk = behavior_topk
        if type(queue_capacity) is not int or queue_capacity < 0:
            raise ValueError("queue_capacity must be a non-negative integer")
        if queue_capacity and behavior_topk:
            raise ValueError("Behavior heads are not recorded for requests of the device-side queue")
        self.queue_capacity = queue_capacity
        self.entry = decoder._get_graph(max_batch_size, cache_len or self.engine.max_model_len, masked=True,
                                        head_k=behavior_topk, head_positions=max_new_tokens,
                                        queue_capacity=queue_capacity)
        self.state, self.cache = self.entry.state, self.entry.cache
        self.cache.release_rows(torch.ones(self.cache.n_rows, device=self.engine.device, dtype=torch.uint8))
        self.cache.conv_state.zero_()
        self.state.reset()
        self._snapshots: dict[int, _SnapshotState] = {}
        self._next_snapshot = 0
        self._free_rows = list(range(self.cache.n_slots, self.cache.n_rows))
        # device-side queue mode (enqueue / poll): request id -> (prompt, sampling, parked row), ids in order
        self._queued: dict[int, tuple] = {}
        self._next_request_id = 0
        self._queue_tail = self._queue_consumed = 0
        self._poll_pending = None  # (event after the reads of poll_begin, whether steps were launched)
        self._read_stream = None   # device-to-host reads of a poll (queue mode), created on first use
        self.last_context = (0.0, 0.0)
        self.requests: list[_Request | None] = [None] * max_batch_size
        self.versions = [0] * max_batch_size
        self.closed = False
        self.policy_version = self.engine.policy_version
        self._timing_events = []
        self.profile_timings = profile_timings
        self._stop_tables: dict = {}
        self.stats = dict(prefilled_tokens=0, resumed_prefix_tokens=0, appended_tokens=0, admitted_requests=0,
                          resumed_requests=0, decode_steps=0, slot_refills=0, peak_live_slots=0, decode_row_steps=0,
                          reserved_row_steps=0, adaptive_graph_captures=0, decode_batches={}, forked_requests=0,
                          copied_prefix_tokens=0, snapshot_prefilled_tokens=0, snapshot_count=0, peak_snapshots=0,
                          peak_snapshot_bytes=0)
        decoder._active_session = self

    # views the reference's tests and examples read
    @property
    def lengths(self): return self.state.lengths
    @property
    def reasons(self): return self.state.reasons
    @property
    def alive(self): return self.state.alive
    @property
    def pending(self): return self.state.pending
    @property
    def rng_positions(self): return self.state.rng_positions
    @property
    def stop_states(self): return self.state.stop_states
    @property
    def tokens(self): return self.state.tokens
    @property
    def logprobs(self): return self.state.logprobs

    def _check_open(self):
        if self.closed or self.decoder._active_session is not self or self.engine._cuda_decoder is not self.decoder:
            raise RuntimeError("Native generation session is closed")
        if self.engine.policy_version != self.policy_version:
            raise ValueError("Session cache belongs to another policy version")

    @contextmanager
    def _timed(self, phase):
        if not self.profile_timings:
            yield
            return
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record()
        try:
            yield
        finally:
            end.record()
            self._timing_events.append((phase, start, end))

    def timing_stats(self):
        if self._timing_events:
            self._timing_events[-1][2].synchronize()
        result = {}
        for phase, start, end in self._timing_events:
            key = phase + "_gpu_seconds"
            result[key] = result.get(key, 0.0) + start.elapsed_time(end) / 1000
        return result

    def _validate(self, prompt, sampling):
        vocab = self.engine.config.vocab_size
        if sampling.behavior_topk > self.behavior_topk:
            raise ValueError("Request behavior head exceeds the session reservation")
        if not prompt:
            raise ValueError("Empty prompts are not supported")
        if any(type(t) is not int or not 0 <= t < vocab for t in prompt):
            raise ValueError("Prompt token outside the model vocabulary")
        if len(prompt) + sampling.max_new_tokens > self.cache.max_seq_len:
            raise ValueError("Request exceeds reserved session context capacity")
        if sampling.max_new_tokens > self.max_new_tokens:
            raise ValueError("Request exceeds the session generation buffer")
        if sampling.top_k or sampling.top_p != 1.0 or sampling.repetition_penalty != 1.0:
            raise ValueError("Sessions support greedy/full-support sampling without repetition penalties")
        if sampling.stop_token_sequences:
            raise ValueError("Sessions use stop_token_ids or stop_table; encode string stops with build_stop_table")
        if any(not 0 <= t < vocab for t in sampling.stop_token_ids):
            raise ValueError("Stop token outside the model vocabulary")
        table = sampling.stop_table
        if table is not None and (table.ndim != 2 or table.size(1) != vocab or table.dtype != torch.int32):
            raise ValueError("stop_table must be an int32 state-by-vocabulary table")

    @staticmethod
    def _stop_key(sampling):
        return (id(sampling.stop_table), sampling.stop_token_ids)

    def _stop_offset(self, sampling) -> int:
        if sampling.stop_table is None and not sampling.stop_token_ids:
            return 0
        key = self._stop_key(sampling)
        if key not in self._stop_tables:
            table = build_token_stop_table(sampling, self.engine.config.vocab_size, self.engine.device)
            try:
                offset = self.state.add_stop_table(table)
            except ValueError:
                self._recycle_stop_tables()
                offset = self.state.add_stop_table(table)
            # keep the source table alive so a later table cannot reuse its id()
            self._stop_tables[key] = (offset, sampling.stop_table, table)
        return self._stop_tables[key][0]

    def _recycle_stop_tables(self) -> None:
        """The arena is full: keep only the tables a resident request still refers to, packed from the
        start, and point those requests' slots at the new offsets (chains of requests with ever new stop
        rules would otherwise fill the arena for good)."""
        resident = {slot: self._stop_key(r.sampling) for slot, r in enumerate(self.requests)
                    if r is not None and (r.sampling.stop_table is not None or r.sampling.stop_token_ids)}
        parked = {self._stop_key(s) for _, s, _ in self._queued.values() if s.stop_table is not None or s.stop_token_ids}
        if parked:
            raise ValueError("stop tables exceed the reserved stop-state arena while requests with stop rules are parked "
                             "in the device-side queue: raise enable_cuda_graphs(stop_states=...)")
        # (a request that is being armed right now is resident already, but its table is the one being added)
        resident = {slot: key for slot, key in resident.items() if key in self._stop_tables}
        keep = {key: entry for key, entry in self._stop_tables.items() if key in set(resident.values())}
        self.state.stop_table_used = self.engine.config.vocab_size
        self._stop_tables = {}
        for key, (_, source, table) in keep.items():
            self._stop_tables[key] = (self.state.add_stop_table(table), source, table)
        if resident:
            slots = torch.tensor(sorted(resident), device=self.engine.device, dtype=torch.int64)
            offsets = torch.tensor([self._stop_tables[resident[s]][0] for s in sorted(resident)],
                                   device=self.engine.device, dtype=torch.int64)
            self.state.stop_offsets.index_copy_(0, slots, offsets)

    def _configure(self, slots, prompts, samplings, *, rng_positions=None, stop_states=None):
        for slot, prompt, sampling in zip(slots, prompts, samplings):
            self.versions[slot] += 1
            self.requests[slot] = _Request(tuple(prompt), sampling, self.versions[slot])
        self.state.configure(
            list(slots), limits=[s.max_new_tokens for s in samplings],
            seeds=[s.seed & 0x7FFFFFFFFFFFFFFF for s in samplings],
            temperatures=[float(s.temperature) for s in samplings], ignore_eos=[int(s.ignore_eos) for s in samplings],
            stop_offsets=[self._stop_offset(s) for s in samplings], rng_offsets=0,
            rng_positions=rng_positions, stop_states=stop_states)

    @torch.inference_mode()
    def admit(self, prompts: Sequence[Sequence[int]], samplings: Sequence[LFM25SamplingConfig], *,
              slots: Sequence[int] | None = None, device_prompts: Sequence[torch.Tensor] | None = None) -> list[int]:
        """Prefill ``prompts`` into free slots (lowest first unless ``slots`` names them) and start their
        generation. ``device_prompts`` (optional, one int64 tensor per prompt, already on the engine's
        device and holding the same ids) skips the host-to-device copy of the token ids."""
        self._check_open()
        self._not_in_queue_mode("admit")
        if len(prompts) != len(samplings):
            raise ValueError("One sampling configuration is required per prompt")
        if device_prompts is not None and len(device_prompts) != len(prompts):
            raise ValueError("device_prompts must align with prompts")
        free = [i for i, request in enumerate(self.requests) if request is None]
        slots = list(free[:len(prompts)] if slots is None else slots)
        if len(slots) != len(prompts) or len(set(slots)) != len(slots) or any(i not in free for i in slots):
            raise ValueError("Admission requires distinct free session slots")
        order = sorted(range(len(slots)), key=lambda i: slots[i])
        work = [(slots[i], prompts[i], samplings[i]) for i in order]
        for _, prompt, sampling in work:
            self._validate(prompt, sampling)
        if not work:
            return slots
        ordered_slots = [slot for slot, _, _ in work]
        with self._timed("prefill"):
            if device_prompts is None:
                self.engine._prefill_packed(self.cache, ordered_slots, [list(p) for _, p, _ in work], [0] * len(work),
                                            self.entry.logits, self.decoder.max_prefill_tokens)
            else:
                staged = [device_prompts[i] for i in order]
                if any(t.numel() != len(p) for t, (_, p, _) in zip(staged, work)):
                    raise ValueError("device_prompts must hold the same ids as prompts")
                self.engine._prefill_packed(self.cache, ordered_slots, [len(p) for _, p, _ in work], [0] * len(work),
                                            self.entry.logits, self.decoder.max_prefill_tokens,
                                            flat_tokens=torch.cat(staged).to(torch.int64))
        for slot, prompt, _ in work:
            self.stats["slot_refills"] += int(self.versions[slot] > 0)
            self.stats["prefilled_tokens"] += len(prompt)
            self.stats["admitted_requests"] += 1
        self._configure(ordered_slots, [p for _, p, _ in work], [s for _, _, s in work])
        self.stats["peak_live_slots"] = max(self.stats["peak_live_slots"], sum(r is not None for r in self.requests))
        return slots

    # ---- prefix snapshots (reference: lfm25_session.py:294-391) ----------------------------------------
    # A snapshot is a spare row of the paged cache: it holds references to the prefix's full pages, a
    # private tail page, the conv taps and the next-token logits. Children share the full pages and copy
    # only the tail page, where the reference copies the whole prefix per child.
    def _take_row(self) -> int:
        if not self._free_rows:
            raise RuntimeError("No free snapshot row: release a snapshot or raise enable_cuda_graphs(snapshot_rows=...)")
        return self._free_rows.pop(0)

    def _snapshot_bytes(self, state: _SnapshotState) -> int:
        cache = self.cache
        kv = 2 * state.length * cache.n_attn_layers * cache.n_kv_heads * cache.head_dim * cache.kv_pool.element_size()
        if cache.kv_scales is not None:
            kv += 2 * state.length * cache.n_attn_layers * cache.n_kv_heads * 4
        conv = cache.n_conv_layers * 3 * cache.hidden_size * cache.conv_state.element_size()
        return kv + conv + state.logits.numel() * state.logits.element_size()

    def _store_snapshot(self, prefix, row, length, logits, seed=0, rng_position=0, stop_state=0):
        self._next_snapshot += 1
        lease = LFM25PrefixSnapshot(self, self._next_snapshot, self.policy_version, tuple(prefix))
        self._snapshots[lease.identity] = _SnapshotState(lease, row, length, logits, seed, rng_position, stop_state)
        self.stats["snapshot_count"] += 1
        self.stats["peak_snapshots"] = max(self.stats["peak_snapshots"], len(self._snapshots))
        size = sum(self._snapshot_bytes(s) for s in self._snapshots.values())
        self.stats["peak_snapshot_bytes"] = max(self.stats["peak_snapshot_bytes"], size)
        return lease

    def _run_into_row(self, row: int, tokens, start: int) -> torch.Tensor:
        logits = torch.empty((1, self.engine.config.vocab_size), device=self.engine.device, dtype=self.engine.dtype)
        try:
            self.engine._prefill_packed(self.cache, [row], [list(tokens)], [start], logits,
                                        self.decoder.max_prefill_tokens, logits_rows=[0])
            self.cache.check_status()
        except Exception:
            self._drop_row(row)
            raise
        return logits

    def _drop_row(self, row: int) -> None:
        mask = torch.zeros(self.cache.n_rows, dtype=torch.uint8)
        mask[row] = 1
        self.cache.release_rows(mask.to(self.engine.device))
        self._free_rows.append(row)
        self._free_rows.sort()

    @torch.inference_mode()
    def prefill_snapshot(self, prompt: Sequence[int]) -> LFM25PrefixSnapshot:
        """Prefill one exact prefix under the current weights, once."""
        self._check_open()
        prompt = tuple(prompt)
        self._validate(prompt, LFM25SamplingConfig(max_new_tokens=1))
        row = self._take_row()
        with self._timed("prefill"):
            logits = self._run_into_row(row, prompt, 0)
        self.stats["prefilled_tokens"] += len(prompt)
        self.stats["snapshot_prefilled_tokens"] += len(prompt)
        return self._store_snapshot(prompt, row, len(prompt), logits)

    @torch.inference_mode()
    def snapshot(self, handle: LFM25ContinuationHandle) -> LFM25PrefixSnapshot:
        """Park a finished request's context: its cached pages by reference, and its pending last token
        appended once here (the reference replays it once per child at fork time)."""
        request = self._request_for(handle)
        length = len(handle.prefix_token_ids) - 1
        if int(self.cache.seq_lens[handle.slot]) != length:
            raise ValueError("Cached position does not match the pending-token prefix")
        if length + 1 > self.cache.max_seq_len:
            raise ValueError("Request exceeds reserved session context capacity")
        row = self._take_row()
        dev = self.engine.device
        with self._timed("cache_copy"):
            self.cache.fork(torch.tensor([handle.slot], device=dev, dtype=torch.int32),
                            torch.tensor([row], device=dev, dtype=torch.int32),
                            torch.tensor([length], device=dev, dtype=torch.int32))
        with self._timed("append"):
            logits = self._run_into_row(row, handle.prefix_token_ids[-1:], length)
        return self._store_snapshot(handle.prefix_token_ids, row, length + 1, logits, request.sampling.seed,
                                    int(self.state.rng_positions[handle.slot]), int(self.state.stop_states[handle.slot]))

    def _snapshot_for(self, snapshot) -> _SnapshotState:
        self._check_open()
        if snapshot.policy_version != self.engine.policy_version:
            raise ValueError("Snapshot belongs to another policy version")
        state = self._snapshots.get(snapshot.identity)
        if snapshot.session is not self or state is None or state.lease is not snapshot:
            raise ValueError("Snapshot is released or belongs to another session")
        return state

    @torch.inference_mode()
    def fork(self, snapshot: LFM25PrefixSnapshot, samplings: Sequence[LFM25SamplingConfig], *,
             slots: Sequence[int] | None = None) -> list[int]:
        """Admit independent children of a snapshot into free slots, without prefill."""
        self._not_in_queue_mode("fork")
        state = self._snapshot_for(snapshot)
        free = [i for i, request in enumerate(self.requests) if request is None]
        slots = list(free[:len(samplings)] if slots is None else slots)
        if len(slots) != len(samplings) or len(set(slots)) != len(slots) or any(i not in free for i in slots):
            raise ValueError("Fork requires distinct free session slots")
        for sampling in samplings:
            self._validate(snapshot.prefix_token_ids, sampling)
        if not slots:
            return slots
        dev, n = self.engine.device, len(slots)
        with self._timed("cache_copy"):
            children = torch.tensor(slots, device=dev, dtype=torch.int32)
            self.cache.fork(torch.full((n,), state.row, device=dev, dtype=torch.int32), children,
                            torch.full((n,), state.length, device=dev, dtype=torch.int32))
            self.entry.logits.index_copy_(0, children.long(), state.logits.expand(n, -1))
        for slot in slots:
            self.stats["slot_refills"] += int(self.versions[slot] > 0)
        self._configure(slots, [snapshot.prefix_token_ids] * n, list(samplings))
        self.stats["forked_requests"] += n
        # tokens physically copied: only the partly filled last page of the prefix, per child
        self.stats["copied_prefix_tokens"] += (state.length % self.cache.page_size) * n
        self.stats["peak_live_slots"] = max(self.stats["peak_live_slots"], sum(r is not None for r in self.requests))
        return slots

    def release_snapshot(self, snapshot: LFM25PrefixSnapshot) -> None:
        state = self._snapshot_for(snapshot)
        del self._snapshots[snapshot.identity]
        self._drop_row(state.row)

    def _request_for(self, handle):
        self._check_open()
        if handle.session is not self or not 0 <= handle.slot < self.batch_size:
            raise ValueError("Continuation handle belongs to another session")
        request = self.requests[handle.slot]
        if request is None or request.version != handle.version or not request.delivered or request.handle is not handle:
            raise ValueError("Continuation handle is stale or already consumed")
        return request

    @torch.inference_mode()
    def resume(self, handles, prompts, samplings, *, preserve_rng: bool = False) -> None:
        if not len(handles) == len(prompts) == len(samplings):
            raise ValueError("One prompt and sampling configuration is required per handle")
        if len({h.slot for h in handles}) != len(handles):
            raise ValueError("Cannot resume a handle twice")
        work = []
        for handle, prompt, sampling in zip(handles, prompts, samplings):
            request = self._request_for(handle)
            self._validate(prompt, sampling)
            prefix = handle.prefix_token_ids
            if tuple(prompt[:len(prefix)]) != prefix:
                raise ValueError("Continuation requires the exact cached token prefix")
            if preserve_rng and (tuple(prompt) != prefix or sampling.seed != request.sampling.seed
                                 or sampling.stop_table is not request.sampling.stop_table
                                 or sampling.stop_token_ids != request.sampling.stop_token_ids):
                raise ValueError("Internal pauses must preserve the exact context, seed and stop rules")
            work.append((handle, tuple(prompt), sampling, request))
        if not work:
            return
        slots = [h.slot for h, _, _, _ in work]
        if preserve_rng:
            positions = self.state.rng_positions[slots].cpu().tolist()
            states = self.state.stop_states[slots].cpu().tolist()
        else:
            positions, states = [0] * len(slots), [0] * len(slots)
        # The final generated token never entered the cache: append it and the new suffix as one
        # continuation chunk starting at the slot's cached length (= len(prefix) - 1).
        appends = [list((h.prefix_token_ids[-1], *prompt[len(h.prefix_token_ids):])) for h, prompt, _, _ in work]
        starts = [len(h.prefix_token_ids) - 1 for h, _, _, _ in work]
        order = sorted(range(len(work)), key=lambda i: slots[i])
        with self._timed("append"):
            self.engine._prefill_packed(self.cache, [slots[i] for i in order], [appends[i] for i in order],
                                        [starts[i] for i in order], self.entry.logits, self.decoder.max_prefill_tokens)
        self._configure(slots, [p for _, p, _, _ in work], [s for _, _, s, _ in work],
                        rng_positions=positions, stop_states=states)
        for handle, prompt, _, _ in work:
            self.stats["resumed_prefix_tokens"] += len(handle.prefix_token_ids) - 1
            self.stats["appended_tokens"] += len(prompt) - len(handle.prefix_token_ids) + 1
            self.stats["resumed_requests"] += 1

    def _not_in_queue_mode(self, what: str) -> None:
        if self.queue_capacity:
            raise RuntimeError(f"{what} is not available on a session with a device-side queue: its slots are "
                               "assigned on the device (use enqueue)")

    # ---- device-side queue: eviction and admission inside the decode graph ---------------------------------
    @torch.inference_mode()
    def enqueue(self, prompts: Sequence[Sequence[int]], samplings: Sequence[LFM25SamplingConfig], *,
                device_prompts: Sequence[torch.Tensor] | None = None) -> list[int]:
        """Park ``prompts`` for admission on the device and return their request ids.

        Each prompt is prefilled now into a spare row of the paged cache; the decode graph itself moves it
        into the first slot that is free or whose request has just finished (lowest slot first, requests in
        the order they were enqueued), so between two ``poll`` calls finished rows are evicted and replaced
        without the host. Needs ``generation_session(queue_capacity=...)``; at most ``queue_capacity`` prompts
        wait at a time (``queue_space()``)."""
        self._check_open()
        if not self.queue_capacity:
            raise RuntimeError("enqueue needs a session opened with queue_capacity > 0")
        if len(prompts) != len(samplings):
            raise ValueError("One sampling configuration is required per prompt")
        n = len(prompts)
        if n == 0:
            return []
        if n > self.queue_space():
            raise ValueError("Admission queue is full: poll first, or open the session with a larger queue_capacity")
        for prompt, sampling in zip(prompts, samplings):
            self._validate(prompt, sampling)
        queue, dev = self.state.queue, self.engine.device
        rows = [self._free_rows.pop(0) for _ in range(n)]
        entries = [(self._queue_tail + i) % self.queue_capacity for i in range(n)]
        ids = list(range(self._next_request_id, self._next_request_id + n))
        with self._timed("prefill"):
            if device_prompts is None:
                self.engine._prefill_packed(self.cache, rows, [list(p) for p in prompts], [0] * n, queue["logits"],
                                            self.decoder.max_prefill_tokens, logits_rows=entries)
            else:
                self.engine._prefill_packed(self.cache, rows, [len(p) for p in prompts], [0] * n, queue["logits"],
                                            self.decoder.max_prefill_tokens, logits_rows=entries,
                                            flat_tokens=torch.cat(list(device_prompts)).to(torch.int64))
        index = torch.tensor(entries, device=dev, dtype=torch.int64)

        def put(name, values, dtype):
            queue[name].index_copy_(0, index, torch.tensor(values, device=dev, dtype=dtype))

        put("rows", rows, torch.int32)
        put("requests", ids, torch.int32)
        put("limits", [s.max_new_tokens for s in samplings], torch.int32)
        put("seeds", [s.seed & 0x7FFFFFFFFFFFFFFF for s in samplings], torch.int64)
        put("temperatures", [float(s.temperature) for s in samplings], torch.float32)
        put("ignore_eos", [int(s.ignore_eos) for s in samplings], torch.uint8)
        put("stop_offsets", [self._stop_offset(s) for s in samplings], torch.int64)
        queue["tail"].add_(n)  # publishes the entries: stream-ordered after everything above
        self._queue_tail += n
        self._next_request_id += n
        for rid, prompt, sampling, row in zip(ids, prompts, samplings, rows):
            self._queued[rid] = (tuple(prompt), sampling, row)
            self.stats["prefilled_tokens"] += len(prompt)
            self.stats["admitted_requests"] += 1
        return ids

    def queue_space(self) -> int:
        """Prompts that can be enqueued now: free queue entries, parked rows and result rows."""
        if not self.queue_capacity:
            return 0
        waiting = self._queue_tail - self._queue_consumed
        results_free = self.state.queue["result_capacity"] - len(self._queued)
        return max(0, min(self.queue_capacity - waiting, len(self._free_rows), results_free))

    def _poll_queue(self, steps: int) -> list[LFM25SessionResult]:
        self.poll_begin(steps=steps)
        return self.poll_end()

    @torch.inference_mode()
    def poll_begin(self, *, steps: int | None = None) -> None:
        """First half of ``poll`` in queue mode: launch ``steps`` replays (slot turnover runs inside each) and one
        more turnover, so that the last step's finishers are published and replaced, and start copying what the
        host reads (queue head, result index, status word, live context) on a stream of its own. Returns at once:
        whatever the caller launches next (``enqueue`` of the next prompts) queues behind the decode steps while
        the host is still free to prepare it, and ``poll_end`` does not wait for it."""
        self._check_open()
        if not self.queue_capacity:
            raise RuntimeError("poll_begin / poll_end need a session opened with queue_capacity > 0")
        if self._poll_pending is not None:
            raise RuntimeError("poll_end the previous poll first")
        steps = self.decoder.finish_check_interval if steps is None else steps
        if type(steps) is not int or steps <= 0:
            raise ValueError("steps must be a positive integer")
        queue, dev = self.state.queue, self.engine.device
        launched = bool(self._queued)
        if launched:
            with self._timed("decode"):
                for _ in range(steps):
                    self.entry.graph.replay()
                self.decoder._turnover(self.entry)
            self.stats["decode_steps"] += steps
            self.stats["decode_row_steps"] += self.batch_size * steps
            self.stats["reserved_row_steps"] += self.batch_size * steps
            batches = self.stats["decode_batches"]
            batches[str(self.batch_size)] = batches.get(str(self.batch_size), 0) + steps
        if self._read_stream is None:
            self._read_stream = torch.cuda.Stream(device=dev)
            ring = queue["result_capacity"]
            self._host_head = torch.zeros(1, dtype=queue["head"].dtype).pin_memory()
            self._host_reasons = torch.zeros(ring, dtype=torch.int8).pin_memory()
            self._host_status = torch.zeros(1, dtype=torch.int32).pin_memory()
            self._host_context = torch.zeros(2, dtype=torch.float64).pin_memory()
        reads = self._read_stream
        reads.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(reads):
            self._host_head.copy_(queue["head"], non_blocking=True)
            self._host_reasons.copy_(queue["result_reasons"], non_blocking=True)
            self._host_status.copy_(self.cache.status, non_blocking=True)
            occupied = queue["slot_requests"] >= 0
            context = torch.stack([(self.cache.seq_lens[:self.batch_size] * occupied).sum(dtype=torch.float64),
                                   occupied.sum(dtype=torch.float64)])
            self._host_context.copy_(context, non_blocking=True)
            done = torch.cuda.Event()
            done.record(reads)
        self._poll_pending = (done, launched)

    @torch.inference_mode()
    def poll_end(self) -> list[LFM25SessionResult]:
        """Second half of ``poll`` in queue mode: wait for the reads of ``poll_begin`` (not for work launched since)
        and deliver the requests that have finished."""
        self._check_open()
        if self._poll_pending is None:
            raise RuntimeError("poll_begin first")
        done_event, launched = self._poll_pending
        self._poll_pending = None
        done_event.synchronize()
        if not launched:
            return []
        queue, dev = self.state.queue, self.engine.device
        head = int(self._host_head.item())
        reasons = self._host_reasons.tolist()
        self.last_context = tuple(self._host_context.tolist())  # (cached tokens of the live rows, live rows)
        if int(self._host_status.item()):
            self.cache.check_status()
        ring = queue["result_capacity"]
        # parked rows whose prompt a slot has adopted are free again
        # (request ids are handed out in queue order, so the ids below `head` are the entries consumed so far)
        adopted = sorted(rid for rid, (_, _, row) in self._queued.items() if row is not None and rid < head)
        for rid in adopted:
            prompt, sampling, row = self._queued[rid]
            self._free_rows.append(row)
            self._queued[rid] = (prompt, sampling, None)
        self._free_rows.sort()
        self.stats["slot_refills"] += max(0, head - max(self._queue_consumed, self.batch_size))
        self._queue_consumed = head
        self.stats["peak_live_slots"] = max(self.stats["peak_live_slots"], min(self.batch_size, head))
        done = [rid for rid in sorted(self._queued) if self._queued[rid][2] is None and reasons[rid % ring]]
        if not done:
            return []
        # a finished request's result row is stable until the host marks it delivered, so it is read on the
        # read stream while the caller's stream goes on with later work
        with torch.cuda.stream(self._read_stream):
            index = torch.tensor([rid % ring for rid in done], device=dev)
            lengths = queue["result_lengths"][index].cpu().tolist()
            longest = max(lengths)
            tokens = self.state.tokens[:, :longest].index_select(0, index).cpu().tolist()
            logprobs = self.state.logprobs[:, :longest].index_select(0, index).cpu().tolist()
            queue["result_reasons"].index_fill_(0, index, 0)  # delivered: the result rows may be reused
        # work launched from here on (a later request that lands in one of these result rows) is ordered
        # behind that clearing; the read stream holds nothing else, so the caller's stream does not stall
        torch.cuda.current_stream(dev).wait_stream(self._read_stream)
        results = []
        for rid, length, ids, probs in zip(done, lengths, tokens, logprobs):
            prompt, sampling, _ = self._queued.pop(rid)
            results.append(LFM25SessionResult(None, prompt, tuple(ids[:length]),
                                              tuple(probs[:length]) if sampling.return_logprobs else None,
                                              reasons[rid % ring], None, rid))
        return results

    def _select_graph(self, live):
        captures = len(self.entry.compact_graphs)
        graph, size = self.decoder._select_graph(self.entry, live)
        self.stats["adaptive_graph_captures"] += len(self.entry.compact_graphs) - captures
        return graph, size

    @torch.inference_mode()
    def poll(self, *, steps: int | None = None) -> list[LFM25SessionResult]:
        self._check_open()
        steps = self.decoder.finish_check_interval if steps is None else steps
        if type(steps) is not int or steps <= 0:
            raise ValueError("steps must be a positive integer")
        if self.queue_capacity:
            return self._poll_queue(steps)
        live = [i for i, r in enumerate(self.requests) if r is not None and not r.delivered]
        if not live:
            return []
        graph, batch = self._select_graph(live)
        with self._timed("decode"):
            for _ in range(steps):
                graph.replay()
        self.stats["decode_steps"] += steps
        self.stats["decode_row_steps"] += batch * steps
        self.stats["reserved_row_steps"] += self.batch_size * steps
        batches = self.stats["decode_batches"]
        batches[str(batch)] = batches.get(str(batch), 0) + steps
        reasons = self.state.reasons.cpu().tolist()  # the one device->host read per poll
        self.cache.check_status()
        done = [i for i in live if reasons[i]]
        if not done:
            return []
        index = torch.tensor(done, device=self.engine.device)
        lengths = self.state.lengths[index].cpu().tolist()
        longest = max(lengths)
        tokens = self.state.tokens[:, :longest].index_select(0, index).cpu().tolist()
        logprobs = self.state.logprobs[:, :longest].index_select(0, index).cpu().tolist()
        results = []
        for slot, length, ids, probs in zip(done, lengths, tokens, logprobs):
            request = self.requests[slot]
            request.delivered = True
            ids = tuple(ids[:length])
            handle = LFM25ContinuationHandle(self, slot, request.version, request.prompt + ids)
            request.handle = handle
            k = request.sampling.behavior_topk
            head = (BehaviorTopK(self.state.head_ids[slot, :length, :k].cpu(),
                                 self.state.head_logprobs[slot, :length, :k].cpu()) if k else None)
            results.append(LFM25SessionResult(handle, request.prompt, ids,
                                              tuple(probs[:length]) if request.sampling.return_logprobs else None,
                                              reasons[slot], head))
        return results

    @torch.inference_mode()
    def release(self, handle: LFM25ContinuationHandle) -> None:
        self._request_for(handle)
        slot = handle.slot
        self.requests[slot] = None
        self.versions[slot] += 1
        mask = torch.zeros(self.batch_size, dtype=torch.uint8)
        mask[slot] = 1
        mask = mask.to(self.engine.device)
        self.state.alive.masked_fill_(mask.bool(), 0)
        self.state.pending.masked_fill_(mask.bool(), 0)
        self.cache.release(mask)

    @torch.inference_mode()
    def close(self):
        if not self.closed:
            self.closed = True
            self._poll_pending = None
            if self._read_stream is not None:  # reads in flight finish before the state they read is reused
                torch.cuda.current_stream(self.engine.device).wait_stream(self._read_stream)
            self.requests = [None] * self.batch_size
            self.state.alive.zero_()
            self.state.pending.zero_()
            if self._snapshots:  # parked prefixes give their pages back with the session
                mask = torch.zeros(self.cache.n_rows, dtype=torch.uint8)
                mask[[s.row for s in self._snapshots.values()]] = 1
                self.cache.release_rows(mask.to(self.engine.device))
                self._snapshots.clear()
            if self.decoder._active_session is self:
                self.decoder._active_session = None

    def __enter__(self):
        self._check_open()
        return self

    def __exit__(self, *_):
        self.close()
