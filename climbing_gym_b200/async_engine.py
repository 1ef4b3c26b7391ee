"""asyncio front end of the token engine: the adapter rollout workers talk to.

Same surface as the reference adapter (src/climbing_gym/inference/lfm25_async_engine.py:35-729):
``generate`` / ``generate_many`` coalesce concurrent requests that share a sampling configuration
into one packed ``LFM25Engine.generate`` call; ``generate_chains`` drives multi-phase requests
through a generation session with exact-prefix continuation; ``sync_from_model`` swaps policy
weights once in-flight work has drained. All engine work is serialised behind one lock and runs on
executor threads, so the event loop never blocks on the GPU.

Design notes: requests wait in per-sampling-key buckets (insertion ordered) instead of one list that
is re-partitioned on every flush, and one dispatcher task drains the buckets oldest key first.
"""
from __future__ import annotations

import asyncio
import gc
import math
import threading
import uuid
from collections import OrderedDict
from dataclasses import dataclass, replace
from typing import Any, Callable, Mapping, Sequence

import torch

from .config import InferenceEngineConfig, LFM25SamplingConfig, SamplingConfig
from .text_stops import build_stop_table, trim_after_stop
from .types import BehaviorTopK, GenerationOutput, GenerationResult

_CLOSED = "LFM25AsyncInferenceEngine is closed"
# odd 64-bit multipliers that spread (chain, phase) over the seed space
_CHAIN_STRIDE, _PHASE_STRIDE, _SEED_MASK = 0x517CC1B727220A95, 0x6C8E9CF570932BD5, 0x7FFFFFFFFFFFFFFF
# a stop string may be tokenised differently after these lead-ins
_STOP_LEAD_INS = ("", " ", "\n", ">")


@dataclass
class _Ticket:
    """One queued generate() call."""

    prompt: Any
    prompt_text: str
    prompt_token_ids: tuple
    sampling: SamplingConfig
    request_id: str
    future: "asyncio.Future[GenerationResult]"


def finish_reason_names(reason: int) -> tuple[str | None, str | None]:
    """Engine finish code -> (finish_reason, stop_reason) of the public result
    (lfm25_async_engine.py:712-719): 1 EOS, 2 stop sequence, 3 length."""
    return {1: ("stop", "eos"), 2: ("stop", "stop"), 3: ("length", None)}.get(int(reason), (None, None))


def sampling_bucket_key(sampling: SamplingConfig) -> tuple:
    return (float(sampling.temperature), int(sampling.top_k), float(sampling.top_p), int(sampling.max_tokens),
            int(sampling.n), tuple(sampling.stop), sampling.logprobs, tuple(sorted(dict(sampling.extra_params).items())))


def to_engine_sampling(sampling: SamplingConfig, *, seed: int, tokenizer=None) -> LFM25SamplingConfig:
    if int(sampling.n) != 1:
        raise ValueError("LFM25AsyncInferenceEngine requires sampling.n == 1")
    if sampling.stop and tokenizer is None:
        raise ValueError("A tokenizer is required for string stop sequences")
    extra = dict(sampling.extra_params)
    sequences = []
    for stop in sampling.stop:
        for lead_in in _STOP_LEAD_INS:
            ids = tuple(tokenizer.encode(lead_in + stop, add_special_tokens=False))
            if ids not in sequences:
                sequences.append(ids)
    return LFM25SamplingConfig(
        temperature=float(sampling.temperature), top_k=0 if int(sampling.top_k) == -1 else int(sampling.top_k),
        top_p=float(sampling.top_p), repetition_penalty=float(extra.get("repetition_penalty", 1.0)),
        max_new_tokens=int(sampling.max_tokens), return_logprobs=sampling.logprobs is not None, seed=seed,
        ignore_eos=bool(extra.get("ignore_eos", False)), stop_token_sequences=tuple(sequences),
        behavior_topk=extra.get("behavior_topk", 0))


def _batch_limit(config: InferenceEngineConfig, requested: int | None) -> int:
    if requested is not None and (type(requested) is not int or requested <= 0):
        raise ValueError("max_batch_size must be a positive integer")
    limit = requested if requested is not None else (config.max_num_seqs or 64)
    return min(limit, config.max_num_seqs) if config.max_num_seqs is not None else limit


class LFM25AsyncInferenceEngine:
    """Async batching adapter around the in-process B200 token engine."""

    def __init__(self, config: InferenceEngineConfig, *, batch_wait_seconds: float = 0.001,
                 max_batch_size: int | None = None, compile_decode: bool = True, cuda_graphs: bool = False,
                 bf16_weight_packing: bool = True, max_cuda_graphs: int = 1, max_prefill_tokens: int = 4096,
                 fp8_mlp: bool = False, fp8_kv: bool = False, adaptive_batching: bool = False,
                 fp8_lm_head: bool = False, fp8_operators: bool = False) -> None:
        for enabled, what in ((fp8_mlp, "FP8 MLP requires"), (fp8_kv, "FP8 KV cache requires"),
                              (adaptive_batching, "adaptive batching requires"),
                              (fp8_lm_head, "FP8 vocabulary head requires"), (fp8_operators, "FP8 operators require")):
            if enabled and not cuda_graphs:
                raise ValueError(f"Native {what} cuda_graphs=True")
        if fp8_operators:
            raise ValueError("FP8 operator projections currently require LFM3")
        from .engine import LFM25Engine
        from .weights import load_tokenizer

        self._setup(config, batch_wait_seconds, _batch_limit(config, max_batch_size))
        self.tokenizer = load_tokenizer(config.model_path)
        self._engine = LFM25Engine.from_pretrained(config.model_path, dtype=config.dtype, device="cuda",
                                                   max_model_len=config.max_model_len)
        self._owns_engine = True
        del compile_decode  # the decode step of this engine is always its captured kernel graph
        try:
            # the CUDA library is the only compute path of this package, so the graph decoder is always installed
            self._engine.enable_cuda_graphs(bf16_weight_packing=bf16_weight_packing, max_graphs=max_cuda_graphs,
                                            max_prefill_tokens=max_prefill_tokens, fp8_mlp=fp8_mlp, fp8_kv=fp8_kv,
                                            adaptive_batching=adaptive_batching, fp8_lm_head=fp8_lm_head)
        except BaseException as error:
            try:
                self.close()
            except BaseException as cleanup:  # pragma: no cover - double fault
                error.add_note(f"Native setup cleanup also failed: {cleanup}")
            raise

    def _setup(self, config: InferenceEngineConfig, batch_wait_seconds: float, max_batch_size: int) -> None:
        self.config = config
        self.batch_wait_seconds = max(0.0, float(batch_wait_seconds))
        self.max_batch_size = max_batch_size
        self._buckets: "OrderedDict[tuple, list[_Ticket]]" = OrderedDict()
        self._queue_lock: asyncio.Lock | None = None
        self._dispatcher: asyncio.Task | None = None
        self._closed = False
        self._engine_lock = threading.Lock()
        self._seed_lock = threading.Lock()
        self._generation_index = 0
        self._stop_tables: dict = {}
        self.last_session_stats: dict = {}

    @classmethod
    def from_components(cls, *, engine, tokenizer: Any, config: InferenceEngineConfig | None = None,
                        batch_wait_seconds: float = 0.0, max_batch_size: int = 64) -> "LFM25AsyncInferenceEngine":
        """Wrap a caller-owned engine and tokenizer (the engine outlives close())."""
        self = cls.__new__(cls)
        config = config or InferenceEngineConfig(model_path="")
        self._setup(config, batch_wait_seconds, _batch_limit(config, max_batch_size))
        self.tokenizer, self._engine, self._owns_engine = tokenizer, engine, False
        return self

    # ---- introspection -------------------------------------------------------------------------------
    @property
    def raw_engine(self):
        if self._engine is None:
            raise RuntimeError(_CLOSED)
        return self._engine

    def supports_token_prompt_bridge(self) -> bool:
        return True

    # ---- prompts -------------------------------------------------------------------------------------
    def tokenize_prompt(self, prompt, *, assistant_prefill: str | None = None,
                        chat_template_enable_thinking: bool | None = None) -> tuple:
        """Render and tokenise a prompt exactly as generation would, without generating."""
        prefill = str(self.config.assistant_prefill) if assistant_prefill is None else str(assistant_prefill)
        return self._resolve_prompt(prompt, assistant_prefill=prefill,
                                    chat_template_enable_thinking=chat_template_enable_thinking)[2]

    @classmethod
    def tokenize_for_config(cls, config: InferenceEngineConfig, tokenizer: Any, prompt, *,
                            assistant_prefill: str | None = None,
                            chat_template_enable_thinking: bool | None = None) -> tuple:
        """tokenize_prompt with only a tokenizer at hand (no model, no GPU state)."""
        renderer = cls.__new__(cls)
        renderer.config, renderer.tokenizer = config, tokenizer
        return renderer.tokenize_prompt(prompt, assistant_prefill=assistant_prefill,
                                        chat_template_enable_thinking=chat_template_enable_thinking)

    def _encode_text(self, text: str) -> tuple:
        return tuple(int(t) for t in self.tokenizer.encode(str(text), add_special_tokens=False))

    def _render_chat(self, prompt: str, enable_thinking: bool | None) -> str:
        if not bool(self.config.apply_chat_template):
            return str(prompt)
        render = getattr(self.tokenizer, "apply_chat_template", None)
        if not callable(render):
            raise TypeError("apply_chat_template=true requires a tokenizer with apply_chat_template(...)")
        thinking = bool(self.config.chat_template_enable_thinking) if enable_thinking is None else bool(enable_thinking)
        messages = [{"role": "user", "content": str(prompt)}]
        try:
            return str(render(messages, tokenize=False, add_generation_prompt=True, enable_thinking=thinking))
        except TypeError as exc:
            text = str(exc)
            if "enable_thinking" not in text or ("unexpected keyword" not in text and "got an unexpected" not in text):
                raise
            return str(render(messages, tokenize=False, add_generation_prompt=True))

    def _resolve_prompt(self, prompt, *, assistant_prefill: str = "",
                        chat_template_enable_thinking: bool | None = None):
        """-> (prompt as echoed in the result, prompt text, prompt token ids)."""
        prefill = str(assistant_prefill or "")
        if isinstance(prompt, Mapping):
            text = str(prompt.get("prompt", prompt.get("text", "")) or "")
            given = prompt.get("prompt_token_ids")
            ids = self._encode_text(text) if given is None else tuple(int(t) for t in given or ())
            if not prefill:
                return prompt, text, ids
            text, ids = text + prefill, ids + self._encode_text(prefill)
            echoed = dict(prompt)
            for key in ("prompt", "text"):
                if key in echoed:
                    echoed[key] = text
                    break
            echoed["prompt_token_ids"] = list(ids)
            return echoed, text, ids
        if isinstance(prompt, str):
            text = self._render_chat(prompt, chat_template_enable_thinking) + prefill
            return text, text, self._encode_text(text)
        ids = tuple(int(t) for t in prompt)
        text = self.tokenizer.decode(ids, skip_special_tokens=False)
        if prefill:
            text, ids = text + prefill, ids + self._encode_text(prefill)
        return list(ids), text, ids

    def _resolve_sampling(self, sampling) -> SamplingConfig:
        if sampling is None:
            return self.config.default_sampling
        if isinstance(sampling, SamplingConfig):
            return sampling
        if isinstance(sampling, Mapping):
            raise TypeError("sampling must be a SamplingConfig or a sampling-attribute object, not a mapping")
        return SamplingConfig(
            temperature=float(getattr(sampling, "temperature", 0.0)), top_k=int(getattr(sampling, "top_k", -1)),
            top_p=float(getattr(sampling, "top_p", 1.0)),
            max_tokens=int(getattr(sampling, "max_tokens", getattr(sampling, "max_new_tokens", 256))),
            n=int(getattr(sampling, "n", 1)), logprobs=getattr(sampling, "logprobs", None),
            stop=getattr(sampling, "stop", ()) or (), extra_params=getattr(sampling, "extra_params", {}) or {})

    def _engine_sampling(self, sampling: SamplingConfig, seed: int) -> LFM25SamplingConfig:
        native = to_engine_sampling(sampling, seed=seed, tokenizer=self.tokenizer)
        if not sampling.stop:
            return native
        key = tuple(sampling.stop)
        if key not in self._stop_tables:  # one DFA per distinct stop set, kept on the device
            table = build_stop_table(self.tokenizer, key, vocab_size=self._engine.config.vocab_size)
            self._stop_tables[key] = table.to(self._engine.device)
        return replace(native, stop_token_sequences=(), stop_table=self._stop_tables[key])

    def _next_seed(self) -> int:
        with self._seed_lock:
            index, self._generation_index = self._generation_index, self._generation_index + 1
        return (int(self.config.seed) + index) % (1 << 64)

    # ---- lifecycle -----------------------------------------------------------------------------------
    def sync_from_model(self, model: Any, *, drain_timeout: int | float = 300):
        """Wait for in-flight generation to drain, then update the packed weights in place."""
        timeout = float(drain_timeout)
        if not math.isfinite(timeout) or timeout < 0.0:
            raise ValueError("drain_timeout must be finite and >= 0")
        if self._closed:
            raise RuntimeError(_CLOSED)
        if not self._engine_lock.acquire(timeout=timeout):
            raise TimeoutError(f"Timed out after {timeout:g}s waiting for native LFM2.5 generation to drain")
        try:
            if self._closed:
                raise RuntimeError(_CLOSED)
            return self._engine.sync_from_model(model, drain_timeout=drain_timeout)
        finally:
            self._engine_lock.release()

    def release_inference_buffers(self) -> None:
        with self._engine_lock:
            if self._engine is not None:
                self._engine.release_inference_buffers()

    def sleep(self, *, level: int = 1, mode: str = "abort") -> None:
        del level, mode
        self.release_inference_buffers()

    def wake(self, *, tags: Sequence[str] | None = None) -> None:
        del tags

    def close(self) -> None:
        """Cancel queued requests, wait for running work and drop the engine reference (an engine
        loaded by this adapter also frees its inference buffers)."""
        self._closed = True
        for tickets in self._buckets.values():
            for ticket in tickets:
                if not ticket.future.done():
                    ticket.future.cancel()
        self._buckets.clear()
        with self._engine_lock:
            engine, self._engine = self._engine, None
            if engine is None:
                return
            if self._owns_engine:
                engine.release_inference_buffers()
            self._stop_tables.clear()
        owned, device = self._owns_engine, getattr(engine, "device", None)
        del engine
        if owned:
            gc.collect()
            if device is not None and device.type == "cuda":
                torch.cuda.empty_cache()

    # ---- batched single-phase generation -----------------------------------------------------------------
    def _lock(self) -> asyncio.Lock:
        if self._queue_lock is None:
            self._queue_lock = asyncio.Lock()
        return self._queue_lock

    async def generate(self, prompt, *, sampling=None, request_id: str | None = None,
                       chat_template_enable_thinking: bool | None = None,
                       assistant_prefill: str = "") -> GenerationResult:
        if self._closed:
            raise RuntimeError(_CLOSED)
        resolved = self._resolve_sampling(sampling)
        echoed, text, ids = self._resolve_prompt(
            prompt, assistant_prefill=str(assistant_prefill) if assistant_prefill else str(self.config.assistant_prefill),
            chat_template_enable_thinking=chat_template_enable_thinking)
        ticket = _Ticket(echoed, text, ids, resolved, request_id or f"req-{uuid.uuid4().hex}",
                         asyncio.get_running_loop().create_future())
        async with self._lock():
            if self._closed:
                raise RuntimeError(_CLOSED)
            self._buckets.setdefault(sampling_bucket_key(resolved), []).append(ticket)
            if self._dispatcher is None or self._dispatcher.done():
                self._dispatcher = asyncio.create_task(self._dispatch())
        return await ticket.future

    async def generate_many(self, prompts: Sequence, *, sampling=None) -> list[GenerationResult]:
        return await asyncio.gather(*(self.generate(prompt, sampling=sampling) for prompt in prompts))

    async def _dispatch(self) -> None:
        """Drain the buckets: oldest sampling key first, at most max_batch_size requests per engine call."""
        if self.batch_wait_seconds > 0:
            await asyncio.sleep(self.batch_wait_seconds)
        while True:
            async with self._lock():
                if not self._buckets:
                    return
                key, tickets = next(iter(self._buckets.items()))
                batch, rest = tickets[:self.max_batch_size], tickets[self.max_batch_size:]
                if rest:
                    self._buckets[key] = rest
                else:
                    del self._buckets[key]
            if not batch:
                continue
            try:
                results = await asyncio.get_running_loop().run_in_executor(None, self._run_batch, tuple(batch))
            except Exception as exc:
                for ticket in batch:
                    if not ticket.future.done():
                        ticket.future.set_exception(exc)
                continue
            for ticket, result in zip(batch, results, strict=True):
                if not ticket.future.done():
                    ticket.future.set_result(result)

    def _run_batch(self, batch: tuple) -> list[GenerationResult]:
        from .engine import flatten_token_batches

        with self._engine_lock:
            if self._closed:
                raise RuntimeError(_CLOSED)
            sampling = self._engine_sampling(batch[0].sampling, self._next_seed())
            flat, cu, longest = flatten_token_batches([list(t.prompt_token_ids) for t in batch], device=self._engine.device)
            output = self._engine.generate(flat, cu, longest, repeats=1, sampling=sampling)
            if self._engine.device.type == "cuda":
                torch.cuda.synchronize(self._engine.device)
            return self._results_of(batch, output)

    def _results_of(self, batch: Sequence[_Ticket], output) -> list[GenerationResult]:
        # one device->host transfer per tensor, not per row
        lengths = output.lengths[:, 0].cpu()
        longest = int(lengths.max()) if lengths.numel() else 0
        tokens = output.token_ids[:, 0, :longest].cpu()
        reasons = output.finish_reasons[:, 0].cpu()
        logprobs = None if output.logprobs is None else output.logprobs[:, 0, :longest].cpu()
        head_ids = None if output.topk_token_ids is None else output.topk_token_ids[:, 0, :longest].cpu()
        head_lp = None if output.topk_logprobs is None else output.topk_logprobs[:, 0, :longest].cpu()
        results = []
        for row, ticket in enumerate(batch):
            n = int(lengths[row])
            ids = tuple(int(t) for t in tokens[row, :n].tolist())
            lps = None if logprobs is None else tuple(float(v) for v in logprobs[row, :n].tolist())
            finish, stop = finish_reason_names(int(reasons[row]))
            text = self.tokenizer.decode(ids, skip_special_tokens=False)
            if stop == "stop" and ticket.sampling.stop:
                text = trim_after_stop(text, ticket.sampling.stop)  # the last token may run past the stop string
            head = None if head_ids is None else BehaviorTopK(head_ids[row, :n].clone(), head_lp[row, :n].clone())
            results.append(GenerationResult(
                request_id=ticket.request_id, prompt=ticket.prompt, prompt_token_ids=ticket.prompt_token_ids,
                outputs=(GenerationOutput(0, text, ids, lps, finish, stop, head),), finished=True,
                raw_output=output if head_ids is None else None))
        return results

    async def abort_async(self, request_id: str | Sequence[str]) -> None:
        wanted = {str(request_id)} if isinstance(request_id, str) else {str(r) for r in request_id}
        async with self._lock():
            for key in list(self._buckets):
                kept = []
                for ticket in self._buckets[key]:
                    if ticket.request_id in wanted:
                        ticket.future.cancel()
                    else:
                        kept.append(ticket)
                if kept:
                    self._buckets[key] = kept
                else:
                    del self._buckets[key]

    def abort(self, request_id: str | Sequence[str]) -> None:
        try:
            loop = asyncio.get_running_loop()
        except RuntimeError:
            asyncio.run(self.abort_async(request_id))
        else:
            loop.create_task(self.abort_async(request_id))

    # ---- multi-phase chains over a generation session ---------------------------------------------------------
    async def generate_chains(self, requests: Sequence[tuple], *,
                              on_result: Callable[[int, GenerationResult], tuple | None], max_new_tokens: int,
                              reuse_cache: bool = True, poll_interval: int | None = None) -> list[list[GenerationResult]]:
        """Run independent, possibly multi-phase requests with continuous batching.

        ``on_result(index, result)`` is called on the worker thread for every finished phase and
        returns the next ``(prompt, sampling)`` of that chain or None. A next prompt that extends the
        tokens already in the slot's cache consumes only its new tokens; anything else starts a fresh
        context. A finished chain's slot is refilled from the queue at once. Every (chain, phase) has
        its own RNG stream, independent of slot assignment and of what else is running."""
        if self._closed:
            raise RuntimeError(_CLOSED)
        if not requests:
            return []
        cancelled = threading.Event()
        worker = asyncio.get_running_loop().run_in_executor(
            None, self._run_chains, tuple(requests), on_result, max_new_tokens, reuse_cache, poll_interval, cancelled)
        try:
            return await asyncio.shield(worker)
        except asyncio.CancelledError:
            cancelled.set()
            try:
                await asyncio.shield(worker)  # drain before the caller may touch the engine again
            except Exception:
                pass
            raise

    def _run_chains(self, requests, on_result, max_new_tokens, reuse_cache, poll_interval, cancelled):
        with self._engine_lock:
            if self._closed:
                raise RuntimeError(_CLOSED)
            if cancelled.is_set():
                return [[] for _ in requests]
            seed = self._next_seed()
            results: list[list[GenerationResult]] = [[] for _ in requests]
            phase = [0] * len(requests)

            def prepare(index: int, request):
                prompt, sampling = request
                sampling = self._resolve_sampling(sampling)
                echoed, _, ids = self._resolve_prompt(prompt, assistant_prefill=str(self.config.assistant_prefill))
                key = (seed + index * _CHAIN_STRIDE + phase[index] * _PHASE_STRIDE) & _SEED_MASK
                return index, echoed, ids, sampling, self._engine_sampling(sampling, key)

            head_k = max(int(dict(self._resolve_sampling(s).extra_params).get("behavior_topk", 0)) for _, s in requests)
            waiting = iter(enumerate(requests))
            running: dict[int, tuple] = {}
            options = {"behavior_topk": head_k} if head_k else {}
            with self._engine.generation_session(max_batch_size=min(self.max_batch_size, len(requests)),
                                                 max_new_tokens=max_new_tokens, **options) as session:
                # range first: zip stops at the exhausted range without drawing another request from the queue
                first = [prepare(*item) for _, item in zip(range(session.batch_size), waiting)]
                running.update(zip(session.admit([p[2] for p in first], [p[4] for p in first]), first))
                while running and not cancelled.is_set() and not self._closed:
                    continued, admitted = [], []
                    for done in session.poll(steps=poll_interval):
                        slot = done.handle.slot
                        index, echoed, ids, sampling, _ = running.pop(slot)
                        finish, stop = finish_reason_names(done.finish_reason)
                        text = self.tokenizer.decode(done.token_ids, skip_special_tokens=False)
                        if stop == "stop" and sampling.stop:
                            text = trim_after_stop(text, sampling.stop)
                        result = GenerationResult(
                            request_id=f"chain-{index}-phase-{phase[index]}", prompt=echoed, prompt_token_ids=ids,
                            outputs=(GenerationOutput(0, text, done.token_ids, done.logprobs, finish, stop,
                                                      getattr(done, "behavior_topk", None)),),
                            finished=True, raw_output=None)
                        results[index].append(result)
                        following = on_result(index, result)
                        if following is None:
                            session.release(done.handle)
                            item = next(waiting, None)
                            if item is not None:
                                admitted.append((slot, prepare(*item)))
                            continue
                        phase[index] += 1
                        prepared = prepare(index, following)
                        cached = done.handle.prefix_token_ids
                        if reuse_cache and prepared[2][:len(cached)] == cached:
                            continued.append((done.handle, prepared))
                        else:
                            session.release(done.handle)
                            admitted.append((slot, prepared))
                    if continued:
                        session.resume([h for h, _ in continued], [p[2] for _, p in continued],
                                       [p[4] for _, p in continued])
                        running.update((h.slot, p) for h, p in continued)
                    if admitted:
                        session.admit([p[2] for _, p in admitted], [p[4] for _, p in admitted],
                                      slots=[s for s, _ in admitted])
                        running.update(admitted)
                self.last_session_stats = dict(session.stats)
            if self._closed and not cancelled.is_set():
                raise RuntimeError("LFM25AsyncInferenceEngine closed during generation")
            return results


AsyncInferenceEngine = LFM25AsyncInferenceEngine

__all__ = ["LFM25AsyncInferenceEngine", "AsyncInferenceEngine", "finish_reason_names", "sampling_bucket_key",
           "to_engine_sampling"]
