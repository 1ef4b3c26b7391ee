"""Host logic of the asyncio adapter, against a fake engine and tokenizer (no GPU): request
coalescing by sampling key, result assembly, prompt rendering, abort / close / weight-sync
ordering and the chain scheduler's resume-or-readmit decisions. Mirrors the behaviours the
reference pins in tests/test_lfm25_async_engine.py."""
import asyncio
import threading
import time
from types import SimpleNamespace

import pytest
import torch

from climbing_gym_b200.async_engine import (LFM25AsyncInferenceEngine, finish_reason_names, sampling_bucket_key,
                                            to_engine_sampling)
from climbing_gym_b200.config import InferenceEngineConfig, SamplingConfig
from climbing_gym_b200.types import LFM25GenerationOutput


class CharTokenizer:
    """One token per character, ids = code points."""

    def encode(self, text, add_special_tokens=False):
        return [ord(c) for c in text]

    def __len__(self):
        return 256

    def decode(self, ids, skip_special_tokens=False, clean_up_tokenization_spaces=False):
        return "".join(chr(int(i)) for i in ids)

    def apply_chat_template(self, messages, tokenize=False, add_generation_prompt=True, enable_thinking=True):
        return f"<user>{messages[0]['content']}</user><think={int(enable_thinking)}>"


class FakeSession:
    def __init__(self, engine, max_batch_size, max_new_tokens):
        self.engine, self.batch_size, self.max_new_tokens = engine, max_batch_size, max_new_tokens
        self.live, self.stats, self.log = {}, {"admitted_requests": 0, "resumed": 0}, engine.session_log

    def __enter__(self):
        return self

    def __exit__(self, *_):
        self.log.append(("closed",))

    def admit(self, prompts, samplings, *, slots=None):
        free = [s for s in range(self.batch_size) if s not in self.live]
        slots = list(free[:len(prompts)] if slots is None else slots)
        for slot, prompt, sampling in zip(slots, prompts, samplings):
            self.live[slot] = (tuple(prompt), sampling)
            self.stats["admitted_requests"] += 1
            self.log.append(("admit", slot, tuple(prompt), sampling.seed))
        return slots

    def resume(self, handles, prompts, samplings):
        for handle, prompt, sampling in zip(handles, prompts, samplings):
            self.live[handle.slot] = (tuple(prompt), sampling)
            self.stats["resumed"] += 1
            self.log.append(("resume", handle.slot, tuple(prompt), sampling.seed))

    def release(self, handle):
        self.live.pop(handle.slot, None)
        self.log.append(("release", handle.slot))

    def poll(self, *, steps=None):
        # every live request finishes at once: completion = "!" then the prompt's last token
        done = []
        for slot, (prompt, sampling) in sorted(self.live.items()):
            tokens = (ord("!"), prompt[-1])
            handle = SimpleNamespace(slot=slot, prefix_token_ids=prompt + tokens)
            done.append(SimpleNamespace(handle=handle, token_ids=tokens, logprobs=(-0.5, -0.25), finish_reason=3))
        return done


class FakeEngine:
    def __init__(self):
        self.device = torch.device("cpu")
        self.config = SimpleNamespace(vocab_size=256)
        self.calls, self.session_log, self.synced, self.released = [], [], [], 0
        self.block = None

    def generate(self, flat, cu, longest, *, repeats, sampling):
        if self.block is not None:
            self.block.wait(5)
        prompts = [flat[cu[i]:cu[i + 1]].tolist() for i in range(cu.numel() - 1)]
        self.calls.append((prompts, sampling))
        n, cap = len(prompts), sampling.max_new_tokens
        tokens = torch.zeros((n, 1, cap), dtype=torch.int64)
        lengths = torch.zeros((n, 1), dtype=torch.int32)
        reasons = torch.zeros((n, 1), dtype=torch.int8)
        for row, prompt in enumerate(prompts):
            out = list(reversed(prompt))[:cap]  # the "model" echoes the prompt backwards
            tokens[row, 0, :len(out)] = torch.tensor(out)
            lengths[row, 0] = len(out)
            reasons[row, 0] = 3 if len(out) == cap else 1
            if sampling.stop_table is not None and ord("X") in out:
                cut = out.index(ord("X")) + 2  # the stop string ends inside the NEXT token's text
                lengths[row, 0], reasons[row, 0] = min(cut, len(out)), 2
        logprobs = torch.full((n, 1, cap), -1.5) if sampling.return_logprobs else None
        return LFM25GenerationOutput(tokens, lengths, logprobs, reasons)

    def generation_session(self, *, max_batch_size, max_new_tokens, **_):
        return FakeSession(self, max_batch_size, max_new_tokens)

    def sync_from_model(self, model, *, drain_timeout=300):
        self.synced.append(model)
        return self

    def release_inference_buffers(self):
        self.released += 1


def make(**kwargs):
    engine = FakeEngine()
    config = kwargs.pop("config", InferenceEngineConfig(model_path="", seed=11))
    adapter = LFM25AsyncInferenceEngine.from_components(engine=engine, tokenizer=CharTokenizer(), config=config, **kwargs)
    return adapter, engine


def test_requests_sharing_a_sampling_key_run_as_one_packed_call():
    adapter, engine = make(max_batch_size=8)
    greedy = SamplingConfig(temperature=0.0, max_tokens=4, logprobs=1)
    warm = SamplingConfig(temperature=0.7, max_tokens=4)

    async def run():
        return await asyncio.gather(adapter.generate("abc", sampling=greedy), adapter.generate("xyz", sampling=warm),
                                    adapter.generate([100, 101], sampling=greedy, request_id="mine"))

    a, b, c = asyncio.run(run())
    assert len(engine.calls) == 2
    assert engine.calls[0][0] == [[97, 98, 99], [100, 101]] and engine.calls[1][0] == [[120, 121, 122]]
    assert [call[1].seed for call in engine.calls] == [11, 12]  # config.seed + generation index
    assert a.text == "cba" and a.token_ids == (99, 98, 97) and a.completion_logprobs == (-1.5, -1.5, -1.5)
    assert a.outputs[0].finish_reason == "stop" and a.outputs[0].stop_reason == "eos"
    assert b.completion_logprobs is None and b.prompt == "xyz"
    assert c.request_id == "mine" and c.prompt == [100, 101] and c.prompt_token_ids == (100, 101)
    assert a.request_id.startswith("req-") and a.finished


def test_batches_respect_max_batch_size_and_length_finish():
    adapter, engine = make(max_batch_size=2)
    sampling = SamplingConfig(max_tokens=2)
    results = asyncio.run(adapter.generate_many(["abcd", "efgh", "ijkl"], sampling=sampling))
    assert [len(call[0]) for call in engine.calls] == [2, 1]
    assert [r.text for r in results] == ["dc", "hg", "lk"]
    assert all(r.outputs[0].finish_reason == "length" and r.outputs[0].stop_reason is None for r in results)


def test_stop_strings_build_one_table_and_trim_the_text():
    adapter, engine = make()
    sampling = SamplingConfig(max_tokens=8, stop=("X",))
    first = asyncio.run(adapter.generate("abXcd", sampling=sampling))
    asyncio.run(adapter.generate("Xq", sampling=sampling))
    native = engine.calls[0][1]
    assert native.stop_table is not None and native.stop_token_sequences == ()
    assert engine.calls[1][1].stop_table is native.stop_table  # cached per stop set
    assert first.token_ids == (100, 99, 88, 98) and first.text == "dcX"  # ids kept, text cut at the stop
    assert first.outputs[0].stop_reason == "stop"


def test_prompt_rendering_and_prefill():
    config = InferenceEngineConfig(model_path="", apply_chat_template=True, assistant_prefill="A:")
    adapter, _ = make(config=config)
    assert adapter.tokenize_prompt("hi") == tuple(map(ord, "<user>hi</user><think=1>A:"))
    assert adapter.tokenize_prompt("hi", assistant_prefill="", chat_template_enable_thinking=False) == \
        tuple(map(ord, "<user>hi</user><think=0>"))
    assert adapter.tokenize_prompt([104, 105], assistant_prefill="!") == (104, 105, 33)
    echoed, text, ids = adapter._resolve_prompt({"prompt": "p", "prompt_token_ids": [1, 2]}, assistant_prefill="z")
    assert ids == (1, 2, 122) and text == "pz" and echoed == {"prompt": "pz", "prompt_token_ids": [1, 2, 122]}
    assert LFM25AsyncInferenceEngine.tokenize_for_config(config, CharTokenizer(), "q", assistant_prefill="") == \
        tuple(map(ord, "<user>q</user><think=1>"))
    assert adapter.supports_token_prompt_bridge()


def test_sampling_translation_and_validation():
    native = to_engine_sampling(SamplingConfig(temperature=0.5, top_k=-1, max_tokens=7, logprobs=1, stop=("ab",),
                                               extra_params={"ignore_eos": True, "repetition_penalty": 1.1}),
                                seed=5, tokenizer=CharTokenizer())
    assert native.top_k == 0 and native.max_new_tokens == 7 and native.return_logprobs and native.ignore_eos
    assert native.seed == 5 and native.repetition_penalty == 1.1
    assert native.stop_token_sequences == ((97, 98), (32, 97, 98), (10, 97, 98), (62, 97, 98))
    with pytest.raises(ValueError, match="n == 1"):
        to_engine_sampling(SamplingConfig(n=2), seed=0)
    with pytest.raises(ValueError, match="tokenizer"):
        to_engine_sampling(SamplingConfig(stop=("x",)), seed=0)
    assert sampling_bucket_key(SamplingConfig(max_tokens=3)) != sampling_bucket_key(SamplingConfig(max_tokens=4))
    assert [finish_reason_names(r) for r in (0, 1, 2, 3)] == [(None, None), ("stop", "eos"), ("stop", "stop"), ("length", None)]
    adapter, _ = make()
    with pytest.raises(TypeError, match="not a mapping"):
        adapter._resolve_sampling({"temperature": 1.0})
    duck = adapter._resolve_sampling(SimpleNamespace(temperature=0.3, max_new_tokens=9))
    assert duck.temperature == 0.3 and duck.max_tokens == 9 and duck.top_k == -1
    with pytest.raises(ValueError, match="positive integer"):
        make(max_batch_size=0)
    with pytest.raises(ValueError, match="cuda_graphs=True"):
        LFM25AsyncInferenceEngine(InferenceEngineConfig(model_path=""), fp8_kv=True)


def test_abort_cancels_a_queued_request_and_close_cancels_the_rest():
    adapter, engine = make(batch_wait_seconds=0.05)

    async def run():
        keep = asyncio.ensure_future(adapter.generate("ab", sampling=SamplingConfig(max_tokens=2), request_id="keep"))
        drop = asyncio.ensure_future(adapter.generate("cd", sampling=SamplingConfig(max_tokens=2), request_id="drop"))
        await asyncio.sleep(0)
        await adapter.abort_async("drop")
        result = await keep
        with pytest.raises(asyncio.CancelledError):
            await drop
        return result

    assert asyncio.run(run()).text == "ba" and engine.calls[0][0] == [[97, 98]]

    async def closing():
        queued = asyncio.ensure_future(adapter.generate("zz", sampling=SamplingConfig(max_tokens=2)))
        await asyncio.sleep(0)
        adapter.close()
        with pytest.raises(asyncio.CancelledError):
            await queued
        with pytest.raises(RuntimeError, match="closed"):
            await adapter.generate("again")

    asyncio.run(closing())
    assert engine.released == 0  # a caller-owned engine keeps its buffers
    with pytest.raises(RuntimeError, match="closed"):
        adapter.raw_engine


def test_weight_sync_waits_for_running_generation():
    adapter, engine = make()
    engine.block = threading.Event()
    order = []

    async def run():
        task = asyncio.ensure_future(adapter.generate("ab", sampling=SamplingConfig(max_tokens=2)))
        await asyncio.sleep(0.05)  # the batch now holds the engine lock inside generate()

        def sync():
            adapter.sync_from_model("policy-1")
            order.append("synced")

        thread = threading.Thread(target=sync)
        thread.start()
        await asyncio.sleep(0.05)
        assert order == [] and engine.synced == []
        with pytest.raises(TimeoutError, match="drain"):
            adapter.sync_from_model("policy-x", drain_timeout=0.01)
        engine.block.set()
        await task
        order.append("generated")
        thread.join(5)

    asyncio.run(run())
    assert engine.synced == ["policy-1"] and "synced" in order
    with pytest.raises(ValueError, match="finite"):
        adapter.sync_from_model("p", drain_timeout=float("inf"))
    adapter.sleep()
    assert engine.released == 1


def test_chains_resume_exact_extensions_and_readmit_everything_else():
    adapter, engine = make(max_batch_size=2)
    sampling = SamplingConfig(max_tokens=2, logprobs=1)
    plan = {0: ["extend", None], 1: ["restart", None], 2: [None]}
    seen = []

    def on_result(index, result):
        seen.append((index, result.request_id, result.text))
        step = plan[index].pop(0)
        if step == "extend":   # previous prompt + completion + new text: consumes only the new tokens
            return list(result.prompt_token_ids) + list(result.token_ids) + [ord("+")], sampling
        if step == "restart":  # unrelated prompt: fresh context in the same slot
            return "new", sampling
        return None

    chains = asyncio.run(adapter.generate_chains([("ab", sampling), ("cd", sampling), ("ef", sampling)],
                                                 on_result=on_result, max_new_tokens=2))
    assert [len(c) for c in chains] == [2, 2, 1]
    assert chains[0][0].text == "!b" and chains[0][1].request_id == "chain-0-phase-1"
    assert chains[0][1].prompt_token_ids == (97, 98, 33, 98, 43)
    log = engine.session_log
    kinds = [entry[0] for entry in log]
    assert kinds.count("resume") == 1 and ("resume", 0, (97, 98, 33, 98, 43)) == log[kinds.index("resume")][:3]
    assert ("release", 1) in log and ("admit", 1, (110, 101, 119)) in [e[:3] for e in log]  # "new" re-admitted in slot 1
    assert ("admit", 1, (101, 102)) in [e[:3] for e in log] or ("admit", 0, (101, 102)) in [e[:3] for e in log]
    seeds = [e[3] for e in log if e[0] in ("admit", "resume")]
    assert len(set(seeds)) == len(seeds)  # every (chain, phase) draws from its own stream
    assert adapter.last_session_stats["admitted_requests"] == 4 and log[-1] == ("closed",)
    assert asyncio.run(adapter.generate_chains([], on_result=on_result, max_new_tokens=2)) == []


def test_stop_token_sequence_automaton_matches_suffix_search():
    import random

    from climbing_gym_b200.text_stops import build_token_sequence_table

    patterns = [(5, 6, 7), (6, 8), (9,), (5, 5, 6)]
    table = build_token_sequence_table(patterns, 16)
    assert table.dtype == torch.int32 and table.shape[1] == 16
    rng = random.Random(0)
    for _ in range(500):
        history, state = [rng.choice([5, 6, 7, 8, 9, 1]) for _ in range(14)], 0
        for end, token in enumerate(history, 1):
            value = int(table[state, token])
            state = value & 65535
            want = any(len(p) <= end and tuple(history[end - len(p):end]) == p for p in patterns)
            assert (value >= 65536) == want, (history, end)
    with pytest.raises(ValueError, match="nonempty"):
        build_token_sequence_table([()], 16)
    with pytest.raises(ValueError, match="vocabulary"):
        build_token_sequence_table([(3, 99)], 16)


def test_product_of_two_stop_automata_matches_when_either_does():
    import random

    from climbing_gym_b200.text_stops import build_token_sequence_table, product_stop_table

    first = build_token_sequence_table([(1, 2, 3), (4, 4)], 8)
    second = build_token_sequence_table([(2, 3, 5), (7,)], 8)
    both = product_stop_table(first, second)
    assert both.dtype == torch.int32 and both.shape == (first.size(0) * second.size(0), 8)
    rng = random.Random(1)
    for _ in range(300):
        a = b = state = 0
        for token in (rng.randrange(8) for _ in range(12)):
            va, vb, value = int(first[a, token]), int(second[b, token]), int(both[state, token])
            a, b, state = va & 65535, vb & 65535, value & 65535
            assert state == a * second.size(0) + b
            assert (value >= 65536) == (va >= 65536 or vb >= 65536)
    with pytest.raises(ValueError, match="same vocabulary"):
        product_stop_table(first, build_token_sequence_table([(1,)], 9))


def test_graph_capture_holds_the_cyclic_collector():
    """decoder._quiet_collector: what is garbage is collected before a stream capture starts, the cyclic collector
    stays off while the capture runs (a CUDA graph destroyed by it in the middle of a capture invalidates the
    capture) and comes back afterwards, also when the capture raises."""
    import gc
    import weakref

    from climbing_gym_b200.decoder import _quiet_collector

    class Node:
        pass

    a, b = Node(), Node()
    a.other, b.other = b, a  # a cycle: only the cyclic collector frees it
    probe = weakref.ref(a)
    del a, b
    assert gc.isenabled()
    with _quiet_collector():
        assert probe() is None, "garbage is collected before the capture begins"
        assert not gc.isenabled()
    assert gc.isenabled()
    with pytest.raises(RuntimeError):
        with _quiet_collector():
            raise RuntimeError("capture failed")
    assert gc.isenabled()
    gc.disable()
    try:
        with _quiet_collector():
            pass
        assert not gc.isenabled(), "a collector that was off stays off"
    finally:
        gc.enable()
