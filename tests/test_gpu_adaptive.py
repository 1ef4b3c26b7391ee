"""Adaptive batching (compact decode graphs over the shared paged cache) and the decode-graph cache.

Follows the reference's own tests of this behaviour (tests/test_lfm25_adaptive.py:63-167,
tests/test_lfm25_cuda.py:368-396): a session whose live rows fit a smaller bucket (16 * 2^k) replays a
graph of that many rows that reaches the requests through a slot table, requests keep their state across
graph changes, batch generation shrinks its compute batch as rows stop, results do not depend on the
bucket, and the graph cache evicts least-recently-used entries and rounds capacities.
"""
from dataclasses import replace

import numpy as np
import pytest
import torch

from climbing_gym_b200 import synthetic
from climbing_gym_b200.config import LFM25SamplingConfig

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def dev():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    return torch.device("cuda:0")


def make_engine(dev, dtype, **options):
    from climbing_gym_b200.engine import LFM25Engine

    cfg = synthetic.tiny_config()
    state = synthetic.make_state_dict(cfg, seed=0, untied_head=True)
    engine = LFM25Engine.from_state_dict(cfg, {k: torch.from_numpy(v) for k, v in state.items()}, device=dev,
                                         dtype=dtype, max_model_len=256)
    engine.enable_cuda_graphs(**options)
    return engine


def flat(prompts, dev):
    from climbing_gym_b200.engine import flatten_token_batches

    return flatten_token_batches(prompts, device=dev)


def run_sparse_session(engine, prompts, samplings, slots, *, steps):
    done = {}
    with engine.generation_session(max_batch_size=32, max_new_tokens=24, cache_len=128) as session:
        session.admit(prompts, samplings, slots=slots)
        for _ in range(40):
            for result in session.poll(steps=steps):
                done[result.handle.slot] = result
                session.release(result.handle)
            if len(done) == len(prompts):
                break
        stats = dict(session.stats)
        compact = dict(session.entry.compact_graphs)
        assert session.poll(steps=1) == []
        assert session.cache.free_pages() == session.cache.n_pages
    return done, stats, compact


@pytest.mark.parametrize("dtype,fp8_kv", [(torch.float32, False), (torch.bfloat16, False), (torch.bfloat16, True)])
def test_sparse_session_runs_in_the_16_row_bucket_with_identical_results(dev, dtype, fp8_kv):
    prompts = synthetic.uniform_prompts(4, 5, 40, 4096, seed=31)
    sample = LFM25SamplingConfig(temperature=0.8, max_new_tokens=20, ignore_eos=True, seed=91)
    samplings = [replace(sample, max_new_tokens=n, seed=91 + i) for i, n in enumerate((2, 7, 20, 20))]
    slots = [0, 8, 17, 31]
    full, full_stats, _ = run_sparse_session(make_engine(dev, dtype, max_graphs=1, fp8_kv=fp8_kv), prompts, samplings,
                                             slots, steps=3)
    sparse, stats, compact = run_sparse_session(
        make_engine(dev, dtype, max_graphs=1, fp8_kv=fp8_kv, adaptive_batching=True), prompts, samplings, slots, steps=3)
    assert list(compact) == [16] and stats["adaptive_graph_captures"] == 1
    assert stats["decode_batches"] == {"16": stats["decode_steps"]}
    assert full_stats["decode_batches"] == {"32": full_stats["decode_steps"]}
    assert stats["decode_row_steps"] < stats["reserved_row_steps"] == full_stats["decode_row_steps"]
    for slot, sampling in zip(slots, samplings):
        assert len(sparse[slot].token_ids) == sampling.max_new_tokens and sparse[slot].finish_reason == 3
        if dtype == torch.float32:
            # CUDA-core GEMMs accumulate in a fixed order whatever the grid: the bucket changes nothing
            assert sparse[slot].token_ids == full[slot].token_ids
            assert np.allclose(sparse[slot].logprobs, full[slot].logprobs, atol=1e-5)
        else:
            # 16-row and 32-row steps share the 32-token GEMM tile; a differing split-K choice may move a
            # log-prob by a bf16 rounding, never a request's identity
            same = sum(a == b for a, b in zip(sparse[slot].token_ids, full[slot].token_ids))
            assert same >= len(full[slot].token_ids) - 1
            n = next((i for i, (a, b) in enumerate(zip(sparse[slot].token_ids, full[slot].token_ids)) if a != b),
                     len(full[slot].token_ids))
            assert np.allclose(sparse[slot].logprobs[:n], full[slot].logprobs[:n], atol=5e-2 if fp8_kv else 2e-2)


def test_requests_keep_their_state_across_resume_refill_and_graph_changes(dev):
    engine = make_engine(dev, torch.float32, max_graphs=1, adaptive_batching=True)
    sample = LFM25SamplingConfig(temperature=0.8, max_new_tokens=20, ignore_eos=True, seed=91)
    with engine.generation_session(max_batch_size=32, max_new_tokens=20, cache_len=128) as session:
        session.admit([[1, 4], [1, 8], [1, 17], [1, 31]],
                      [replace(sample, max_new_tokens=2), replace(sample, max_new_tokens=7), sample, sample],
                      slots=[0, 8, 17, 31])
        first = session.poll(steps=2)[0]
        assert first.handle.slot == 0
        graph = session.entry.compact_graphs[16].graph
        peers = session.cache.conv_state[:, [8, 17, 31]].clone()
        lengths = session.cache.seq_lens[[8, 17, 31]].clone()
        session.resume([first.handle], [first.handle.prefix_token_ids + (40, 41)], [replace(sample, max_new_tokens=3)])
        assert torch.equal(session.cache.conv_state[:, [8, 17, 31]], peers)
        assert torch.equal(session.cache.seq_lens[[8, 17, 31]], lengths)
        resumed = session.poll(steps=3)[0]
        assert resumed.handle.slot == 0 and len(resumed.token_ids) == 3
        session.release(resumed.handle)
        session.admit([[1, 22, 23]], [replace(sample, max_new_tokens=4)], slots=[0])
        results = []
        for _ in range(12):
            results.extend(session.poll(steps=3))
            if len(results) == 4:
                break
        assert len(results) == 4
        assert session.entry.compact_graphs[16].graph is graph, "the bucket's graph is captured once"
        assert session.stats["slot_refills"] == 1 and session.stats["adaptive_graph_captures"] == 1
        assert session.stats["decode_row_steps"] < session.stats["reserved_row_steps"]
        assert session.stats["decode_batches"] == {"16": session.stats["decode_steps"]}
        for result in results:
            session.release(result.handle)
        assert session.poll(steps=1) == []


def test_session_moves_to_a_smaller_bucket_when_most_rows_finish(dev):
    engine = make_engine(dev, torch.bfloat16, max_graphs=1, adaptive_batching=True, fp8_mlp=True, fp8_kv=True,
                         fp8_lm_head=True)
    prompts = [[1, 2 + i, 40 + i] for i in range(32)]
    sample = LFM25SamplingConfig(temperature=0.8, seed=91, max_new_tokens=65, ignore_eos=True)
    limits = [1] * 24 + [65] * 8
    samplings = [replace(sample, max_new_tokens=n, seed=91 + i) for i, n in enumerate(limits)]
    with engine.generation_session(max_batch_size=32, max_new_tokens=65, cache_len=128) as session:
        session.admit(prompts, samplings)
        outputs = []
        while len(outputs) < 32:
            outputs.extend(session.poll(steps=32))
        assert session.stats["decode_batches"] == {"32": 32, "16": 64}
    assert sorted(len(r.token_ids) for r in outputs) == sorted(limits)
    assert all(np.isfinite(r.logprobs).all() for r in outputs)


@pytest.mark.parametrize("fp8_kv", [False, True])
def test_direct_generation_shrinks_after_stops_and_preserves_greedy_results(dev, fp8_kv):
    engine = make_engine(dev, torch.float32 if not fp8_kv else torch.bfloat16, max_graphs=1, fp8_kv=fp8_kv)
    inputs = flat(synthetic.uniform_prompts(32, 3, 12, 4096, seed=77), dev)
    first = engine.generate(*inputs, repeats=1, sampling=LFM25SamplingConfig(temperature=0.0, max_new_tokens=1))
    first_tokens = first.token_ids[:, 0, 0].tolist()
    # the last three rows keep going; every row whose first token is not also one of theirs stops on it
    stops = tuple(sorted(set(first_tokens[:29]) - set(first_tokens[29:])))
    stopping = sum(token in stops for token in first_tokens)
    assert 16 <= stopping < 32, "the seeded prompts must leave between 1 and 16 rows alive after the first token"
    sampling = LFM25SamplingConfig(temperature=0.0, max_new_tokens=65, ignore_eos=True, stop_token_ids=stops)
    reference = engine.generate(*inputs, repeats=1, sampling=sampling)
    engine.enable_cuda_graphs(max_graphs=1, fp8_kv=fp8_kv, adaptive_batching=True)
    actual = engine.generate(*inputs, repeats=1, sampling=sampling)
    assert torch.equal(actual.lengths, reference.lengths)
    assert torch.equal(actual.finish_reasons, reference.finish_reasons)
    if not fp8_kv:
        assert torch.equal(actual.token_ids, reference.token_ids)
    else:
        assert float((actual.token_ids == reference.token_ids).float().mean()) > 0.95
    assert 16 in next(iter(engine._cuda_decoder.graphs.values())).compact_graphs


def test_graph_cache_rounds_capacities_and_evicts_least_recently_used(dev):
    engine = make_engine(dev, torch.bfloat16, max_graphs=1, max_prefill_tokens=128)
    decoder = engine._cuda_decoder
    prompts = [[1] + [row + 2] * (row % 10) for row in range(64)]
    sampling = LFM25SamplingConfig(temperature=0.0, max_new_tokens=20, ignore_eos=True)
    output = engine.generate(*flat(prompts, dev), repeats=1, sampling=sampling)
    assert output.token_ids.shape == (64, 1, 20)
    # 64 rows or more: capacities are multiples of 32 tokens in the reference, of one 64-token page here
    assert next(iter(decoder.graphs.values())).cache.max_seq_len == 64
    assert not decoder.packed_weights
    prompts[0] += [70] * 60
    engine.generate(*flat(prompts, dev), repeats=1, sampling=sampling)
    assert len(decoder.graphs) == 1, "max_graphs = 1: the smaller entry was evicted"
    assert next(iter(decoder.graphs.values())).cache.max_seq_len == 128
    # below 64 rows capacities are multiples of 128 tokens
    engine.generate(*flat([[1, 2, 3]] * 4, dev), repeats=1, sampling=sampling)
    assert list(decoder.graphs) == [(4, 128, False)]
    # two entries, least recently used goes first
    engine.enable_cuda_graphs(max_graphs=2)
    decoder = engine._cuda_decoder
    small, large = flat([[1, 2, 3]] * 4, dev), flat([[1, 2, 3]] * 8, dev)
    engine.generate(*small, repeats=1, sampling=sampling)
    engine.generate(*large, repeats=1, sampling=sampling)
    engine.generate(*small, repeats=1, sampling=sampling)      # refreshes the 4-row entry
    engine.generate(*flat([[1, 2, 3]] * 16, dev), repeats=1, sampling=sampling)
    assert [key[0] for key in decoder.graphs] == [4, 16]
    # same key, same entry and graph object; results repeat
    again = engine.generate(*small, repeats=1, sampling=sampling)
    entry = decoder.graphs[(4, 128, False)]
    repeat = engine.generate(*small, repeats=1, sampling=sampling)
    assert decoder.graphs[(4, 128, False)] is entry and torch.equal(again.token_ids, repeat.token_ids)
    engine.release_inference_buffers()
    assert not decoder.graphs and not decoder.fp8_weights


def test_single_request_graphs_stream_packed_weights_and_drop_them_with_the_graph(dev):
    """Batch-1 decode reads the vocabulary head and the MLP matrices through the lossless 12-bit stream; the
    copies follow a policy sync in place and are released when no batch-1 graph survives (reference:
    tests/test_lfm25_cuda.py:256-275, 383-396)."""
    engine = make_engine(dev, torch.bfloat16, max_graphs=1, max_prefill_tokens=128)
    decoder = engine._cuda_decoder
    sampling = LFM25SamplingConfig(temperature=0.0, max_new_tokens=6, ignore_eos=True)
    one = flat([[1, 2, 3]], dev)
    original = engine.generate(*one, repeats=1, sampling=sampling)
    assert decoder.packed_weights, "a batch-1 graph prepares the packed copies"
    n_layers = len(engine.weights.layers)
    assert len(decoder.packed_weights) == 2 * n_layers + 1
    plain = make_engine(dev, torch.bfloat16, max_graphs=1, bf16_weight_packing=False)
    unpacked = plain.generate(*one, repeats=1, sampling=sampling)
    assert not plain._cuda_decoder.packed_weights
    # lossless weights: only the summation order differs from the tensor-core GEMM
    assert float((original.logprobs - unpacked.logprobs).abs().max()) <= 2e-2
    assert float((original.token_ids == unpacked.token_ids).float().mean()) >= 0.8
    addresses = [p.mantissa.data_ptr() for p in decoder.packed_weights.values()]
    cfg = synthetic.tiny_config()

    class Model:
        config = cfg

        def state_dict(self):
            return {k: torch.from_numpy(v) for k, v in synthetic.make_state_dict(cfg, seed=1, untied_head=True).items()}

    engine.sync_from_model(Model())
    assert addresses == [p.mantissa.data_ptr() for p in decoder.packed_weights.values()]
    for packed in decoder.packed_weights.values():
        assert torch.equal(packed.unpack().view(torch.int16), packed.original.view(torch.int16))
    synced = engine.generate(*one, repeats=1, sampling=sampling)
    assert not torch.equal(synced.token_ids, original.token_ids)
    engine.generate(*flat([[1, 2, 3]] * 64, dev), repeats=1, sampling=sampling)
    assert not decoder.packed_weights, "the 64-row graph evicted the only batch-1 graph"
    repeated = engine.generate(*one, repeats=1, sampling=sampling)
    assert decoder.packed_weights and torch.equal(repeated.token_ids, synced.token_ids)
