"""Top-k / top-p sampling: the threshold kernel against a numpy restatement of the reference's
`_apply_top_k_top_p` (src/climbing_gym/inference/lfm25_engine.py:1759-1775), the sampler drawing only
from the surviving support, and the engine-level identities (top_k = 1 and a vanishing top_p are
greedy decoding)."""
import ctypes as C

import numpy as np
import pytest
import torch

from climbing_gym_b200 import synthetic
from climbing_gym_b200.config import LFM25SamplingConfig
from oracle.numerics import round_bf16

pytestmark = pytest.mark.gpu

nv = pytest.importorskip("climbing_gym_b200._native")


@pytest.fixture(scope="module")
def dev():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    nv.load()
    return torch.device("cuda:0")


def reference_support(logits, temperature, top_k, top_p):
    """Boolean mask of the values the reference keeps (rows of distinct values, so that its sort order
    is unambiguous): top-k by value threshold, then top-p on the tempered softmax of the survivors,
    dropping every sorted position whose inclusive cumulative probability exceeds top_p except the first."""
    keep = np.ones(logits.shape, bool)
    for r, row in enumerate(logits.astype(np.float64)):
        scaled = row / temperature[r]
        if 0 < top_k[r] < row.size:
            keep[r] &= scaled >= np.sort(scaled)[-top_k[r]]
        if top_p[r] < 1.0:
            order = np.argsort(-np.where(keep[r], scaled, -np.inf), kind="stable")
            kept_scaled = np.where(keep[r], scaled, -np.inf)[order]
            probs = np.exp(kept_scaled - kept_scaled[0])
            cumulative = np.cumsum(probs / probs.sum())
            remove = cumulative > top_p[r]
            remove[0] = False
            keep[r, order[remove]] = False
    return keep


def distinct_logits(rng, rows, vocab, scale, bf16):
    if not bf16:
        return (rng.standard_normal((rows, vocab)) * scale).astype(np.float32)
    # bf16 has few values per binade: build rows out of distinct representable values
    grid = np.unique(round_bf16(np.linspace(-8.0, 8.0, 20 * vocab).astype(np.float32)))
    return np.stack([rng.permutation(rng.choice(grid, size=vocab, replace=False)) for _ in range(rows)]).astype(np.float32)


@pytest.mark.parametrize("bf16,vocab", [(False, 4096), (True, 1024), (True, 65536)])
def test_thresholds_reproduce_the_reference_support(dev, bf16, vocab):
    rng = np.random.default_rng(vocab + bf16)
    rows = 12
    if bf16 and vocab > 1024:  # not enough distinct bf16 values for 65536 distinct logits: rows with ties
        logits_np = round_bf16(rng.standard_normal((rows, vocab)) * 3.0)
    else:
        logits_np = distinct_logits(rng, rows, vocab, 2.5, bf16)
    temperature = np.array([1.0, 0.7, 1.3, 1.0, 0.5, 2.0, 1.0, 1.0, 0.9, 1.0, 0.0, 1.0], np.float32)
    top_k = np.array([50, 0, 5, 1, 0, 200, vocab, 0, 17, 3, 10, 0], np.int32)
    top_p = np.array([1.0, 0.9, 0.5, 1.0, 0.999, 0.3, 0.8, 1e-6, 0.95, 1.0, 0.5, 1.0], np.float32)
    alive = np.ones(rows, np.uint8)
    alive[9] = 0
    logits = torch.from_numpy(logits_np).to(dev)
    if bf16:
        logits = logits.to(torch.bfloat16)
    out = torch.full((rows,), 123.0, device=dev)
    args = [torch.from_numpy(a).to(dev) for a in (temperature, top_k, top_p, alive)]
    nv.call("cgym_filter_thresholds", nv.ptr(out), nv.ptr(logits), nv.ptr(args[0]), nv.ptr(args[1]), nv.ptr(args[2]),
            nv.ptr(args[3]), rows, vocab, nv.BF16 if bf16 else nv.F32, nv.stream_ptr())
    thresholds = out.cpu().numpy()
    assert np.isneginf(thresholds[[9, 10, 11]]).all()  # dead row, greedy row, row without a filter
    ties = bf16 and vocab > 1024
    live = [r for r in range(rows) if r not in (9, 10, 11)]
    want = reference_support(logits_np[live], temperature[live], top_k[live], top_p[live])
    for i, r in enumerate(live):
        got = logits_np[r] >= thresholds[r]
        assert got[np.argmax(logits_np[r])], "the most probable value always stays"
        if not ties:
            # top-k is exact; the top-p cut compares fp32 sums of exponentials with top_p, so the element
            # sitting exactly at the cut may fall on either side of a float64 restatement
            limit = 0 if top_p[r] >= 1.0 else 1
            assert (got != want[i]).sum() <= limit, (r, int(got.sum()), int(want[i].sum()))
        else:
            # with tied values the kernel keeps or drops a tie group as a whole: the two supports may
            # differ only in elements equal to a boundary value
            boundary = set(np.unique(logits_np[r][got != want[i]]).tolist())
            assert len(boundary) <= 2, (r, boundary)
            if top_k[r] and top_p[r] >= 1.0:
                assert got.sum() >= min(top_k[r], vocab)


def test_sampler_draws_only_from_the_filtered_support_with_renormalised_frequencies(dev):
    from climbing_gym_b200.decoder import SlotState

    rows, vocab, cap = 8192, 64, 1
    rng = np.random.default_rng(5)
    base = np.sort(rng.standard_normal(vocab).astype(np.float32) * 2.0)[::-1].copy()
    logits = torch.from_numpy(np.tile(base, (rows, 1))).to(dev)
    seq_lens = torch.zeros(rows, device=dev, dtype=torch.int32)
    st = SlotState(rows, cap, vocab, 2, seq_lens, stop_states=2)
    st.limits.fill_(1)
    st.alive.fill_(1)
    st.ignore_eos.fill_(1)
    st.temperatures.fill_(0.8)
    st.seeds.copy_(torch.arange(rows) * 7919 + 3)
    st.top_k.fill_(10)
    st.top_p.fill_(0.85)
    nv.call("cgym_filter_thresholds", nv.ptr(st.min_logits), nv.ptr(logits), nv.ptr(st.temperatures), nv.ptr(st.top_k),
            nv.ptr(st.top_p), nv.ptr(st.alive), rows, vocab, nv.F32, nv.stream_ptr())
    nv.call("cgym_sample_record", nv.ptr(logits), C.byref(st.struct_filtered), None, None, None, rows, vocab, nv.F32,
            nv.ptr(st.sample_ws), nv.stream_ptr())
    torch.cuda.synchronize()
    keep = reference_support(base[None], np.array([0.8]), np.array([10]), np.array([0.85]))[0]
    assert 1 < keep.sum() <= 10
    tokens = st.tokens.cpu().numpy()[:, 0]
    assert keep[tokens].all(), "a token outside the support was drawn"
    probs = np.where(keep, np.exp((base - base.max()) / 0.8), 0.0)
    probs /= probs.sum()
    counts = np.bincount(tokens, minlength=vocab) / rows
    assert np.abs(counts - probs).max() < 0.025  # 8192 draws: > 4 sigma of the largest bin
    # the recorded log-prob stays the raw, untempered, unfiltered one
    raw = base - (base.max() + np.log(np.exp(base - base.max()).sum()))
    assert np.allclose(st.logprobs.cpu().numpy()[:, 0], raw[tokens], atol=3e-6)


def make_engine(dev):
    from climbing_gym_b200.engine import LFM25Engine

    cfg = synthetic.tiny_config()
    state = synthetic.make_state_dict(cfg, seed=0, untied_head=True)
    engine = LFM25Engine.from_state_dict(cfg, {k: torch.from_numpy(v) for k, v in state.items()}, device=dev,
                                         dtype=torch.float32, max_model_len=256)
    engine.enable_cuda_graphs(max_graphs=4)
    return engine


def test_degenerate_filters_are_greedy_decoding_and_filtered_runs_are_reproducible(dev):
    from climbing_gym_b200.engine import flatten_token_batches

    engine = make_engine(dev)
    prompts = synthetic.uniform_prompts(6, 8, 40, 4096, seed=1)
    flat = flatten_token_batches(prompts, device=dev)

    def run(**kw):
        out = engine.generate(*flat, repeats=1, sampling=LFM25SamplingConfig(max_new_tokens=12, seed=9, **kw))
        return out.token_ids.cpu().numpy()[:, 0], out.logprobs.cpu().numpy()[:, 0]

    greedy, greedy_lp = run(temperature=0.0)
    for kw in (dict(temperature=1.0, top_k=1), dict(temperature=0.7, top_p=1e-7)):
        tokens, lp = run(**kw)
        assert np.array_equal(tokens, greedy), kw
        assert np.allclose(lp, greedy_lp, atol=1e-5)
    a, _ = run(temperature=1.0, top_k=40, top_p=0.9)
    b, _ = run(temperature=1.0, top_k=40, top_p=0.9)
    full, _ = run(temperature=1.0)
    assert np.array_equal(a, b) and not np.array_equal(a, full)
