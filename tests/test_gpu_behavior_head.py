"""Behaviour head (the k most probable tokens of the unfiltered distribution, recorded beside every
generated token): cgym_topk_head against the reference's own outputs (tests/golden/head.json), against
the oracle restatement on rows full of ties, and through `generate` and a generation session."""
import numpy as np
import pytest
import torch

from climbing_gym_b200 import synthetic
from climbing_gym_b200.config import LFM25SamplingConfig
from oracle import kernels as ok
from oracle.numerics import round_bf16

pytestmark = pytest.mark.gpu

nv = pytest.importorskip("climbing_gym_b200._native")


@pytest.fixture(scope="module")
def dev():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    nv.load()
    return torch.device("cuda:0")


def run_head(dev, logits, k, *, lengths=None, alive=None, capacity=1, dtype=torch.float32):
    rows, vocab = logits.shape
    x = torch.from_numpy(logits).to(dev).to(dtype).contiguous()
    ids = torch.full((rows, capacity, k), -7, device=dev, dtype=torch.int32)
    probs = torch.full((rows, capacity, k), 9.0, device=dev, dtype=torch.float32)
    lens = None if lengths is None else torch.tensor(lengths, device=dev, dtype=torch.int32)
    live = None if alive is None else torch.tensor(alive, device=dev, dtype=torch.uint8)
    nv.call("cgym_topk_head", nv.ptr(ids), nv.ptr(probs), nv.ptr(x), nv.ptr(live), nv.ptr(lens), rows, vocab, capacity,
            k, nv.dtype_code(dtype), nv.stream_ptr(dev))
    torch.cuda.synchronize(dev)
    return ids.cpu().numpy(), probs.cpu().numpy()


def exact_head(logits, k):
    """Oracle head with the partition function taken in float64 (selected token: the arg max)."""
    wide = logits.astype(np.float64)
    top = wide.max(1, keepdims=True)
    log_z = (top[:, 0] + np.log(np.exp(wide - top).sum(1)))
    return ok.behavior_head(logits, wide.argmax(1), (top[:, 0] - log_z).astype(np.float32), k)


def test_head_kernel_reproduces_reference_vectors(dev, golden):
    g = golden("head")
    logits = (np.random.default_rng(8).standard_normal((g["batch"], g["vocab"])) * 2.0).astype(np.float32)
    for case in g["heads"]:
        ids, probs = run_head(dev, logits, case["k"])
        assert ids[:, 0].tolist() == case["ids"], case["k"]
        # the reference takes log Z from its sampler's log-prob, the kernel from its own log-sum-exp
        assert np.allclose(probs[:, 0], case["logprobs"], atol=1e-5), case["k"]
    rec = g["record_head"]
    ids, probs = run_head(dev, logits, rec["k"], lengths=rec["lengths"], alive=rec["alive"], capacity=rec["capacity"])
    want_ids, want_probs = np.array(rec["ids"]), np.array(rec["logprobs"])
    written = np.zeros(ids.shape[:2], bool)
    for row, (length, live) in enumerate(zip(rec["lengths"], rec["alive"])):
        written[row, length] = live
    assert np.array_equal(ids[written], want_ids[written]) and np.allclose(probs[written], want_probs[written], atol=1e-5)
    assert (ids[~written] == -7).all() and (probs[~written] == 9.0).all(), "only [row, lengths[row]] of live rows is written"


@pytest.mark.parametrize("dtype,vocab", [(torch.float32, 4096), (torch.bfloat16, 4096), (torch.bfloat16, 65536),
                                         (torch.float32, 1000)])
@pytest.mark.parametrize("k", [1, 7, 128])
def test_head_kernel_orders_ties_by_lowest_id(dev, dtype, vocab, k):
    rng = np.random.default_rng(vocab + k)
    rows = 6
    logits = (rng.standard_normal((rows, vocab)) * 3.0).astype(np.float32)
    if dtype == torch.bfloat16:
        logits = round_bf16(logits)  # a few hundred distinct values: ties everywhere, also at the k-th place
    logits[1] = np.float32(0.5)                       # every logit equal: the head is ids 0..k-1
    logits[2, -k:] = logits[2].max() + np.float32(1)  # the winners at the very end of the row, all tied
    logits[3, : vocab // 2] = -np.inf                 # masked half
    want_ids, want_probs = exact_head(logits, k)
    ids, probs = run_head(dev, logits, k, dtype=dtype)
    assert np.array_equal(ids[:, 0], want_ids)
    assert np.allclose(probs[:, 0], want_probs, atol=2e-5)
    assert ids[1, 0].tolist() == list(range(k))


def test_head_kernel_rejects_bad_sizes(dev):
    logits = np.zeros((2, 64), np.float32)
    for k in (0, 65, 129):
        with pytest.raises(nv.NativeKernelError):
            run_head(dev, logits, k)


def make_engine(dev, dtype):
    from climbing_gym_b200.engine import LFM25Engine

    cfg = synthetic.tiny_config()
    state = synthetic.make_state_dict(cfg, seed=0, untied_head=True)
    state["model.lm_head.weight"] *= np.float32(12.0)  # a peaked next-token distribution: draws land in the head
    engine = LFM25Engine.from_state_dict(cfg, {k: torch.from_numpy(v) for k, v in state.items()}, device=dev,
                                         dtype=dtype, max_model_len=256)
    engine.enable_cuda_graphs(max_graphs=4)
    return engine


def check_heads(token_ids, logprobs, head_ids, head_probs):
    """The head belongs to the distribution the token was drawn from: descending, normalised below 1,
    and where the drawn token is in the head its log-prob there is the sampler's."""
    hits = 0
    for token, logp, ids, probs in zip(token_ids, logprobs, head_ids, head_probs):
        assert (np.diff(probs) <= 0).all() and np.exp(probs.astype(np.float64)).sum() <= 1.0 + 1e-5
        assert len(set(ids.tolist())) == len(ids)
        where = np.flatnonzero(ids == token)
        if where.size:
            hits += 1
            assert abs(probs[where[0]] - logp) < 2e-5
        else:
            assert logp <= probs[-1] + 2e-5, "a token outside the head cannot be more probable than its last entry"
    return hits


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_generate_returns_heads_without_changing_the_draw(dev, dtype):
    from climbing_gym_b200.engine import flatten_token_batches

    engine = make_engine(dev, dtype)
    prompts = synthetic.uniform_prompts(3, 5, 40, 4096, seed=3)
    flat = flatten_token_batches(prompts, device=dev)
    base = dict(temperature=1.0, max_new_tokens=20, seed=5, ignore_eos=True)
    plain = engine.generate(*flat, repeats=2, sampling=LFM25SamplingConfig(**base))
    out = engine.generate(*flat, repeats=2, sampling=LFM25SamplingConfig(behavior_topk=6, **base))
    assert plain.topk_token_ids is None and plain.topk_logprobs is None
    assert torch.equal(plain.token_ids, out.token_ids) and torch.equal(plain.logprobs, out.logprobs)
    assert out.topk_token_ids.shape == (3, 2, 20, 6) and out.topk_token_ids.dtype == torch.int32
    assert out.topk_logprobs.shape == (3, 2, 20, 6) and out.topk_logprobs.dtype == torch.float32
    hits = check_heads(out.token_ids.cpu().numpy().reshape(-1), out.logprobs.cpu().numpy().reshape(-1),
                       out.topk_token_ids.cpu().numpy().reshape(-1, 6), out.topk_logprobs.cpu().numpy().reshape(-1, 6))
    assert hits > 0
    # samples of one prompt draw their first token from the same prefill logits
    first = out.topk_token_ids[:, :, 0].cpu().numpy()
    assert (first[:, 0] == first[:, 1]).all()


def test_session_delivers_each_requests_own_head_width(dev):
    engine = make_engine(dev, torch.float32)
    prompts = synthetic.uniform_prompts(3, 5, 30, 4096, seed=4)
    widths, limits = [4, 0, 2], [9, 12, 5]
    with engine.generation_session(max_batch_size=2, max_new_tokens=12, behavior_topk=4) as session:
        with pytest.raises(ValueError, match="session reservation"):
            session.admit([prompts[0]], [LFM25SamplingConfig(temperature=1.0, max_new_tokens=4, behavior_topk=5)])
        waiting, slot_of, done = [0, 1, 2], {}, {}

        def admit(count):
            ids = [waiting.pop(0) for _ in range(count)]
            got = session.admit([prompts[i] for i in ids],
                                [LFM25SamplingConfig(temperature=1.0, max_new_tokens=limits[i], seed=40 + i,
                                                     ignore_eos=True, behavior_topk=widths[i]) for i in ids])
            slot_of.update(zip(got, ids))

        admit(2)
        while slot_of:
            for result in session.poll(steps=3):
                done[slot_of.pop(result.handle.slot)] = result
                session.release(result.handle)
                if waiting:
                    admit(1)
    for i, result in done.items():
        head = result.behavior_topk
        if not widths[i]:
            assert head is None
            continue
        assert head.token_ids.shape == (limits[i], widths[i]) and head.logprobs.shape == (limits[i], widths[i])
        assert not head.token_ids.is_cuda
        check_heads(np.array(result.token_ids), np.array(result.logprobs, np.float32), head.token_ids.numpy(),
                    head.logprobs.numpy())
    # request 2 reuses a slot: its head starts again at position 0 and matches a fresh session's
    with engine.generation_session(max_batch_size=1, max_new_tokens=12, behavior_topk=2) as session:
        session.admit([prompts[2]], [LFM25SamplingConfig(temperature=1.0, max_new_tokens=limits[2], seed=42,
                                                         ignore_eos=True, behavior_topk=2)])
        alone = []
        while not alone:
            alone = session.poll(steps=4)
    assert alone[0].token_ids == done[2].token_ids
    assert torch.equal(alone[0].behavior_topk.token_ids, done[2].behavior_topk.token_ids)
    assert torch.allclose(alone[0].behavior_topk.logprobs, done[2].behavior_topk.logprobs, atol=1e-6)
