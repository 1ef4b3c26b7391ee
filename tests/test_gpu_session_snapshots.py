"""Session prefix snapshots (prefill_snapshot / snapshot / fork / release_snapshot): children of a
snapshot must generate exactly what the same request generates when it is admitted (or resumed) the
ordinary way, while holding the prefix's full pages by reference."""
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


def make_engine(dev, dtype=torch.float32, **options):
    from climbing_gym_b200.engine import LFM25Engine

    cfg = synthetic.tiny_config()
    state = synthetic.make_state_dict(cfg, seed=0, untied_head=True)
    engine = LFM25Engine.from_state_dict(cfg, {k: torch.from_numpy(v) for k, v in state.items()}, device=dev,
                                         dtype=dtype, max_model_len=512)
    engine.enable_cuda_graphs(max_graphs=2, **options)
    return engine


def sampling(seed, n=10, temperature=1.0):
    return LFM25SamplingConfig(temperature=temperature, max_new_tokens=n, seed=seed, ignore_eos=True)


def drain(session, slot_ids):
    """Poll until every slot in slot_ids finished; {slot: result} (nothing is released)."""
    done = {}
    while len(done) < len(slot_ids):
        for result in session.poll(steps=4):
            done[result.handle.slot] = result
    return done


def test_children_of_a_prefilled_snapshot_match_admitted_requests(dev):
    engine = make_engine(dev)
    prompt = synthetic.uniform_prompts(1, 150, 150, 4096, seed=21)[0]  # two full pages and a 22-token tail
    seeds = [3, 4, 5]
    with engine.generation_session(max_batch_size=4, max_new_tokens=10) as session:
        slots = session.admit([prompt] * 3, [sampling(s) for s in seeds])
        plain = drain(session, slots)
    with engine.generation_session(max_batch_size=4, max_new_tokens=10) as session:
        pages = session.cache.n_pages
        snap = session.prefill_snapshot(prompt)
        assert snap.prefix_token_ids == tuple(prompt) and session.cache.free_pages() == pages - 3
        slots = session.fork(snap, [sampling(s) for s in seeds], slots=[3, 0, 2])
        assert slots == [3, 0, 2]
        # snapshot + 3 children share the 2 full pages; each child owns a tail page
        assert int(session.cache.refcount.max()) == 4 and session.cache.free_pages() == pages - 3 - 3
        forked = drain(session, slots)
        for slot, plain_slot in zip(slots, (0, 1, 2)):
            assert forked[slot].token_ids == plain[plain_slot].token_ids
            assert np.allclose(forked[slot].logprobs, plain[plain_slot].logprobs, atol=1e-5)
            assert forked[slot].prompt_token_ids == tuple(prompt)
        stats = session.stats
        assert stats["forked_requests"] == 3 and stats["snapshot_count"] == 1 and stats["peak_snapshots"] == 1
        assert stats["snapshot_prefilled_tokens"] == 150 and stats["copied_prefix_tokens"] == 3 * (150 % 64)
        assert stats["peak_snapshot_bytes"] > 0
        # the snapshot outlives its children and can be forked again
        for result in forked.values():
            session.release(result.handle)
        assert session.cache.free_pages() == pages - 3
        again = session.fork(snap, [sampling(seeds[0])])
        assert drain(session, again)[again[0]].token_ids == plain[0].token_ids
        session.release_snapshot(snap)
        with pytest.raises(ValueError, match="released"):
            session.fork(snap, [sampling(1)])
        with pytest.raises(ValueError, match="released"):
            session.release_snapshot(snap)


def test_snapshot_of_a_finished_request_continues_like_resume(dev):
    engine = make_engine(dev)
    prompt = synthetic.uniform_prompts(1, 70, 70, 4096, seed=22)[0]
    with engine.generation_session(max_batch_size=3, max_new_tokens=12) as session:
        pages = session.cache.n_pages
        slot = session.admit([prompt], [sampling(9, n=6)])[0]
        first = drain(session, [slot])[slot]
        prefix = first.handle.prefix_token_ids
        assert len(prefix) == 76
        snap = session.snapshot(first.handle)
        assert snap.prefix_token_ids == prefix
        children = session.fork(snap, [sampling(31, n=12), sampling(32, n=12)])
        session.resume([first.handle], [prefix], [sampling(31, n=12)])
        done = drain(session, [slot, *children])
        assert done[children[0]].token_ids == done[slot].token_ids, "same context, seed and RNG position"
        assert np.allclose(done[children[0]].logprobs, done[slot].logprobs, atol=1e-5)
        assert done[children[1]].token_ids != done[children[0]].token_ids
        assert done[children[0]].prompt_token_ids == prefix
        with pytest.raises(ValueError, match="distinct free"):
            session.fork(snap, [sampling(1)], slots=[slot])
        for result in done.values():
            session.release(result.handle)
        session.release_snapshot(snap)
        assert session.cache.free_pages() == pages
    with engine.generation_session(max_batch_size=3, max_new_tokens=12) as other:
        with pytest.raises(ValueError, match="another session"):
            other.fork(snap, [sampling(1)])


def test_snapshot_rows_are_bounded_and_returned_on_close(dev):
    engine = make_engine(dev, dtype=torch.bfloat16, fp8_kv=True, snapshot_rows=1)
    prompts = synthetic.uniform_prompts(2, 40, 90, 4096, seed=23)
    with engine.generation_session(max_batch_size=2, max_new_tokens=8) as session:
        pages = session.cache.n_pages
        snap = session.prefill_snapshot(prompts[0])
        with pytest.raises(RuntimeError, match="snapshot row"):
            session.prefill_snapshot(prompts[1])
        slots = session.fork(snap, [sampling(0, n=8, temperature=0.0)] * 2)
        done = drain(session, slots)
        assert done[slots[0]].token_ids == done[slots[1]].token_ids, "greedy children of one e4m3 prefix agree"
        for result in done.values():
            session.release(result.handle)
        session.release_snapshot(snap)
        assert session.cache.free_pages() == pages
        other = session.prefill_snapshot(prompts[1])
        assert other.identity != snap.identity
    # closing the session gave every page back, the parked prefix included
    assert session.cache.free_pages() == pages
