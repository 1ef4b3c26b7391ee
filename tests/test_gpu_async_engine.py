"""The asyncio adapter over the real CUDA engine (its host logic is covered against fakes on CPU in
tests/test_async_engine.py): coalesced ``generate_many``, multi-phase ``generate_chains`` with resume,
fresh-context re-admission and refill, clean-up when the callback raises, and cancellation that drains the
worker. Follows the reference's tests of the same behaviours (tests/test_lfm25_session.py:192-261)."""
import asyncio

import pytest
import torch

from climbing_gym_b200 import synthetic
from climbing_gym_b200.async_engine import LFM25AsyncInferenceEngine
from climbing_gym_b200.config import LFM25SamplingConfig, SamplingConfig

pytestmark = pytest.mark.gpu


class IdTokenizer:
    """Token ids are their own text: "12 7 " <-> [12, 7] (enough for the adapter's decode / echo)."""

    def encode(self, text, add_special_tokens=False):
        return [int(t) for t in text.split()]

    def __len__(self):
        return 4096

    def decode(self, ids, skip_special_tokens=False, clean_up_tokenization_spaces=False):
        return "".join(f"{int(i)} " for i in ids)


def make_engine(fp8_kv=False):
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    from climbing_gym_b200.engine import LFM25Engine

    dev = torch.device("cuda:0")
    cfg = synthetic.tiny_config()
    state = synthetic.make_state_dict(cfg, seed=0, untied_head=True)
    raw = LFM25Engine.from_state_dict(cfg, {k: torch.from_numpy(v) for k, v in state.items()}, device=dev,
                                      dtype=torch.bfloat16 if fp8_kv else torch.float32, max_model_len=256)
    raw.enable_cuda_graphs(max_graphs=1, fp8_kv=fp8_kv)
    return raw


def test_generate_many_coalesces_requests_and_matches_the_engine():
    raw = make_engine()
    engine = LFM25AsyncInferenceEngine.from_components(engine=raw, tokenizer=IdTokenizer(), max_batch_size=4)
    sampling = SamplingConfig(temperature=0, max_tokens=6, logprobs=1, extra_params={"ignore_eos": True})
    prompts = [[1, 2 + i, 9] for i in range(6)]
    results = asyncio.run(engine.generate_many(prompts, sampling=sampling))
    assert len(results) == 6 and all(r.finished and len(r.outputs[0].token_ids) == 6 for r in results)
    from climbing_gym_b200.engine import flatten_token_batches

    direct = raw.generate(*flatten_token_batches(prompts, device=raw.device), repeats=1,
                          sampling=LFM25SamplingConfig(temperature=0.0, max_new_tokens=6, ignore_eos=True))
    for row, result in enumerate(results):
        assert list(result.outputs[0].token_ids) == direct.token_ids[row, 0].tolist()
        assert result.outputs[0].text == IdTokenizer().decode(result.outputs[0].token_ids)
        assert len(result.outputs[0].completion_logprobs) == 6
    engine.close()
    assert raw._cuda_decoder is not None, "a caller-owned engine outlives the adapter"


@pytest.mark.parametrize("fp8_kv", [False, True])
def test_chains_resume_refill_fresh_context_and_clean_up_on_callback_error(fp8_kv):
    raw = make_engine(fp8_kv)
    engine = LFM25AsyncInferenceEngine.from_components(engine=raw, tokenizer=IdTokenizer(), max_batch_size=2)
    sampling = SamplingConfig(temperature=0, max_tokens=3, logprobs=1, extra_params={"ignore_eos": True})
    requests = [([1, 2 + i], sampling) for i in range(5)]
    phases = [0] * 5

    def advance(index, result):
        assert result.finished and len(result.outputs[0].completion_logprobs) == 3
        phases[index] += 1
        if phases[index] == 1:  # extends the cached tokens: resumed in place
            return tuple(result.prompt_token_ids) + tuple(result.outputs[0].token_ids) + (40,), sampling
        if phases[index] == 2:  # unrelated prompt: the slot is released and re-admitted
            return [1, 30 + index], sampling
        return None

    results = asyncio.run(engine.generate_chains(requests, on_result=advance, max_new_tokens=3, poll_interval=2))
    assert [len(chain) for chain in results] == [3] * 5
    stats = engine.last_session_stats
    assert stats["resumed_requests"] == 5 and stats["admitted_requests"] == 10 and stats["prefilled_tokens"] == 20
    assert raw._cuda_decoder._active_session is None

    def fail(*_):
        raise ValueError("callback failed")

    with pytest.raises(ValueError, match="callback failed"):
        asyncio.run(engine.generate_chains(requests, on_result=fail, max_new_tokens=3))
    assert raw._cuda_decoder._active_session is None
    assert engine._engine_lock.acquire(blocking=False)
    engine._engine_lock.release()


def test_chain_cancellation_drains_the_worker_and_the_cache_lease():
    raw = make_engine()
    engine = LFM25AsyncInferenceEngine.from_components(engine=raw, tokenizer=IdTokenizer(), max_batch_size=2)
    sampling = SamplingConfig(max_tokens=1, extra_params={"ignore_eos": True})

    async def run():
        loop = asyncio.get_running_loop()
        task = None
        requested = False

        def advance(index, result):
            nonlocal requested
            if not requested:
                requested = True
                loop.call_soon_threadsafe(task.cancel)
            return [1, 7], sampling

        task = asyncio.create_task(engine.generate_chains([([1, 2], sampling)], on_result=advance, max_new_tokens=1,
                                                          poll_interval=1))
        with pytest.raises(asyncio.CancelledError):
            await task
        assert raw._cuda_decoder._active_session is None
        assert engine._engine_lock.acquire(blocking=False)
        engine._engine_lock.release()

    asyncio.run(run())
