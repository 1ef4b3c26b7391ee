"""The drop-in boundary, exercised with the reference's own engine object (the reference package staged
under oracle/_ref): ``bridge.install`` puts this package's decoder into ``LFM25Engine._cuda_decoder`` of a
reference engine built on the GPU, and the reference's own ``generate`` / ``sync_from_model`` /
``release_inference_buffers`` then run over it. The same reference engine, without a decoder, is the
reference's eager CUDA path: in fp32 the two must agree to 1e-4 on every token's log-prob.

Also here: the paged KV layout written from the description in include/cgym_b200.h alone (no library
call touches the page), read back through cgym_paged_attention."""
import sys

import numpy as np
import pytest
import torch

from climbing_gym_b200 import _native as nv
from climbing_gym_b200 import synthetic
from oracle.build_ref import staged_path
from oracle.numerics import round_bf16

pytestmark = pytest.mark.gpu

PROMPTS = synthetic.uniform_prompts(6, 8, 48, 4096, seed=0)


@pytest.fixture(scope="module")
def dev():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    return torch.device("cuda:0")


def stage_reference():
    staged = staged_path()
    if staged is None:
        pytest.skip("the reference package is not staged (python oracle/build_ref.py --reference <checkout>)")
    if str(staged) not in sys.path:
        sys.path.insert(0, str(staged))


def reference_engine(dev, dtype, seed=0):
    stage_reference()
    from climbing_gym.inference.lfm25_engine import LFM25Engine, LFM25PackedWeights
    from climbing_gym.models.lfm2 import LFM2Config

    cfg = synthetic.tiny_config()
    state = {k: torch.from_numpy(v) for k, v in synthetic.make_state_dict(cfg, seed=seed, untied_head=True).items()}
    rcfg = LFM2Config.from_dict({**cfg.to_dict(), "attn_backend": "eager"})
    weights = LFM25PackedWeights.from_state_dict(rcfg, state, device=dev, dtype=dtype)
    return LFM25Engine(weights, max_model_len=256), state


def test_decoder_installs_on_the_reference_engine_and_matches_its_eager_path(dev):
    stage_reference()
    from climbing_gym.inference.lfm25_engine import LFM25SamplingConfig, flatten_token_batches
    from climbing_gym_b200 import bridge

    engine, _ = reference_engine(dev, torch.float32)
    flat = flatten_token_batches(PROMPTS, device=dev)
    sampling = LFM25SamplingConfig(temperature=0.0, max_new_tokens=12, ignore_eos=True)
    eager = engine.generate(*flat, repeats=1, sampling=sampling)  # the reference's own eager CUDA path
    before = nv.launch_count()
    decoder = bridge.install(engine, max_graphs=1)
    assert engine._cuda_decoder is decoder
    assert decoder.engine.weights.layers[0].w13_weight.data_ptr() == engine.weights.layers[0].w13_weight.data_ptr()
    ours = engine.generate(*flat, repeats=1, sampling=sampling)  # the reference's method, this package's decoder
    assert nv.launch_count() > before, "the call went through this library's kernels"
    assert torch.equal(ours.token_ids, eager.token_ids) and torch.equal(ours.lengths, eager.lengths)
    assert torch.equal(ours.finish_reasons.to(eager.finish_reasons.dtype), eager.finish_reasons)
    assert float((ours.logprobs - eager.logprobs).abs().max()) <= 1e-4
    # repeats share prompt pages here; the reference copies: same outputs
    pair = engine.generate(*flatten_token_batches(PROMPTS[:3], device=dev), repeats=2, sampling=sampling)
    assert torch.equal(pair.token_ids[:, 0], pair.token_ids[:, 1]) and torch.equal(pair.token_ids[:, 0], eager.token_ids[:3, 0])
    # sessions come from this package once installed
    with engine.generation_session(max_batch_size=2, max_new_tokens=12, cache_len=128) as session:
        session.admit([PROMPTS[0], PROMPTS[1]], [sampling, sampling])
        results = {r.handle.slot: r for r in session.poll(steps=12)}
    assert list(results[0].token_ids) == eager.token_ids[0, 0].tolist()
    assert list(results[1].token_ids) == eager.token_ids[1, 0].tolist()
    # the reference's in-place weight sync reaches the decoder: same buffers, version bumped, new results
    cfg = synthetic.tiny_config()

    class Model:
        config = cfg

        def __init__(self, state):
            self._state = state

        def state_dict(self):
            return self._state

    fresh_state = {k: torch.from_numpy(v) for k, v in synthetic.make_state_dict(cfg, seed=1, untied_head=True).items()}
    address = engine.weights.layers[0].w13_weight.data_ptr()
    engine.sync_from_model(Model(fresh_state))
    assert engine.policy_version == 1 and decoder.engine.policy_version == 1
    assert engine.weights.layers[0].w13_weight.data_ptr() == address
    synced = engine.generate(*flat, repeats=1, sampling=sampling)
    assert not torch.equal(synced.token_ids, eager.token_ids)
    other, _ = reference_engine(dev, torch.float32, seed=1)
    want = other.generate(*flat, repeats=1, sampling=sampling)
    assert torch.equal(synced.token_ids, want.token_ids)
    assert float((synced.logprobs - want.logprobs).abs().max()) <= 1e-4
    engine.release_inference_buffers()
    assert not decoder.graphs
    bridge.uninstall(engine)
    assert engine._cuda_decoder is None
    again = engine.generate(*flat, repeats=1, sampling=sampling)  # eager path of the reference once more
    assert torch.equal(again.token_ids, want.token_ids)


def test_bf16_decoder_tracks_the_reference_eager_cuda_path(dev):
    stage_reference()
    from climbing_gym.inference.lfm25_engine import LFM25SamplingConfig, flatten_token_batches
    from climbing_gym_b200 import bridge

    engine, _ = reference_engine(dev, torch.bfloat16)
    flat = flatten_token_batches(PROMPTS, device=dev)
    sampling = LFM25SamplingConfig(temperature=0.0, max_new_tokens=12, ignore_eos=True)
    eager = engine.generate(*flat, repeats=1, sampling=sampling)
    bridge.install(engine, max_graphs=1)
    ours = engine.generate(*flat, repeats=1, sampling=sampling)
    tokens, ref = ours.token_ids[:, 0].cpu().numpy(), eager.token_ids[:, 0].cpu().numpy()
    for row in range(len(PROMPTS)):
        differs = np.nonzero(tokens[row] != ref[row])[0]
        stop = int(differs[0]) if len(differs) else tokens.shape[1]
        delta = (ours.logprobs[row, 0, :stop] - eager.logprobs[row, 0, :stop]).abs()
        assert float(delta.max()) <= 2e-2 if stop else True, (row, stop)
    assert np.mean(tokens == ref) > 0.7


def test_a_page_written_from_the_header_description_is_read_by_the_attention_kernel(dev):
    """K as [token][dim], V^T as [dim][token], 16-byte chunks of every row XOR-ed with the row index: computed
    here in numpy exactly as include/cgym_b200.h states it, stored with plain tensor writes."""
    from climbing_gym_b200.paged import PagedHybridCache

    rng = np.random.default_rng(3)
    hq, hkv, d, page = 8, 2, 64, 64
    lens = [150, 64, 1]
    cache = PagedHybridCache(n_attn_layers=1, n_conv_layers=1, n_slots=3, max_seq_len=192, n_kv_heads=hkv, head_dim=d,
                             hidden_size=64, dtype=torch.bfloat16, device=dev, page_size=page)
    e = 8  # bf16 elements per 16-byte chunk

    def swz(row, chunk, n):
        return chunk ^ (row & 7) if n >= 8 else chunk ^ ((row // (8 // n)) & (n - 1))

    pool = np.zeros(cache.kv_pool.shape, np.float32).reshape(-1)  # [layer][page][head][2 * P * D]
    table = np.full((3, cache.max_blocks), -1, np.int32)
    stored, next_page = [], 5  # pages handed out in an arbitrary order: the block table is the only link
    for slot, n in enumerate(lens):
        k, v = round_bf16(rng.standard_normal((n, hkv, d))), round_bf16(rng.standard_normal((n, hkv, d)))
        stored.append((k, v))
        for block in range(-(-n // page)):
            page_id = (next_page * 7) % cache.n_pages
            next_page += 1
            table[slot, block] = page_id
            for head in range(hkv):
                base = ((0 * cache.n_pages + page_id) * hkv + head) * (2 * page * d)
                for t in range(min(page, n - block * page)):
                    token = block * page + t
                    for dim in range(d):
                        pool[base + t * d + swz(t, dim // e, d // e) * e + dim % e] = k[token, head, dim]
                        pool[base + page * d + dim * page + swz(dim, t // e, page // e) * e + t % e] = v[token, head, dim]
    cache.kv_pool.copy_(torch.from_numpy(pool.reshape(cache.kv_pool.shape)).to(dev).to(torch.bfloat16))
    cache.block_table.copy_(torch.from_numpy(table).to(dev))
    q_np = round_bf16(rng.standard_normal((3, hq, d)))
    q = torch.from_numpy(q_np).to(dev).to(torch.bfloat16)
    out = torch.zeros((3, hq, d), device=dev, dtype=torch.bfloat16)
    kv_lens = torch.tensor(lens, device=dev, dtype=torch.int32)
    for impl in (1, 2):  # CUDA-core and tensor-core readers of the same layout
        nv.call("cgym_paged_attention", nv.ptr(out), nv.ptr(q), nv.ptr(kv_lens), None, None, cache.kv, 0, 3, hq,
                d ** -0.5, 1, None, nv.BF16, impl, nv.ptr(cache.status), nv.stream_ptr())
        got = out.float().cpu().numpy()
        assert int(cache.status.item()) == 0
        for row, n in enumerate(lens):
            k, v = stored[row]
            g = hq // hkv
            s = np.einsum("hgd,thd->hgt", q_np[row].reshape(hkv, g, d), k) * d ** -0.5
            p = np.exp(s - s.max(-1, keepdims=True))
            want = (np.einsum("hgt,thd->hgd", round_bf16(p), v) / p.sum(-1, keepdims=True)).reshape(hq, d)
            assert np.abs(got[row] - want).max() <= 0.012, (impl, row)
    # the library's own gather agrees with what was written
    k_back, v_back = cache.dense_kv(0, 0, 150)
    assert np.array_equal(k_back.cpu().numpy(), stored[0][0]) and np.array_equal(v_back.cpu().numpy(), stored[0][1])
