"""Repetition penalty on the fused path: cgym_repetition_penalty against the oracle's restatement of the
reference rule (bit-exact fp32), greedy generation against the reference's own outputs
(tests/golden/penalty.json) and sampled generation against the oracle's draws."""
import numpy as np
import pytest
import torch

from climbing_gym_b200 import synthetic
from climbing_gym_b200.config import LFM25SamplingConfig
from oracle import kernels as ok
from oracle.lfm25_oracle import OracleConfig, OracleEngine, OracleSampling
from oracle.numerics import round_bf16

pytestmark = pytest.mark.gpu

nv = pytest.importorskip("climbing_gym_b200._native")

PROMPTS = synthetic.uniform_prompts(8, 8, 64, 4096, seed=0)[:4]


@pytest.fixture(scope="module")
def dev():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    nv.load()
    return torch.device("cuda:0")


@pytest.mark.parametrize("dtype,vocab", [(torch.float32, 4096), (torch.bfloat16, 65536), (torch.float32, 1001)])
def test_penalty_kernel_is_bit_exact_and_marks_the_latest_token(dev, dtype, vocab):
    rng = np.random.default_rng(vocab)
    rows, capacity = 5, 6
    logits = (rng.standard_normal((rows, vocab)) * 2.0).astype(np.float32)
    if dtype == torch.bfloat16:
        logits = round_bf16(logits)
    seen = rng.random((rows, vocab)) < 0.2
    penalties = np.array([1.3, 0.8, 1.0, 2.0, 1.5], np.float32)
    lengths = np.array([0, 3, 6, 1, 2], np.int32)
    alive = np.array([1, 1, 1, 0, 1], np.uint8)
    tokens = rng.integers(0, vocab, size=(rows, capacity)).astype(np.int64)
    tokens[1, 2] = vocab - 1  # the last element of a row (ragged tail when vocab is not a multiple of 8)
    seen[1, vocab - 1] = False
    want_seen = seen.copy()
    want = logits.copy()
    for row in range(rows):
        if not alive[row]:
            continue
        if lengths[row] > 0:
            want_seen[row, tokens[row, lengths[row] - 1]] = True
        want[row] = ok.apply_repetition_penalty(logits[row], want_seen[row], float(penalties[row])) \
            if penalties[row] != 1.0 else logits[row]

    x = torch.from_numpy(logits).to(dev).to(dtype).contiguous()
    out = torch.full((rows, vocab), 77.0, device=dev, dtype=torch.float32)
    seen_dev = torch.from_numpy(seen.astype(np.uint8)).to(dev)
    args = [torch.from_numpy(a).to(dev) for a in (tokens, lengths, alive, penalties)]
    nv.call("cgym_repetition_penalty", nv.ptr(out), nv.ptr(x), nv.ptr(seen_dev), *(nv.ptr(a) for a in args), rows, vocab,
            capacity, nv.dtype_code(dtype), nv.stream_ptr(dev))
    torch.cuda.synchronize(dev)
    got = out.cpu().numpy()
    live = alive.astype(bool)
    assert np.array_equal(got[live].view(np.int32), want[live].view(np.int32))
    assert (got[~live] == 77.0).all(), "dead rows are left untouched"
    assert np.array_equal(seen_dev.cpu().numpy().astype(bool)[live], want_seen[live])
    assert np.array_equal(seen_dev.cpu().numpy().astype(bool)[~live], seen[~live])


def make_engine(dev, dtype):
    from climbing_gym_b200.engine import LFM25Engine

    cfg = synthetic.tiny_config()
    state = synthetic.make_state_dict(cfg, seed=0, untied_head=True)
    engine = LFM25Engine.from_state_dict(cfg, {k: torch.from_numpy(v) for k, v in state.items()}, device=dev,
                                         dtype=dtype, max_model_len=256)
    engine.enable_cuda_graphs(max_graphs=4)
    return engine


def make_oracle(dtype):
    cfg = synthetic.tiny_config()
    state = synthetic.make_state_dict(cfg, seed=0, untied_head=True)
    ocfg = OracleConfig(vocab_size=cfg.vocab_size, hidden_size=cfg.hidden_size, mlp_hidden_size=cfg.mlp_hidden_size,
                        num_attention_heads=cfg.num_attention_heads, num_key_value_heads=cfg.num_key_value_heads,
                        layer_types=tuple(cfg.layer_types), rope_theta=cfg.rope_theta, norm_eps=cfg.norm_eps,
                        conv_kernel_size=cfg.conv_kernel_size, eos_token_id=cfg.eos_token_id)
    return OracleEngine(ocfg, state, dtype=dtype, max_model_len=256)


def flat(dev):
    from climbing_gym_b200.engine import flatten_token_batches

    return flatten_token_batches(PROMPTS, device=dev)


@pytest.mark.parametrize("penalty", [1.3, 0.8])
def test_greedy_generate_with_penalty_reproduces_reference(dev, golden, penalty):
    want = golden("penalty")[f"generate_fp32_{penalty}"]
    engine = make_engine(dev, torch.float32)
    out = engine.generate(*flat(dev), repeats=2,
                          sampling=LFM25SamplingConfig(temperature=0.0, max_new_tokens=24, repetition_penalty=penalty,
                                                       ignore_eos=True))
    assert out.token_ids.cpu().tolist() == want["token_ids"]
    assert np.allclose(out.logprobs.cpu().numpy(), np.array(want["logprobs"]), atol=1e-4)
    # the plain entry is untouched by the penalised one
    plain = engine.generate(*flat(dev), repeats=2,
                            sampling=LFM25SamplingConfig(temperature=0.0, max_new_tokens=24, ignore_eos=True))
    assert plain.token_ids.cpu().tolist() != want["token_ids"]


def test_sampled_generate_with_penalty_matches_oracle_draws(dev):
    engine = make_engine(dev, torch.float32)
    config = dict(temperature=0.9, max_new_tokens=16, seed=321, ignore_eos=True, repetition_penalty=1.25)
    out = engine.generate(*flat(dev), repeats=2, sampling=LFM25SamplingConfig(**config))
    oracle = make_oracle("fp32").generate(PROMPTS, 2, OracleSampling(**config))
    assert out.token_ids.cpu().tolist() == oracle["token_ids"].tolist()
    assert np.allclose(out.logprobs.cpu().numpy(), oracle["logprobs"], atol=1e-4)
    again = engine.generate(*flat(dev), repeats=2, sampling=LFM25SamplingConfig(**config))
    assert torch.equal(out.token_ids, again.token_ids), "the seen mask is rebuilt for every call"


def test_penalty_composes_with_top_k_on_bf16(dev):
    engine = make_engine(dev, torch.bfloat16)
    base = dict(temperature=1.0, max_new_tokens=16, seed=7, ignore_eos=True, repetition_penalty=1.5)
    greedy_like = engine.generate(*flat(dev), repeats=1, sampling=LFM25SamplingConfig(top_k=1, **base))
    greedy = engine.generate(*flat(dev), repeats=1,
                             sampling=LFM25SamplingConfig(**{**base, "temperature": 0.0}))
    assert torch.equal(greedy_like.token_ids, greedy.token_ids), "top_k = 1 of the penalised logits is their arg max"
    assert torch.allclose(greedy_like.logprobs, greedy.logprobs, atol=1e-6)
