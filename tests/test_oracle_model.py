"""The numpy oracle engine against outputs of the reference's eager CPU engine.

tests/golden/model.json was produced by tests/golden/make_golden.py running the reference
``LFM25Engine`` on CPU (fp32 and bf16) on the seeded tiny hybrid model: conv,conv,attn,conv,
hidden 256, 4 q / 2 kv heads, vocab 4096, 8 prompts of 8..64 tokens, 32 greedy tokens, with
and without an EOS forced at a seeded step per sequence.
"""
import numpy as np
import pytest

from climbing_gym_b200 import synthetic
from oracle.lfm25_oracle import OracleConfig, OracleEngine, OracleSampling


def oracle_config(cfg):
    return OracleConfig(vocab_size=cfg.vocab_size, hidden_size=cfg.hidden_size, mlp_hidden_size=cfg.mlp_hidden_size,
                        num_attention_heads=cfg.num_attention_heads, num_key_value_heads=cfg.num_key_value_heads,
                        layer_types=tuple(cfg.layer_types), rope_theta=cfg.rope_theta, norm_eps=cfg.norm_eps,
                        conv_kernel_size=cfg.conv_kernel_size, eos_token_id=cfg.eos_token_id)


def build(untied, dtype, **kw):
    cfg = synthetic.tiny_config()
    state = synthetic.make_state_dict(cfg, seed=0, untied_head=untied)
    return cfg, OracleEngine(oracle_config(cfg), state, dtype=dtype, max_model_len=256, **kw)


PROMPTS = synthetic.uniform_prompts(8, 8, 64, 4096, seed=0)


@pytest.mark.parametrize("tag,untied", [("untied", True), ("tied", False)])
@pytest.mark.parametrize("eos", [False, True])
def test_generate_fp32_identical_tokens_and_bookkeeping(golden, tag, untied, eos):
    want = golden("model")[f"generate_{'eos_' if eos else ''}{tag}_fp32"]
    _, engine = build(untied, "fp32")
    sampling = OracleSampling(temperature=0.0, max_new_tokens=32,
                              force_eos_at=tuple(want["force_eos_at"]) if eos else None)
    got = engine.generate(PROMPTS, 1, sampling)
    assert got["token_ids"].tolist() == want["token_ids"]
    assert got["lengths"].tolist() == want["lengths"]
    assert got["finish_reasons"].tolist() == want["finish_reasons"]
    assert np.allclose(got["logprobs"], np.array(want["logprobs"]), atol=1e-4)


@pytest.mark.parametrize("tag,untied", [("untied", True), ("tied", False)])
def test_generate_bf16_tracks_reference_bf16(golden, tag, untied):
    """bf16 on CPU: the reference's torch kernels and numpy differ in fp32 accumulation order, so
    logits can differ in the last bf16 place; tokens must agree except at near-ties and log-probs
    within the bf16 tolerance of 2e-2."""
    want = golden("model")[f"generate_{tag}_bf16"]
    _, engine = build(untied, "bf16")
    got = engine.generate(PROMPTS, 1, OracleSampling(temperature=0.0, max_new_tokens=32))
    ours, ref = got["token_ids"][:, 0], np.array(want["token_ids"])[:, 0]
    first_diff = [int(np.argmax(a != b)) if (a != b).any() else 32 for a, b in zip(ours, ref)]
    assert np.mean(np.array(first_diff) == 32) >= 0.5, first_diff
    lp, ref_lp = got["logprobs"][:, 0], np.array(want["logprobs"])[:, 0]
    for row, stop in enumerate(first_diff):
        assert np.allclose(lp[row, :stop], ref_lp[row, :stop], atol=2e-2)
        if stop < 32:  # a divergence is only legitimate at a near-tie of the two winners
            assert abs(lp[row, stop] - ref_lp[row, stop]) < 2e-2, (row, stop)


@pytest.mark.parametrize("tag,untied", [("untied", True), ("tied", False)])
def test_prefill_logits_repeats_and_scoring(golden, tag, untied):
    g = golden("model")
    _, engine = build(untied, "fp32")
    want = g[f"prefill_{tag}_fp32"]
    for i, prompt in enumerate(PROMPTS[:4]):
        _, logits = engine.prefill(prompt)
        assert int(np.argmax(logits)) == want["argmax"][i]
        assert np.allclose(logits[:16], want["head"][i], atol=1e-4)
        m = logits.max()
        assert abs(float(m + np.log(np.exp(logits - m).sum())) - want["lse"][i]) < 1e-4
    rep = g[f"generate_repeats_{tag}_fp32"]
    got = engine.generate(PROMPTS[:3], 2, OracleSampling(temperature=0.0, max_new_tokens=8))
    assert got["token_ids"].tolist() == rep["token_ids"] and got["lengths"].tolist() == rep["lengths"]
    completions = synthetic.uniform_prompts(4, 3, 12, 4096, seed=5)
    scores = engine.score_completions(PROMPTS[:4], completions)
    for mine, ref in zip(scores, g[f"score_{tag}_fp32"]):
        assert np.allclose(mine, ref, atol=2e-5)


def test_chunked_prefill_equals_one_shot_fp32():
    _, engine = build(True, "fp32")
    prompt = PROMPTS[3] + PROMPTS[4]
    _, whole = engine.prefill(prompt)
    state = None
    for start in range(0, len(prompt), 7):
        state, part = engine.prefill(prompt[start:start + 7], state)
    assert np.allclose(whole, part, atol=1e-4) and int(whole.argmax()) == int(part.argmax())


def test_fp8_paths_stay_close_to_bf16():
    _, base = build(True, "bf16")
    _, fp8 = build(True, "bf16", fp8_mlp=True, fp8_kv=True)
    a = base.generate(PROMPTS[:4], 1, OracleSampling(temperature=0.0, max_new_tokens=8))
    b = fp8.generate(PROMPTS[:4], 1, OracleSampling(temperature=0.0, max_new_tokens=8))
    same = a["token_ids"] == b["token_ids"]
    assert same.mean() > 0.5
    assert np.abs(a["logprobs"][same] - b["logprobs"][same]).max() < 0.25


@pytest.mark.parametrize("penalty", [1.3, 0.8])
def test_generate_with_repetition_penalty_matches_reference(golden, penalty):
    want = golden("penalty")[f"generate_fp32_{penalty}"]
    _, engine = build(True, "fp32")
    got = engine.generate(PROMPTS[:4], 2, OracleSampling(temperature=0.0, max_new_tokens=24, ignore_eos=True,
                                                         repetition_penalty=penalty))
    assert got["token_ids"].tolist() == want["token_ids"]
    assert np.allclose(got["logprobs"], np.array(want["logprobs"]), atol=1e-4)
    plain = engine.generate(PROMPTS[:4], 2, OracleSampling(temperature=0.0, max_new_tokens=24, ignore_eos=True))
    assert plain["token_ids"].tolist() != want["token_ids"], "the penalty must change the greedy path"
