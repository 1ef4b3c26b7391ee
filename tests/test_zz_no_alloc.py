"""cgym_sample_static (sampler with the slice scratch inside the library image) against
cgym_sample with a caller-owned workspace, through the C ABI.

Both run the same kernel with the same slicing, so tokens must be identical and log-probs agree
to the sampler tests' tolerance (3e-6). The file name sorts last so the entry point is also
exercised after every other test has used the device.
"""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

nv = pytest.importorskip("climbing_gym_b200._native")

MAX_ROWS = 512  # CGYM_SAMPLE_STATIC_MAX_ROWS in include/cgym_b200.h


@pytest.fixture(scope="module")
def dev():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    nv.load()
    return torch.device("cuda:0")


def make_case(dev, rows, vocab, dtype, seed):
    gen = torch.Generator(device="cpu").manual_seed(seed)
    logits = (torch.randn(rows, vocab, generator=gen) * 3.0).to(dev).to(dtype)
    seeds = (torch.arange(rows, dtype=torch.int64) * 104729 + seed).to(dev)
    steps = (torch.arange(rows, dtype=torch.int64) % 7).to(dev)
    temps = torch.where(torch.arange(rows) % 3 == 0, torch.zeros(rows), torch.full((rows,), 0.8)).to(dev)
    offsets = (torch.arange(rows, dtype=torch.int64) * vocab).to(dev)
    return logits, seeds, steps, temps, offsets


def run_workspace(dev, case, code):
    logits, seeds, steps, temps, offsets = case
    rows, vocab = logits.shape
    tokens = torch.full((rows,), -1, device=dev, dtype=torch.int64)
    logp = torch.zeros(rows, device=dev, dtype=torch.float32)
    ws = torch.zeros(int(nv.load().cgym_sample_workspace_bytes(rows)) // 4, device=dev, dtype=torch.float32)
    nv.call("cgym_sample", nv.ptr(tokens), nv.ptr(logp), nv.ptr(logits), nv.ptr(seeds), nv.ptr(steps), nv.ptr(temps),
            nv.ptr(offsets), rows, vocab, code, nv.ptr(ws), nv.stream_ptr())
    torch.cuda.synchronize()
    return tokens.cpu().numpy(), logp.cpu().numpy()


def run_static(dev, case, code):
    logits, seeds, steps, temps, offsets = case
    rows, vocab = logits.shape
    tokens = torch.full((rows,), -1, device=dev, dtype=torch.int64)
    logp = torch.zeros(rows, device=dev, dtype=torch.float32)
    nv.call("cgym_sample_static", nv.ptr(tokens), nv.ptr(logp), nv.ptr(logits), nv.ptr(seeds), nv.ptr(steps),
            nv.ptr(temps), nv.ptr(offsets), rows, vocab, code, nv.stream_ptr())
    torch.cuda.synchronize()
    return tokens.cpu().numpy(), logp.cpu().numpy()


@pytest.mark.parametrize("rows,vocab,dtype", [(5, 65536, torch.float32), (64, 16384, torch.bfloat16),
                                              (MAX_ROWS, 8192, torch.float32), (3, 1000, torch.float32)])
def test_static_scratch_sampler_matches_workspace_sampler_twice_in_a_row(dev, rows, vocab, dtype):
    code = nv.dtype_code(dtype)
    nv.call("cgym_sample_static", None, None, None, None, None, None, None, 0, vocab, code, nv.stream_ptr())  # set-up only
    for call in range(2):  # the second call reuses the scratch the first one left behind
        case = make_case(dev, rows, vocab, dtype, seed=17 + call)
        want_tokens, want_logp = run_workspace(dev, case, code)
        got_tokens, got_logp = run_static(dev, case, code)
        assert (want_tokens >= 0).all() and (want_tokens < vocab).all()
        assert np.array_equal(got_tokens, want_tokens), (call, rows, vocab)
        assert np.allclose(got_logp, want_logp, atol=3e-6), (call, rows, vocab)
    # a smaller batch right after a larger one: its counters sit elsewhere in the scratch
    if rows > 2:
        case = make_case(dev, rows // 2, vocab, dtype, seed=99)
        want_tokens, want_logp = run_workspace(dev, case, code)
        got_tokens, got_logp = run_static(dev, case, code)
        assert np.array_equal(got_tokens, want_tokens)
        assert np.allclose(got_logp, want_logp, atol=3e-6)


def test_static_scratch_sampler_rejects_batches_beyond_its_limit(dev):
    rows, vocab = MAX_ROWS + 1, 64
    case = make_case(dev, rows, vocab, torch.float32, seed=3)
    with pytest.raises(nv.NativeKernelError, match=f"at most {MAX_ROWS} rows"):
        run_static(dev, case, nv.F32)
    torch.cuda.synchronize()
    # the device is still usable and the limit itself is accepted
    tokens, _ = run_static(dev, make_case(dev, MAX_ROWS, vocab, torch.float32, seed=4), nv.F32)
    assert (tokens >= 0).all() and (tokens < vocab).all()
