"""Per-kernel parity of the CUDA path (through the C ABI) against the CPU oracle.

Integer / index work and elementwise bf16 rounding chains must match bit-for-bit; kernels
that contain an rsqrt / exp or a different fp32 summation order are allowed one bf16 ulp on
at most 1 % of the elements (tolerance written at each check).
"""
import ctypes as C

import numpy as np
import pytest
import torch

from inputs import kernel_inputs, rope_tables
from oracle import kernels as ok
from oracle import philox
from oracle.lfm25_oracle import OracleEngine
from oracle.numerics import bf16_bits, decode_e4m3, round_bf16
from oracle.pages import PagePoolOracle

pytestmark = pytest.mark.gpu

nv = pytest.importorskip("climbing_gym_b200._native")


@pytest.fixture(scope="module")
def dev():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    nv.load()
    return torch.device("cuda:0")


def stream():
    return nv.stream_ptr()


def bf(x, dev):
    return torch.from_numpy(np.asarray(x, np.float32)).to(dev).to(torch.bfloat16)


def f32(t):
    return t.float().cpu().numpy()


def assert_bf16_close(got, want, *, exact_fraction=0.99, ulps=1, what=""):
    """bf16 results: every element within `ulps` bf16 steps, at least `exact_fraction` bit-identical."""
    got, want = np.asarray(got, np.float32), np.asarray(want, np.float32)
    a, b = bf16_bits(got).astype(np.int32), bf16_bits(want).astype(np.int32)
    # compare in a sign-magnitude-safe way: differing signs only allowed around zero
    diff = np.abs(a - b)
    near_zero = (np.abs(got) < 1e-30) & (np.abs(want) < 1e-30)
    bad = (diff > ulps) & ~near_zero
    assert not bad.any(), f"{what}: {bad.sum()} elements differ by more than {ulps} ulp; worst {diff.max()}"
    assert np.mean(diff == 0) >= exact_fraction, f"{what}: only {np.mean(diff == 0):.4f} bit-identical"


def assert_gemm_close(got, want, *, exact_fraction=0.97, what=""):
    """GEMM outputs: one bf16 rounding step of the value, plus an absolute term for results that are
    the small remainder of a long cancelling sum (1e-3 of the output RMS, far above fp32
    accumulation-order noise and far below one bf16 step of a typical output)."""
    got, want = np.asarray(got, np.float32), np.asarray(want, np.float32)
    rms = float(np.sqrt(np.mean(want.astype(np.float64) ** 2))) + 1e-30
    err = np.abs(got - want)
    bound = 2.0 ** -7 * np.abs(want) + 1e-3 * rms
    assert np.all(err <= bound), f"{what}: worst excess {np.max(err - bound):.3e} (rms {rms:.3e})"
    exact = np.mean(bf16_bits(got) == bf16_bits(want))
    assert exact >= exact_fraction, f"{what}: only {exact:.4f} bit-identical"


# ------------------------------------------------------------------------------------------ elementwise
def test_rmsnorm_bf16_and_fp32(dev):
    inp = kernel_inputs()
    rows, h = inp["rows"], inp["h"]
    x, r, w = bf(inp["x"], dev), bf(inp["res"], dev), bf(inp["norm_w"], dev)
    y, s = torch.empty_like(x), torch.empty_like(x)
    nv.call("cgym_rmsnorm", nv.ptr(y), nv.ptr(s), nv.ptr(x), nv.ptr(r), nv.ptr(w), rows, h, 1e-5, nv.BF16, stream())
    want_y, want_s = ok.rms_norm(inp["x"], inp["norm_w"], inp["eps"], inp["res"])
    assert np.array_equal(bf16_bits(f32(s)), bf16_bits(want_s)), "residual sum must be bit-exact"
    assert_bf16_close(f32(y), want_y, what="rmsnorm+residual")
    nv.call("cgym_rmsnorm", nv.ptr(y), None, nv.ptr(x), None, nv.ptr(w), rows, h, 1e-5, nv.BF16, stream())
    assert_bf16_close(f32(y), ok.rms_norm(inp["x"], inp["norm_w"], inp["eps"])[0], what="rmsnorm")
    xf, wf = x.float(), w.float()
    yf = torch.empty_like(xf)
    nv.call("cgym_rmsnorm", nv.ptr(yf), None, nv.ptr(xf), None, nv.ptr(wf), rows, h, 1e-5, nv.F32, stream())
    want = ok.rms_norm(inp["x"], inp["norm_w"], inp["eps"], rd=lambda v: np.asarray(v, np.float32))[0]
    assert np.allclose(f32(yf), want, rtol=1e-5, atol=1e-6)


def test_swiglu_and_quantised_variants(dev):
    inp = kernel_inputs()
    rows, f = inp["rows"], inp["f"]
    gu = bf(inp["gate_up"], dev)
    y = torch.empty((rows, f), device=dev, dtype=torch.bfloat16)
    nv.call("cgym_swiglu", nv.ptr(y), nv.ptr(gu), rows, f, nv.BF16, stream())
    assert_bf16_close(f32(y), ok.swiglu(inp["gate_up"]), exact_fraction=0.999, what="swiglu")
    q = torch.empty((rows, f), device=dev, dtype=torch.uint8)
    s = torch.empty(rows, device=dev, dtype=torch.float32)
    nv.call("cgym_swiglu_quant", nv.ptr(q), nv.ptr(s), nv.ptr(gu), rows, f, stream())
    codes, scales = ok.swiglu_quantize(inp["gate_up"])
    assert np.allclose(s.cpu().numpy(), scales, rtol=2 ** -7)
    assert np.mean(q.cpu().numpy() == codes) > 0.98


def test_quantize_rows_bit_exact(dev):
    inp = kernel_inputs()
    x = bf(inp["quant_x"], dev)
    rows, width = x.shape
    q = torch.empty((rows, width), device=dev, dtype=torch.uint8)
    s = torch.empty(rows, device=dev, dtype=torch.float32)
    nv.call("cgym_quantize_rows", nv.ptr(q), nv.ptr(s), nv.ptr(x), rows, width, nv.BF16, stream())
    codes, scales = ok.quantize_rows(inp["quant_x"])
    assert np.array_equal(s.cpu().numpy().view(np.uint32), scales.view(np.uint32))
    assert np.array_equal(decode_e4m3(q.cpu().numpy()), decode_e4m3(codes))  # -0 == +0


def test_rmsnorm_quant(dev):
    inp = kernel_inputs()
    rows, h = inp["rows"], inp["h"]
    x, r, w = bf(inp["x"], dev), bf(inp["res"], dev), bf(inp["norm_w"], dev)
    q = torch.empty((rows, h), device=dev, dtype=torch.uint8)
    s = torch.empty(rows, device=dev, dtype=torch.float32)
    summed = torch.empty_like(x)
    nv.call("cgym_rmsnorm_quant", nv.ptr(q), nv.ptr(s), nv.ptr(summed), nv.ptr(x), nv.ptr(r), nv.ptr(w), rows, h,
            1e-5, stream())
    codes, scales, want_sum = ok.rms_quantize(inp["x"], inp["norm_w"], inp["eps"], inp["res"])
    assert np.array_equal(bf16_bits(f32(summed)), bf16_bits(want_sum))
    assert np.allclose(s.cpu().numpy(), scales, rtol=2 ** -7)
    assert np.mean(q.cpu().numpy() == codes) > 0.97


def test_conv_update_bit_exact(dev):
    inp = kernel_inputs()
    rows, h = inp["rows"], inp["h"]
    bcx, w = bf(inp["bcx"], dev), bf(inp["conv_w"], dev)
    for active, slots in ((None, None), (inp["conv_active"], inp["conv_slots"])):
        state_ref = inp["conv_state"].copy()  # [slots, H, 3]
        state = bf(state_ref.transpose(0, 2, 1).copy(), dev)  # device layout [slots, 3, H]
        y = torch.empty((rows, h), device=dev, dtype=torch.bfloat16)
        a = None if active is None else torch.from_numpy(active.astype(np.uint8)).to(dev)
        sl = None if slots is None else torch.from_numpy(slots).to(dev)
        nv.call("cgym_conv_update", nv.ptr(y), nv.ptr(state), nv.ptr(bcx), nv.ptr(w), nv.ptr(a), nv.ptr(sl), rows, h,
                nv.BF16, stream())
        want = ok.conv_update(inp["bcx"], inp["conv_w"], state_ref, active, slots)
        assert np.array_equal(bf16_bits(f32(y)), bf16_bits(want))
        assert np.array_equal(bf16_bits(f32(state).transpose(0, 2, 1)), bf16_bits(state_ref))


def conv_prefill_reference(bx_rows, c_rows, w, carried):
    """exact products, fp32 sum in tap order, one rounding; returns (y, new taps [3, H])."""
    full = np.concatenate([carried, bx_rows])
    hist = full[1:]
    conv = round_bf16((hist[:-2] * w[:, 0] + hist[1:-1] * w[:, 1]) + hist[2:] * w[:, 2])
    return round_bf16(c_rows * conv), full[-3:]


def test_conv_prefill_packed_and_chunked(dev):
    rng = np.random.default_rng(3)
    h = 256
    lens = [1, 2, 5, 9]
    total = sum(lens)
    bcx_np = round_bf16(rng.standard_normal((total, 3 * h)))
    w_np = round_bf16(0.3 * rng.standard_normal((h, 3)))
    carried_np = round_bf16(rng.standard_normal((6, 3, h)))  # device layout [slot][tap][H]
    starts = [0, 4, 0, 7]  # sequences 1 and 3 continue from stored taps
    slots = [5, 0, 2, 3]
    state = bf(carried_np, dev)
    y = torch.empty((total, h), device=dev, dtype=torch.bfloat16)
    cu = np.concatenate([[0], np.cumsum(lens)]).astype(np.int32)
    args = [torch.from_numpy(np.asarray(v, np.int32)).to(dev) for v in (cu, slots, starts)]
    bcx_dev, w_dev = bf(bcx_np, dev), bf(w_np, dev)  # keep alive past the launch
    nv.call("cgym_conv_prefill", nv.ptr(y), nv.ptr(state), nv.ptr(bcx_dev), nv.ptr(w_dev),
            nv.ptr(args[0]), nv.ptr(args[1]), nv.ptr(args[2]), len(lens), total, h, nv.BF16, stream())
    got_y, got_state = f32(y), f32(state)
    for i, n in enumerate(lens):
        rows = bcx_np[cu[i]:cu[i + 1]]
        bx = round_bf16(rows[:, :h] * rows[:, 2 * h:])
        carried = carried_np[slots[i]] if starts[i] > 0 else np.zeros((3, h), np.float32)
        want_y, want_taps = conv_prefill_reference(bx, rows[:, h:2 * h], w_np, carried)
        assert np.array_equal(bf16_bits(got_y[cu[i]:cu[i + 1]]), bf16_bits(want_y)), f"sequence {i}"
        assert np.array_equal(bf16_bits(got_state[slots[i]]), bf16_bits(want_taps)), f"taps of sequence {i}"
    assert np.array_equal(bf16_bits(got_state[1]), bf16_bits(carried_np[1])), "untouched slot changed"


# ------------------------------------------------------------------------------------------ paged cache pieces
def make_cache(dev, *, dtype=torch.bfloat16, fp8=False, slots=4, max_len=256, page=16, hkv=2, d=64, layers=2, n_pages=None):
    from climbing_gym_b200.paged import PagedHybridCache
    return PagedHybridCache(n_attn_layers=layers, n_conv_layers=1, n_slots=slots, max_seq_len=max_len, n_kv_heads=hkv,
                            head_dim=d, hidden_size=64, dtype=dtype, device=dev, page_size=page, n_pages=n_pages,
                            fp8_kv=fp8)


def test_qk_norm_rope_append_and_gather(dev):
    inp = kernel_inputs()
    rows, hq, hkv, d = inp["rows"], inp["hq"], inp["hkv"], inp["d"]
    cos_np, sin_np = rope_tables(inp["rope_theta"], inp["rope_len"], d)
    cos, sin = torch.from_numpy(cos_np).to(dev), torch.from_numpy(sin_np).to(dev)
    cache = make_cache(dev, slots=rows, max_len=4096 + 64, page=64, hkv=hkv, d=d)
    positions = torch.from_numpy(inp["positions"]).to(dev)
    slot_ids = torch.arange(rows, device=dev, dtype=torch.int32)
    cache.reserve(slot_ids, (positions + 1).int())
    q = torch.empty((rows, hq, d), device=dev, dtype=torch.bfloat16)
    qkv, q_w, k_w = bf(inp["qkv"], dev), bf(inp["q_norm_w"], dev), bf(inp["k_norm_w"], dev)  # keep alive past the launch
    nv.call("cgym_qk_norm_rope_append", nv.ptr(q), None, None, nv.ptr(qkv),
            nv.ptr(q_w), nv.ptr(k_w), nv.ptr(cos), nv.ptr(sin),
            nv.ptr(positions), None, None, cache.kv, 1, rows, hq, 1e-5, nv.BF16, nv.ptr(cache.status), stream())
    want_q, want_k, want_v = ok.qkv_rope(inp["qkv"], inp["q_norm_w"], inp["k_norm_w"], cos_np, sin_np,
                                         inp["positions"], hq, hkv, d, inp["eps"])
    assert_bf16_close(f32(q), want_q, exact_fraction=0.98, what="q")
    assert int(cache.status.item()) == 0
    for row in range(rows):
        pos = int(inp["positions"][row])
        k, v = cache.dense_kv(1, row, pos + 1)
        assert_bf16_close(f32(k[pos]), want_k[row], exact_fraction=0.98, what=f"k row {row}")
        assert np.array_equal(bf16_bits(f32(v[pos])), bf16_bits(want_v[row])), "v is copied bit-exactly"


def attention_reference(q, k, v, scale, ks=None, vs=None, rd=round_bf16):
    """q [Hq, D], k/v [T, Hkv, D] (dequantised codes when scales are given)."""
    hq, hkv = q.shape[0], k.shape[1]
    g = hq // hkv
    qg = q.reshape(hkv, g, -1)
    s = np.einsum("hgd,thd->hgt", qg, k).astype(np.float32) * np.float32(scale)
    if ks is not None:
        s = s * ks.T[:, None, :]
    s = s - s.max(-1, keepdims=True)
    p = np.exp(s)
    total = p.sum(-1, keepdims=True)
    if vs is not None:
        p = p * vs.T[:, None, :]
    return (np.einsum("hgt,thd->hgd", rd(p), v) / total).reshape(hq, -1)


def fill_cache(cache, lens, hkv, d, rd, fp8, rng):
    """Random K/V per slot, written through the scatter entry point; returns what the cache now
    holds per slot as (k, v, k_scales, v_scales) with k/v dequantised codes for e4m3."""
    stored = []
    for slot, n in enumerate(lens):
        k, v = rd(rng.standard_normal((n, hkv, d))), rd(rng.standard_normal((n, hkv, d)))
        if n:
            cache.write_dense_kv(0, slot, 0, torch.from_numpy(k).to(cache.device), torch.from_numpy(v).to(cache.device))
        if fp8:
            kc, ksc = ok.store_kv_e4m3(k)
            vc, vsc = ok.store_kv_e4m3(v)
            stored.append((decode_e4m3(kc), decode_e4m3(vc), ksc, vsc))
        else:
            stored.append((k, v, None, None))
    return stored


@pytest.mark.parametrize("mode,impl,page", [("f32", 1, 16), ("bf16", 1, 16), ("e4m3", 1, 16), ("bf16", 1, 64),
                                            ("bf16", 2, 64), ("e4m3", 2, 64)])
@pytest.mark.parametrize("splits", [1, 3])
def test_paged_attention_matches_softmax_reference(dev, mode, impl, page, splits):
    rng = np.random.default_rng(5)
    hq, hkv, d = 8, 2, 64
    lens = [1, 15, 16, 17, 130, 0, 64, 65, 300]
    rows = len(lens)
    dtype = torch.float32 if mode == "f32" else torch.bfloat16
    cache = make_cache(dev, dtype=dtype, fp8=mode == "e4m3", slots=rows, max_len=320, page=page, hkv=hkv, d=d, layers=1)
    rd = (lambda x: np.asarray(x, np.float32)) if mode == "f32" else round_bf16
    slot_ids = torch.arange(rows, device=dev, dtype=torch.int32)
    cache.reserve(slot_ids, torch.tensor([max(n, 1) for n in lens], device=dev, dtype=torch.int32))
    stored = fill_cache(cache, lens, hkv, d, rd, mode == "e4m3", rng)
    # the gather entry point reads back exactly what was stored (layout round trip)
    k_back, v_back = cache.dense_kv(0, 4, 130)
    ks, vs = stored[4][2], stored[4][3]
    assert np.allclose(f32(k_back), stored[4][0] * (ks[..., None] if ks is not None else 1.0), rtol=1e-6)
    assert np.allclose(f32(v_back), stored[4][1] * (vs[..., None] if vs is not None else 1.0), rtol=1e-6)
    q_np = rd(rng.standard_normal((rows, hq, d)))
    q = torch.from_numpy(q_np).to(dev).to(dtype)
    out = torch.full((rows, hq, d), 7.0, device=dev, dtype=dtype)
    ws = torch.empty(rows * hq * splits * (d + 2), device=dev, dtype=torch.float32)
    kv_lens = torch.tensor(lens, device=dev, dtype=torch.int32)
    nv.call("cgym_paged_attention", nv.ptr(out), nv.ptr(q), nv.ptr(kv_lens), None, None, cache.kv, 0, rows, hq,
            d ** -0.5, splits, nv.ptr(ws), nv.F32 if mode == "f32" else nv.BF16, impl, nv.ptr(cache.status), stream())
    got = f32(out)
    assert int(cache.status.item()) == 0
    tol = 1e-5 if mode == "f32" else 0.012  # the reference's own fp8-KV decode tolerance
    for row, n in enumerate(lens):
        if n == 0:
            assert np.all(got[row] == 0), "empty history must give zeros"
            continue
        k, v, ks, vs = stored[row]
        want = attention_reference(q_np[row], k, v, d ** -0.5, ks, vs, rd)
        err = np.abs(got[row].reshape(hq, d) - want).max()
        assert err <= tol, f"row {row} len {n}: {err}"


@pytest.mark.parametrize("mode", ["bf16", "e4m3"])
@pytest.mark.parametrize("splits", [1, 4, 16])
def test_paged_attention_long_contexts_with_splits(dev, mode, splits):
    """The long-context decode shapes: 32 query / 8 KV heads, rows of 8 K - 12 K cached tokens next to short
    ones (the deep page rings, many pages per warp, and the split / combine path with up to 16 splits)."""
    rng = np.random.default_rng(17)
    hq, hkv, d = 32, 8, 64
    lens = [8192 + 17, 300, 12000, 9000, 64, 8192]
    rows = len(lens)
    cache = make_cache(dev, fp8=mode == "e4m3", slots=rows, max_len=12032, page=64, hkv=hkv, d=d, layers=1)
    cache.reserve(torch.arange(rows, device=dev, dtype=torch.int32), torch.tensor(lens, device=dev, dtype=torch.int32))
    stored = fill_cache(cache, lens, hkv, d, round_bf16, mode == "e4m3", rng)
    q_np = round_bf16(rng.standard_normal((rows, hq, d)))
    q = bf(q_np, dev)
    out = torch.full((rows, hq, d), 7.0, device=dev, dtype=torch.bfloat16)
    ws = torch.empty(rows * hq * splits * (d + 2), device=dev, dtype=torch.float32)
    kv_lens = torch.tensor(lens, device=dev, dtype=torch.int32)
    nv.call("cgym_paged_attention", nv.ptr(out), nv.ptr(q), nv.ptr(kv_lens), None, None, cache.kv, 0, rows, hq,
            d ** -0.5, splits, nv.ptr(ws), nv.BF16, 2, nv.ptr(cache.status), stream())
    got = f32(out)
    assert int(cache.status.item()) == 0
    for row, n in enumerate(lens):
        k, v, ks, vs = stored[row]
        want = attention_reference(q_np[row], k, v, d ** -0.5, ks, vs, round_bf16)
        err = np.abs(got[row].reshape(hq, d) - want).max()
        assert err <= 0.012, f"row {row} len {n} splits {splits}: {err}"


@pytest.mark.parametrize("mode", ["bf16", "e4m3"])
@pytest.mark.parametrize("hq,hkv", [(8, 2), (4, 4), (6, 2)])
def test_prefill_attention_tensor_core_causal_with_prefix(dev, mode, hq, hkv):
    """Packed query tiles against the paged cache: a fresh prompt, a chunk continuing a cached prefix
    and a one-token tail, each token attending causally to [0, its position]."""
    rng = np.random.default_rng(8)
    d, page, g = 64, 64, hq // hkv
    tq = 128 // g
    # (slot, cached prefix length, new tokens)
    seqs = [(0, 0, 150), (2, 70, 45), (1, 200, 1)]
    cache = make_cache(dev, fp8=mode == "e4m3", slots=3, max_len=320, page=page, hkv=hkv, d=d, layers=1)
    totals = {slot: pre + new for slot, pre, new in seqs}
    cache.reserve(torch.tensor(sorted(totals), device=dev, dtype=torch.int32),
                  torch.tensor([totals[s] for s in sorted(totals)], device=dev, dtype=torch.int32))
    stored = fill_cache(cache, [totals[s] for s in range(3)], hkv, d, round_bf16, mode == "e4m3", rng)
    n_rows = sum(new for _, _, new in seqs)
    q_np = round_bf16(rng.standard_normal((n_rows, hq, d)))
    q = bf(q_np, dev)
    out = torch.full((n_rows, hq, d), 7.0, device=dev, dtype=torch.bfloat16)
    row0, ntok, tslot, pos0, base = [], [], [], [], 0
    for slot, pre, new in seqs:
        for off in range(0, new, tq):
            row0.append(base + off); ntok.append(min(tq, new - off)); tslot.append(slot); pos0.append(pre + off)
        base += new
    meta = [torch.tensor(v, device=dev, dtype=torch.int32) for v in (row0, ntok, tslot, pos0)]
    nv.call("cgym_prefill_attention", nv.ptr(out), nv.ptr(q), nv.ptr(meta[0]), nv.ptr(meta[1]), nv.ptr(meta[2]),
            nv.ptr(meta[3]), cache.kv, 0, len(row0), hq, d ** -0.5, nv.BF16, nv.ptr(cache.status), stream())
    got = f32(out)
    assert int(cache.status.item()) == 0
    base = 0
    for slot, pre, new in seqs:
        k, v, ks, vs = stored[slot]
        for t in range(new):
            n = pre + t + 1
            want = attention_reference(q_np[base + t], k[:n], v[:n], d ** -0.5, None if ks is None else ks[:n],
                                       None if vs is None else vs[:n], round_bf16)
            err = np.abs(got[base + t].reshape(hq, d) - want).max()
            assert err <= 0.012, f"slot {slot} token {t}: {err}"
        base += new


def test_page_allocator_trace_matches_oracle(dev):
    slots, page, max_len, n_pages = 6, 16, 128, 20
    cache = make_cache(dev, slots=slots, max_len=max_len, page=page, n_pages=n_pages, layers=1)
    oracle = PagePoolOracle(n_pages, page, max_len // page, slots)

    def check():
        torch.cuda.synchronize()
        assert np.array_equal(cache.block_table.cpu().numpy(), oracle.block_table)
        assert np.array_equal(cache.n_blocks.cpu().numpy(), oracle.n_blocks)
        assert np.array_equal(cache.refcount.cpu().numpy(), oracle.refcount)
        assert np.array_equal(cache.free_bitmap.cpu().numpy().view(np.uint32), oracle.bitmap_words())
        assert np.array_equal(cache.seq_lens.cpu().numpy(), oracle.seq_lens)
        assert int(cache.status.item()) == oracle.status

    def t(values, dtype=torch.int32):
        return torch.tensor(values, device=dev, dtype=dtype)

    # admit three prompts
    cache.reserve(t([0, 2, 3]), t([40, 16, 1]))
    oracle.reserve([0, 2, 3], [40, 16, 1])
    for slot, n in ((0, 40), (2, 16), (3, 1)):
        cache.seq_lens[slot] = n
        oracle.seq_lens[slot] = n
    check()
    # decode steps: slot 2 crosses a page boundary at once, slot 3 after 15 more tokens
    pending = t([1, 0, 1, 1, 0, 0], torch.uint8)
    active = torch.zeros(slots, device=dev, dtype=torch.uint8)
    kv_lens = torch.full((slots,), -7, device=dev, dtype=torch.int32)
    for _ in range(20):
        nv.call("cgym_step_begin", cache.pool, nv.ptr(cache.seq_lens), nv.ptr(pending), nv.ptr(active), None, None,
                nv.ptr(kv_lens), slots, nv.ptr(cache.status), stream())
        assert kv_lens.cpu().tolist() == (cache.seq_lens + 1).cpu().tolist()
        oracle.step([1, 0, 1, 1, 0, 0])
        cache.seq_lens += pending.int()
        oracle.seq_lens += np.array([1, 0, 1, 1, 0, 0], np.int32)
        assert active.cpu().tolist() == [1, 0, 1, 1, 0, 0]
    check()
    # prefix sharing: slots 4 and 5 fork slot 0 (60 tokens: 3 full pages + a private partial page)
    cache.fork(t([0, 0]), t([4, 5]), t([60, 60]))
    oracle.fork([0, 0], [4, 5], [60, 60])
    check()
    # evict slot 0: shared pages stay alive through the children; then evict a child
    cache.release(t([1, 0, 0, 0, 0, 0], torch.uint8)); oracle.release([1, 0, 0, 0, 0, 0]); check()
    cache.release(t([0, 0, 0, 0, 1, 0], torch.uint8)); oracle.release([0, 0, 0, 0, 1, 0]); check()
    # lowest free page first after eviction, and exhaustion is reported, not fatal
    cache.reserve(t([1]), t([128])); oracle.reserve([1], [128]); check()
    cache.reserve(t([0]), t([128])); oracle.reserve([0], [128])
    torch.cuda.synchronize()
    assert int(cache.status.item()) & 1 and oracle.status & 1
    assert np.array_equal(cache.block_table.cpu().numpy(), oracle.block_table)


# ------------------------------------------------------------------------------------------ GEMM
def gemm_call(dev, x, w, *, impl, mask=None, ws_bytes=0):
    m, k = x.shape
    n = w.shape[0]
    y = torch.full((m, n), -3.0, device=dev, dtype=x.dtype)
    ws_bytes = ws_bytes + 4096 if ws_bytes else 0  # room for the split-K partial tiles
    ws = torch.zeros(max(ws_bytes, 16), device=dev, dtype=torch.uint8)
    status = torch.zeros(1, device=dev, dtype=torch.int32)
    nv.call("cgym_gemm", nv.ptr(y), nv.ptr(x), nv.ptr(w), nv.ptr(mask), m, n, k, nv.dtype_code(x.dtype), impl,
            nv.ptr(ws) if ws_bytes else None, ws_bytes, nv.ptr(status), stream())
    torch.cuda.synchronize()
    assert int(status.item()) == 0, f"gemm status {int(status.item())}"
    return y


@pytest.mark.parametrize("shape", [(3, 70, 50), (64, 256, 256), (130, 192, 96)])
def test_gemm_simt_fp32_and_bf16(dev, shape):
    m, n, k = shape
    rng = np.random.default_rng(m)
    x_np, w_np = round_bf16(rng.standard_normal((m, k))), round_bf16(rng.standard_normal((n, k)) * 0.1)
    want = x_np @ w_np.T
    y = gemm_call(dev, torch.from_numpy(x_np).to(dev), torch.from_numpy(w_np).to(dev), impl=1)
    assert np.allclose(f32(y), want, rtol=1e-5, atol=1e-5)
    yb = gemm_call(dev, bf(x_np, dev), bf(w_np, dev), impl=1)
    assert_gemm_close(f32(yb), round_bf16(want), exact_fraction=0.97, what="simt bf16")


@pytest.mark.parametrize("shape", [(1, 128, 64), (8, 256, 256), (64, 512, 2048), (33, 384, 320), (128, 1536, 256),
                                   (200, 256, 768), (300, 4096, 256), (64, 100, 192),
                                   (200, 37888, 64), (300, 16384, 128)])  # the last two: two feature sub-tiles per CTA
def test_gemm_tcgen05_matches_fp32_accumulation(dev, shape):
    m, n, k = shape
    rng = np.random.default_rng(n + k)
    x_np, w_np = round_bf16(rng.standard_normal((m, k))), round_bf16(rng.standard_normal((n, k)) * 0.1)
    want = round_bf16((x_np.astype(np.float64) @ w_np.astype(np.float64).T).astype(np.float32))
    y = gemm_call(dev, bf(x_np, dev), bf(w_np, dev), impl=2)
    assert_gemm_close(f32(y), want, exact_fraction=0.97, what=f"tcgen05 {shape}")
    mask_np = (rng.random(m) < 0.5).astype(np.uint8)
    ym = gemm_call(dev, bf(x_np, dev), bf(w_np, dev), impl=2, mask=torch.from_numpy(mask_np).to(dev))
    got = f32(ym)
    assert np.all(got[mask_np == 0] == -3.0), "masked rows must not be written"
    assert_gemm_close(got[mask_np == 1], want[mask_np == 1], exact_fraction=0.97, what="masked rows")


def test_gemm_tcgen05_split_k_is_deterministic_and_correct(dev):
    m, n, k = 40, 256, 4096
    rng = np.random.default_rng(9)
    x_np, w_np = round_bf16(rng.standard_normal((m, k))), round_bf16(rng.standard_normal((n, k)) * 0.05)
    want = round_bf16((x_np.astype(np.float64) @ w_np.astype(np.float64).T).astype(np.float32))
    # partial tiles exchanged through the workspace (2 tiles x 4 splits x [64][128] fp32 = 256 KiB) ...
    runs = [f32(gemm_call(dev, bf(x_np, dev), bf(w_np, dev), impl=3, ws_bytes=8 * m * n * 4)) for _ in range(2)]
    assert np.array_equal(runs[0], runs[1])
    assert_gemm_close(runs[0], want, exact_fraction=0.97, what="split-K")
    # ... and, without one, through distributed shared memory: same split order, same bits
    dsmem = f32(gemm_call(dev, bf(x_np, dev), bf(w_np, dev), impl=3, ws_bytes=0))
    assert np.array_equal(dsmem, runs[0])
    mask_np = (rng.random(m) < 0.5).astype(np.uint8)
    masked = f32(gemm_call(dev, bf(x_np, dev), bf(w_np, dev), impl=3, ws_bytes=8 * m * n * 4,
                           mask=torch.from_numpy(mask_np).to(dev)))
    assert np.all(masked[mask_np == 0] == -3.0) and np.array_equal(masked[mask_np == 1], runs[0][mask_np == 1])
    auto = f32(gemm_call(dev, bf(x_np, dev), bf(w_np, dev), impl=0, ws_bytes=16 * m * n * 4))
    assert_gemm_close(auto, want, exact_fraction=0.97, what="auto split-K")


@pytest.mark.parametrize("impl", [1, 2])
@pytest.mark.parametrize("shape", [(5, 128, 256), (64, 256, 1024), (100, 384, 512),
                                   (256, 37888, 128), (300, 16384, 128)])  # the last two: two feature sub-tiles per CTA
def test_gemm_fp8_scaled_epilogue(dev, impl, shape):
    m, n, k = shape
    rng = np.random.default_rng(k)
    xq, xs = ok.quantize_rows(round_bf16(rng.standard_normal((m, k))))
    wq, wsc = ok.quantize_rows(round_bf16(rng.standard_normal((n, k)) * 0.05))
    want = ok.fp8_matmul(xq, xs, wq, wsc)
    y = torch.zeros((m, n), device=dev, dtype=torch.bfloat16)
    status = torch.zeros(1, device=dev, dtype=torch.int32)
    args = [torch.from_numpy(a).to(dev) for a in (xq, xs, wq, wsc)]
    nv.call("cgym_gemm_fp8", nv.ptr(y), nv.ptr(args[0]), nv.ptr(args[1]), nv.ptr(args[2]), nv.ptr(args[3]), None,
            m, n, k, impl, None, 0, nv.ptr(status), stream())
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    assert_gemm_close(f32(y), want, exact_fraction=0.97, what=f"fp8 gemm impl {impl}")


DECODE_WS_BYTES = 2 * 148 * 128 * 128 * 4  # the engine's GEMM workspace: one fp32 partial tile per resident CTA


@pytest.mark.parametrize("impl,shape", [(4, (256, 256, 512)), (4, (200, 512, 256)), (4, (300, 1024, 2048)),
                                        (4, (1000, 2048, 448)), (4, (64, 768, 128)),
                                        (5, (256, 256, 512)), (5, (1000, 2048, 448)), (5, (2000, 4096, 256)),
                                        (5, (3000, 8192, 256)), (5, (300, 512, 1024))])
def test_gemm_cta_pair_form(dev, impl, shape):
    """impl 4: two CTAs of a cluster share one 256 x 256 tile (tcgen05.mma.cta_group::2, each CTA stages half of the
    token tile, both copies complete on the leader's barrier). impl 5: the persistent form, one pair per SM pair
    walking over the tiles with two accumulators in TMEM (shapes with one, two and five tiles per pair). Same
    contract as the single-CTA kernel: fp32 accumulation, row mask, row map, FP8 scales, ragged M and a K that is
    not a multiple of the ring."""
    m, n, k = shape
    rng = np.random.default_rng(m * 3 + n + k)
    x_np, w_np = round_bf16(rng.standard_normal((m, k))), round_bf16(rng.standard_normal((n, k)) * 0.1)
    want = round_bf16((x_np.astype(np.float64) @ w_np.astype(np.float64).T).astype(np.float32))
    x, w = bf(x_np, dev), bf(w_np, dev)
    y = gemm_call(dev, x, w, impl=impl)
    assert_gemm_close(f32(y), want, exact_fraction=0.97, what=f"pair {shape}")
    out_rows = m + 7
    row_map = rng.permutation(out_rows)[:m].astype(np.int32)
    row_map[rng.random(m) < 0.2] = -1
    mask = (rng.random(m) < 0.7).astype(np.uint8)
    written = (row_map >= 0) & (mask == 1)
    status = torch.zeros(1, device=dev, dtype=torch.int32)
    dmap, dmask = torch.from_numpy(row_map).to(dev), torch.from_numpy(mask).to(dev)
    ys = torch.full((out_rows, n), -3.0, device=dev, dtype=torch.bfloat16)
    nv.call("cgym_gemm_scatter", nv.ptr(ys), nv.ptr(x), nv.ptr(w), nv.ptr(dmask), nv.ptr(dmap), m, n, k,
            nv.dtype_code(torch.bfloat16), impl, None, 0, nv.ptr(status), stream())
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    got = f32(ys)
    untouched = np.ones(out_rows, dtype=bool)
    untouched[row_map[written]] = False
    assert np.all(got[untouched] == -3.0)
    assert_gemm_close(got[row_map[written]], want[written], exact_fraction=0.97, what=f"pair scatter {shape}")
    if k % 128 == 0:
        xq, xs = ok.quantize_rows(round_bf16(rng.standard_normal((m, k))))
        wq, wsc = ok.quantize_rows(round_bf16(rng.standard_normal((n, k)) * 0.05))
        want8 = ok.fp8_matmul(xq, xs, wq, wsc)
        args = [torch.from_numpy(a).to(dev) for a in (xq, xs, wq, wsc)]
        y8 = torch.zeros((m, n), device=dev, dtype=torch.bfloat16)
        nv.call("cgym_gemm_fp8", nv.ptr(y8), nv.ptr(args[0]), nv.ptr(args[1]), nv.ptr(args[2]), nv.ptr(args[3]), None,
                m, n, k, impl, None, 0, nv.ptr(status), stream())
        torch.cuda.synchronize()
        assert int(status.item()) == 0
        assert_gemm_close(f32(y8), want8, exact_fraction=0.97, what=f"pair fp8 {shape}")


def test_gemm_bounded_wait_gives_up_and_the_context_survives(dev):
    """A wait that nothing satisfies (the producer arms its barriers but copies no tile: test hook) runs into the
    shortened limit; the kernel raises CGYM_STATUS_WAIT_TIMEOUT in the status word, frees its TMEM and returns.
    The next GEMM on the same context is correct. Nothing faults, traps or hangs."""
    STATUS_WAIT_TIMEOUT = 4  # CGYM_STATUS_WAIT_TIMEOUT
    lib = nv.load()
    m, n, k = 64, 512, 1024
    rng = np.random.default_rng(3)
    x_np, w_np = round_bf16(rng.standard_normal((m, k))), round_bf16(rng.standard_normal((n, k)) * 0.1)
    want = round_bf16((x_np.astype(np.float64) @ w_np.astype(np.float64).T).astype(np.float32))
    x, w = bf(x_np, dev), bf(w_np, dev)
    y = torch.zeros((m, n), device=dev, dtype=torch.bfloat16)
    ws = torch.zeros(DECODE_WS_BYTES, device=dev, dtype=torch.uint8)
    status = torch.zeros(1, device=dev, dtype=torch.int32)

    def launch():
        nv.call("cgym_gemm", nv.ptr(y), nv.ptr(x), nv.ptr(w), None, m, n, k, nv.dtype_code(torch.bfloat16), 0,
                nv.ptr(ws), ws.numel(), nv.ptr(status), stream())
        torch.cuda.synchronize()

    torch.cuda.synchronize()
    assert lib.cgym_test_gemm_wait(2_000_000, 1) == 0  # give up after 2 ms; copy nothing
    try:
        launch()
        assert int(status.item()) & STATUS_WAIT_TIMEOUT, "the expired wait must be reported in the status word"
    finally:
        torch.cuda.synchronize()
        assert lib.cgym_test_gemm_wait(0, 0) == 0
    status.zero_()
    launch()
    assert int(status.item()) == 0
    assert_gemm_close(f32(y), want, exact_fraction=0.97, what="gemm after a timed-out launch")


@pytest.mark.parametrize("shape,ws", [((200, 512, 256), 0), ((200, 2048, 2048), 1), ((256, 16384, 512), 0),
                                      ((48, 256, 4096), 1)])
def test_gemm_scatter_writes_mapped_rows_only(dev, shape, ws):
    """cgym_gemm_scatter / cgym_gemm_fp8_scatter: token row m lands in output row row_map[m]; rows mapped to a
    negative index and masked rows leave y untouched (replaces _scatter_logits, lfm25_batching.py:25-33).
    Shapes take the unsplit epilogue (16-byte row segments), split-K through the workspace, two feature
    sub-tiles per CTA and 64-token tiles."""
    m, n, k = shape
    rng = np.random.default_rng(m + n)
    out_rows = m + 24
    row_map = rng.permutation(out_rows)[:m].astype(np.int32)
    row_map[rng.random(m) < 0.15] = -1
    mask = (rng.random(m) < 0.8).astype(np.uint8)
    written = (row_map >= 0) & (mask == 1)
    ws_bytes = DECODE_WS_BYTES if ws else 0
    work = torch.zeros(max(ws_bytes, 16), device=dev, dtype=torch.uint8)
    status = torch.zeros(1, device=dev, dtype=torch.int32)
    dmap, dmask = torch.from_numpy(row_map).to(dev), torch.from_numpy(mask).to(dev)

    x_np, w_np = round_bf16(rng.standard_normal((m, k))), round_bf16(rng.standard_normal((n, k)) * 0.1)
    want = round_bf16((x_np.astype(np.float64) @ w_np.astype(np.float64).T).astype(np.float32))
    y = torch.full((out_rows, n), -3.0, device=dev, dtype=torch.bfloat16)
    x, w = bf(x_np, dev), bf(w_np, dev)
    nv.call("cgym_gemm_scatter", nv.ptr(y), nv.ptr(x), nv.ptr(w), nv.ptr(dmask), nv.ptr(dmap),
            m, n, k, nv.dtype_code(torch.bfloat16), 0, nv.ptr(work) if ws else None, ws_bytes, nv.ptr(status), stream())
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    got = f32(y)
    untouched = np.ones(out_rows, dtype=bool)
    untouched[row_map[written]] = False
    assert np.all(got[untouched] == -3.0), "rows outside the map, masked rows and unmapped rows must stay as they were"
    assert_gemm_close(got[row_map[written]], want[written], exact_fraction=0.97, what=f"scatter bf16 {shape}")

    if k % 128 == 0:
        xq, xs = ok.quantize_rows(round_bf16(rng.standard_normal((m, k))))
        wq, wsc = ok.quantize_rows(round_bf16(rng.standard_normal((n, k)) * 0.05))
        want8 = ok.fp8_matmul(xq, xs, wq, wsc)
        args = [torch.from_numpy(a).to(dev) for a in (xq, xs, wq, wsc)]
        y8 = torch.full((out_rows, n), -3.0, device=dev, dtype=torch.bfloat16)
        nv.call("cgym_gemm_fp8_scatter", nv.ptr(y8), nv.ptr(args[0]), nv.ptr(args[1]), nv.ptr(args[2]), nv.ptr(args[3]),
                nv.ptr(dmask), nv.ptr(dmap), m, n, k, 0, nv.ptr(work) if ws else None, ws_bytes, nv.ptr(status), stream())
        torch.cuda.synchronize()
        assert int(status.item()) == 0
        got8 = f32(y8)
        assert np.all(got8[untouched] == -3.0)
        assert_gemm_close(got8[row_map[written]], want8[written], exact_fraction=0.97, what=f"scatter fp8 {shape}")


# The decode step's own launches: the 1.2B model's projection shapes at the batch sizes that are benchmarked,
# with the engine's workspace size (2 x 148 resident CTAs, one [token tile][128] fp32 partial tile each), so the
# launcher takes the grids the step takes: cluster split-K up to 8 ways over an 8192-deep contraction, and two
# 128-token tiles at 256 rows.


@pytest.mark.parametrize("shape", [(256, 2048, 8192), (256, 16384, 2048), (64, 2048, 8192), (128, 2048, 8192),
                                   (17, 2048, 8192)])
def test_gemm_fp8_at_decode_shapes_with_auto_split_k(dev, shape):
    m, n, k = shape
    rng = np.random.default_rng(m + n)
    xq, xs = ok.quantize_rows(round_bf16(rng.standard_normal((m, k))))
    wq, wsc = ok.quantize_rows(round_bf16(rng.standard_normal((n, k)) * 0.05))
    want = ok.fp8_matmul(xq, xs, wq, wsc)
    args = [torch.from_numpy(a).to(dev) for a in (xq, xs, wq, wsc)]
    ws = torch.zeros(DECODE_WS_BYTES, device=dev, dtype=torch.uint8)
    status = torch.zeros(1, device=dev, dtype=torch.int32)
    runs = []
    for _ in range(2):
        y = torch.full((m, n), -3.0, device=dev, dtype=torch.bfloat16)
        nv.call("cgym_gemm_fp8", nv.ptr(y), nv.ptr(args[0]), nv.ptr(args[1]), nv.ptr(args[2]), nv.ptr(args[3]), None,
                m, n, k, 0, nv.ptr(ws), ws.numel(), nv.ptr(status), stream())
        torch.cuda.synchronize()
        runs.append(f32(y))
    assert int(status.item()) == 0
    assert np.array_equal(runs[0], runs[1]), "split-K must be deterministic"
    assert_gemm_close(runs[0], want, exact_fraction=0.97, what=f"fp8 gemm {shape}")


@pytest.mark.parametrize("shape", [(256, 2048, 2048), (256, 6144, 2048), (256, 3072, 2048), (64, 2048, 8192),
                                   (256, 2048, 8192), (512, 2048, 2048)])
def test_gemm_bf16_at_decode_shapes_with_auto_split_k(dev, shape):
    m, n, k = shape
    rng = np.random.default_rng(m + k)
    x_np, w_np = round_bf16(rng.standard_normal((m, k))), round_bf16(rng.standard_normal((n, k)) * 0.05)
    want = round_bf16((x_np.astype(np.float64) @ w_np.astype(np.float64).T).astype(np.float32))
    y = gemm_call(dev, bf(x_np, dev), bf(w_np, dev), impl=0, ws_bytes=DECODE_WS_BYTES)
    assert_gemm_close(f32(y), want, exact_fraction=0.97, what=f"bf16 gemm {shape}")


# ------------------------------------------------------------------------------------------ sampler
def sampler_logits():
    rng = np.random.default_rng(7)
    logits = (rng.standard_normal((5, 9000)) * 2.0).astype(np.float32)
    logits[1, 17] = logits[1, 4500] = 9.0
    logits[2, :4096] = -np.inf
    return logits


def test_sampler_matches_reference_vectors(dev, golden):
    g = golden("sampler")
    logits_np = sampler_logits()
    logits = torch.from_numpy(logits_np).to(dev)
    rows, vocab = logits_np.shape
    for case in g["cases"]:
        tokens = torch.empty(rows, device=dev, dtype=torch.int64)
        logp = torch.empty(rows, device=dev, dtype=torch.float32)
        if case["mode"] == "batch":
            seeds = torch.full((rows,), case["seed"], dtype=torch.int64)
            steps = torch.full((rows,), case["step"], dtype=torch.int64)
            temps = torch.full((rows,), case["temperature"], dtype=torch.float32)
            offsets = torch.arange(rows, dtype=torch.int64) * vocab
        else:
            seeds, steps = torch.tensor(case["seeds"]), torch.tensor(case["steps"])
            temps, offsets = torch.tensor(case["temperatures"], dtype=torch.float32), torch.zeros(rows, dtype=torch.int64)
        args = [a.to(dev) for a in (seeds, steps, temps, offsets)]
        # one CTA per row, then the sliced variant (several CTAs per row, last arrival combines)
        ws = torch.zeros(int(nv.load().cgym_sample_workspace_bytes(rows)) // 4, device=dev, dtype=torch.float32)
        for workspace in (None, ws, ws):
            tokens.fill_(-1)
            nv.call("cgym_sample", nv.ptr(tokens), nv.ptr(logp), nv.ptr(logits), nv.ptr(args[0]), nv.ptr(args[1]),
                    nv.ptr(args[2]), nv.ptr(args[3]), rows, vocab, nv.F32, nv.ptr(workspace), stream())
            assert tokens.cpu().tolist() == case["tokens"], case
            assert np.allclose(logp.cpu().numpy(), case["logprobs"], atol=3e-6), case
        assert float(ws.abs().max()) >= 0 and int(ws[-rows:].view(torch.int32).abs().max()) == 0, "counters re-armed"


def test_sampler_bf16_logits_and_distribution(dev):
    rng = np.random.default_rng(21)
    rows, vocab = 4096, 16
    base = np.log(np.array([0.3, 0.2, 0.1, 0.05] + [0.35 / 12] * 12, np.float32))
    logits = bf(np.tile(round_bf16(base), (rows, 1)), dev)
    tokens = torch.empty(rows, device=dev, dtype=torch.int64)
    logp = torch.empty(rows, device=dev, dtype=torch.float32)
    seeds = torch.arange(rows, device=dev, dtype=torch.int64) * 7919 + 1
    zeros = torch.zeros(rows, device=dev, dtype=torch.int64)
    temps = torch.ones(rows, device=dev, dtype=torch.float32)
    nv.call("cgym_sample", nv.ptr(tokens), nv.ptr(logp), nv.ptr(logits), nv.ptr(seeds), nv.ptr(zeros), nv.ptr(temps),
            None, rows, vocab, nv.BF16, None, stream())
    counts = np.bincount(tokens.cpu().numpy(), minlength=vocab) / rows
    probs = np.exp(round_bf16(base) - np.log(np.exp(round_bf16(base)).sum()))
    assert np.abs(counts - probs).max() < 0.03  # 4096 draws: ~4 sigma of the largest bin
    want_tokens, want_logp = OracleEngine.sample_per_row(None, f32(logits), seeds.cpu().numpy(), zeros.cpu().numpy(),
                                                         temps.cpu().numpy())
    assert np.mean(tokens.cpu().numpy() == want_tokens) > 0.999
    same = tokens.cpu().numpy() == want_tokens
    assert np.allclose(logp.cpu().numpy()[same], want_logp[same], atol=3e-6)


def test_sample_record_bookkeeping_matches_reference_kernel(dev, golden):
    """Same scenario as golden['record_sample']: the draw is forced through one-hot logits."""
    from climbing_gym_b200.decoder import SlotState
    g = golden("kernels")["record_sample"]
    n, cap, vocab, eos = 6, 4, 16, 2
    sampled = [5, 2, 9, 2, 7, 3]
    seq_lens = torch.zeros(n, device=dev, dtype=torch.int32)
    st = SlotState(n, cap, vocab, eos, seq_lens, stop_states=2)
    st.lengths.copy_(torch.tensor([0, 1, 3, 2, 0, 1]))
    st.limits.fill_(4)
    st.alive.copy_(torch.tensor([1, 1, 1, 1, 0, 1], dtype=torch.uint8))
    st.stop_offsets.copy_(torch.tensor([0, 0, 0, 0, 0, vocab]))
    st.stop_table[vocab + 3] = 65536
    st.ignore_eos.copy_(torch.tensor([0, 0, 0, 1, 0, 0], dtype=torch.uint8))
    st.rng_positions.copy_(torch.tensor([0, 1, 3, 2, 0, 1]))
    logits = torch.full((n, vocab), -20.0, device=dev)
    for row, tok in enumerate(sampled):
        logits[row, tok] = 20.0
    advance = torch.tensor([1, 0, 1, 0, 0, 1], device=dev, dtype=torch.uint8)
    nv.call("cgym_sample_record", nv.ptr(logits), C.byref(st.struct), nv.ptr(advance), None, None, n, vocab, nv.F32,
            nv.ptr(st.sample_ws), stream())
    torch.cuda.synchronize()
    assert st.tokens.cpu().tolist() == g["tokens"]
    for key, tensor in (("lengths", st.lengths), ("reasons", st.reasons), ("alive", st.alive), ("pending", st.pending),
                        ("input", st.input_tokens), ("rng_positions", st.rng_positions), ("stop_states", st.stop_states)):
        assert [int(v) for v in tensor.cpu().tolist()] == [int(v) for v in g[key]], key
    assert seq_lens.cpu().tolist() == [1, 0, 1, 0, 0, 1]
    # logprob of a one-hot row is ~0; the reference run stored its own synthetic logp values instead
    assert np.allclose(st.logprobs.cpu().numpy()[np.array(g["tokens"]) != 0], 0.0, atol=1e-6)


def test_target_logprobs(dev):
    rng = np.random.default_rng(2)
    logits_np = round_bf16(rng.standard_normal((7, 5000)) * 3)
    targets_np = rng.integers(0, 5000, size=7)
    out = torch.empty(7, device=dev, dtype=torch.float32)
    logits_dev, targets_dev = bf(logits_np, dev), torch.from_numpy(targets_np).to(dev)
    nv.call("cgym_target_logprobs", nv.ptr(out), nv.ptr(logits_dev), nv.ptr(targets_dev), 7, 5000, nv.BF16, stream())
    assert np.allclose(out.cpu().numpy(), OracleEngine.logprob_of(logits_np, targets_np), atol=3e-6)


# ------------------------------------------------------------------------------------------ 12-bit bf16 weight stream
def test_bf16_stream_preserves_every_bit_pattern_and_refreshes(dev):
    """All 65,536 bf16 bit patterns (rare exponents, signed zeros, infinities, NaN payloads) survive the packed
    stream; refresh re-encodes in place (reference: tests/test_lfm25_cuda.py:66-78)."""
    from climbing_gym_b200.weights import PackedBF16Weight

    bits = torch.arange(65536, device=dev, dtype=torch.int32).to(torch.int16).reshape(256, 256)
    weights = bits.view(torch.bfloat16).clone()
    packed = PackedBF16Weight.from_weight(weights)
    assert torch.equal(packed.unpack().view(torch.int16), bits)
    addresses = (packed.mantissa.data_ptr(), packed.exponent.data_ptr())
    weights.copy_(weights.flip(0))
    packed.refresh()
    assert torch.equal(packed.unpack().view(torch.int16), weights.view(torch.int16))
    assert addresses == (packed.mantissa.data_ptr(), packed.exponent.data_ptr())
    # the stream really is 12 bits per weight
    assert packed.mantissa.numel() + packed.exponent.numel() == weights.numel() * 3 // 2


@pytest.mark.parametrize("width", (128, 130, 2048, 10752))
def test_bf16_stream_gemv_matches_the_unpacked_product(dev, width):
    from climbing_gym_b200.weights import PackedBF16Weight

    rng = np.random.default_rng(319 + width)
    w_np = round_bf16(rng.standard_normal((256, width)) * 0.025)
    w_np[0, :4] = round_bf16(np.array([0.0, 1e-20, 1000.0, -1e-20]))  # values outside the coded exponent band
    x_np = round_bf16(rng.standard_normal((1, width)))
    weights, x = bf(w_np, dev), bf(x_np, dev)
    packed = PackedBF16Weight.from_weight(weights)
    assert torch.equal(packed.unpack().view(torch.int16), weights.view(torch.int16))
    want = round_bf16((x_np.astype(np.float64) @ w_np.astype(np.float64).T).astype(np.float32))
    got = f32(packed.linear(x))
    assert_gemm_close(got, want, exact_fraction=0.97, what=f"stream gemv {width}")
    kept = torch.full((1, 256), 5.0, device=dev, dtype=torch.bfloat16)
    packed.linear(x, out=kept, row_mask=torch.zeros(1, device=dev, dtype=torch.uint8))
    assert bool((kept == 5.0).all()), "a masked row is not written"
