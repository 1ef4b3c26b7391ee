// Fused sampler: Gumbel-max / greedy draw, sampled-token log-prob from the untempered logits and
// (optionally) the slot scheduler's per-row bookkeeping, one CTA per row, one pass over the row.
//
// Uniforms are Philox-4x32-10 (Salmon et al., SC'11) keyed per row with
// key = (seed + position * 0x9E3779B97F4A7C15) & (2^63 - 1), counter (offset + column, 0, 0, 0),
// first output word, mapped to [0,1) by folding the sign of its int32 view and scaling by 2^-31:
// the stream the reference sampler consumes, so a row's draws do not depend on which slot or
// batch it occupies. Ties resolve to the lowest token id.
#include "common.cuh"

namespace cgym {

constexpr int SAMPLE_THREADS = 1024;

__device__ __forceinline__ uint32_t philox_first_word(uint32_t c0, uint32_t k0, uint32_t k1) {
  uint32_t c1 = 0, c2 = 0, c3 = 0;
#pragma unroll
  for (int r = 0; r < 10; ++r) {
    const uint32_t hi_a = __umulhi(0xD2511F53u, c0), lo_a = 0xD2511F53u * c0;
    const uint32_t hi_b = __umulhi(0xCD9E8D57u, c2), lo_b = 0xCD9E8D57u * c2;
    c0 = hi_b ^ c1 ^ k0;
    c1 = lo_b;
    c2 = hi_a ^ c3 ^ k1;
    c3 = lo_a;
    k0 += 0x9E3779B9u;
    k1 += 0xBB67AE85u;
  }
  return c0;
}

__device__ __forceinline__ float uniform_from_word(uint32_t w) {
  int32_t x = static_cast<int32_t>(w);
  if (x < 0) x = -x - 1;
  return static_cast<float>(x) * 4.6566127342e-10f;
}

struct Best {
  float score;
  int index;
};
__device__ __forceinline__ Best better(Best a, Best b) {
  if (b.score > a.score || (b.score == a.score && b.index < a.index)) return b;
  return a;
}

template <typename T>
__global__ void __launch_bounds__(SAMPLE_THREADS)
sample_kernel(const T* __restrict__ logits, cgym_slot_state st, bool has_state,
              const uint8_t* __restrict__ advance, const int64_t* __restrict__ seeds,
              const int64_t* __restrict__ steps, const float* __restrict__ temperatures,
              const int64_t* __restrict__ rng_offsets, int64_t* __restrict__ sampled_out,
              float* __restrict__ logp_out, int vocab) {
  __shared__ float s_score[32], s_max[32], s_sum[32];
  __shared__ int s_index[32];
  const int row = blockIdx.x;
  if (has_state) {
    if (threadIdx.x == 0 && advance != nullptr && advance[row]) st.seq_lens[row] += 1;
    if (!st.alive[row]) return;
  }
  const float temperature = temperatures[row];
  const uint64_t key = (static_cast<uint64_t>(seeds[row]) +
                        static_cast<uint64_t>(steps[row]) * 0x9E3779B97F4A7C15ull) & 0x7FFFFFFFFFFFFFFFull;
  const uint32_t k0 = static_cast<uint32_t>(key), k1 = static_cast<uint32_t>(key >> 32);
  const uint32_t base = rng_offsets != nullptr ? static_cast<uint32_t>(rng_offsets[row]) : 0u;
  const T* x = logits + static_cast<int64_t>(row) * vocab;
  const float inv_t = temperature > 0.0f ? 1.0f / fmaxf(temperature, 1.0e-30f) : 1.0f;

  Best best{-INFINITY, 0x7fffffff};
  float mx = -INFINITY, sm = 0.0f;
  for (int i = threadIdx.x; i < vocab; i += SAMPLE_THREADS) {
    const float v = Elem<T>::load(x + i);
    if (v > mx) {
      sm = (mx == -INFINITY ? 0.0f : sm * expf(mx - v)) + 1.0f;
      mx = v;
    } else if (v > -INFINITY) {
      sm += expf(v - mx);
    }
    float score = v;
    if (temperature > 0.0f) {
      const float u = fmaxf(uniform_from_word(philox_first_word(base + static_cast<uint32_t>(i), k0, k1)), 1.0e-30f);
      score = __fdiv_rn(v, fmaxf(temperature, 1.0e-30f)) - logf(-logf(u));
    }
    best = better(best, Best{score, i});
  }
  (void)inv_t;
  // warp then block reduction
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    Best other{__shfl_xor_sync(0xffffffffu, best.score, o), __shfl_xor_sync(0xffffffffu, best.index, o)};
    best = better(best, other);
    const float omx = __shfl_xor_sync(0xffffffffu, mx, o), osm = __shfl_xor_sync(0xffffffffu, sm, o);
    const float nm = fmaxf(mx, omx);
    sm = (mx == -INFINITY ? 0.0f : sm * expf(mx - nm)) + (omx == -INFINITY ? 0.0f : osm * expf(omx - nm));
    mx = nm;
  }
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  if (lane == 0) { s_score[warp] = best.score; s_index[warp] = best.index; s_max[warp] = mx; s_sum[warp] = sm; }
  __syncthreads();
  if (warp != 0) return;
  best = Best{s_score[lane], s_index[lane]};
  mx = s_max[lane];
  sm = s_sum[lane];
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    Best other{__shfl_xor_sync(0xffffffffu, best.score, o), __shfl_xor_sync(0xffffffffu, best.index, o)};
    best = better(best, other);
    const float omx = __shfl_xor_sync(0xffffffffu, mx, o), osm = __shfl_xor_sync(0xffffffffu, sm, o);
    const float nm = fmaxf(mx, omx);
    sm = (mx == -INFINITY ? 0.0f : sm * expf(mx - nm)) + (omx == -INFINITY ? 0.0f : osm * expf(omx - nm));
    mx = nm;
  }
  if (lane != 0) return;

  int token = best.index < vocab ? best.index : 0;
  int length = 0;
  if (has_state) {
    length = st.lengths[row];
    if (st.force_eos_at != nullptr && st.force_eos_at[row] == length) token = st.eos_token_id;
  }
  const float logp = Elem<T>::load(x + token) - (mx + logf(sm));
  if (sampled_out != nullptr) sampled_out[row] = token;
  if (logp_out != nullptr) logp_out[row] = logp;
  if (!has_state) return;

  // bookkeeping of the slot scheduler: EOS beats the stop table beats the length limit
  if (length < st.capacity) {
    st.tokens[static_cast<int64_t>(row) * st.capacity + length] = token;
    st.logprobs[static_cast<int64_t>(row) * st.capacity + length] = logp;
  }
  int32_t value = 0;
  if (st.stop_table != nullptr) {
    value = st.stop_table[st.stop_offsets[row] + st.stop_states[row] * vocab + token];
    st.stop_states[row] = value & 65535;
  }
  int8_t reason = 0;
  if (token == st.eos_token_id && !st.ignore_eos[row]) reason = 1;
  else if (value >= 65536) reason = 2;
  else if (length + 1 >= st.limits[row]) reason = 3;
  st.lengths[row] = length + 1;
  st.rng_positions[row] += 1;
  st.reasons[row] = reason;
  st.alive[row] = reason == 0;
  st.pending[row] = reason == 0;
  st.input_tokens[row] = token;
}

}  // namespace cgym

using namespace cgym;

extern "C" int cgym_sample_record(const void* logits, const cgym_slot_state* state, const uint8_t* advance,
                                  int64_t* sampled_out, float* logp_out, int n_slots, int vocab, int dtype,
                                  cgym_stream_t stream) {
  CGYM_REQUIRE(state != nullptr && n_slots >= 0 && vocab > 0, "sample_record: bad arguments");
  CGYM_REQUIRE(state->seeds && state->temperatures && state->rng_positions && state->lengths && state->alive,
               "sample_record: slot state is incomplete");
  if (n_slots == 0) return 0;
  if (dtype == CGYM_F32)
    sample_kernel<float><<<n_slots, SAMPLE_THREADS, 0, as_stream(stream)>>>(
        static_cast<const float*>(logits), *state, true, advance, state->seeds, state->rng_positions,
        state->temperatures, state->rng_offsets, sampled_out, logp_out, vocab);
  else if (dtype == CGYM_BF16)
    sample_kernel<__nv_bfloat16><<<n_slots, SAMPLE_THREADS, 0, as_stream(stream)>>>(
        static_cast<const __nv_bfloat16*>(logits), *state, true, advance, state->seeds, state->rng_positions,
        state->temperatures, state->rng_offsets, sampled_out, logp_out, vocab);
  else
    return fail("sample_record: unsupported logits dtype %d", dtype);
  return check_launch("sample_record");
}

extern "C" int cgym_sample(int64_t* tokens, float* logprobs, const void* logits, const int64_t* seeds,
                           const int64_t* steps, const float* temperatures, const int64_t* rng_offsets, int rows,
                           int vocab, int dtype, cgym_stream_t stream) {
  CGYM_REQUIRE(rows >= 0 && vocab > 0 && seeds && steps && temperatures && tokens, "sample: bad arguments");
  if (rows == 0) return 0;
  cgym_slot_state none{};
  if (dtype == CGYM_F32)
    sample_kernel<float><<<rows, SAMPLE_THREADS, 0, as_stream(stream)>>>(
        static_cast<const float*>(logits), none, false, nullptr, seeds, steps, temperatures, rng_offsets, tokens,
        logprobs, vocab);
  else if (dtype == CGYM_BF16)
    sample_kernel<__nv_bfloat16><<<rows, SAMPLE_THREADS, 0, as_stream(stream)>>>(
        static_cast<const __nv_bfloat16*>(logits), none, false, nullptr, seeds, steps, temperatures, rng_offsets,
        tokens, logprobs, vocab);
  else
    return fail("sample: unsupported logits dtype %d", dtype);
  return check_launch("sample");
}
