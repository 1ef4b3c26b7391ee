// Fused sampler: Gumbel-max / greedy draw, sampled-token log-prob from the untempered logits and
// (optionally) the slot scheduler's per-row bookkeeping, in one launch and one pass over the logits.
//
// Uniforms are Philox-4x32-10 (Salmon et al., SC'11) keyed per row with
// key = (seed + position * 0x9E3779B97F4A7C15) & (2^63 - 1), counter (offset + column, 0, 0, 0),
// first output word, mapped to [0,1) by folding the sign of its int32 view and scaling by 2^-31:
// the stream the reference sampler consumes, so a row's draws do not depend on which slot or
// batch it occupies. Ties resolve to the lowest token id.
//
// Grid (rows, parts): each CTA reduces one slice of a row's vocabulary (the work is Philox-bound,
// so a row is spread over several SMs); with parts > 1 the CTA that arrives last at the row's
// counter combines the slices in slice order (deterministic) and does the bookkeeping. The
// workspace holds 4 floats per (row, part) plus one counter per row, zero between launches.
#include <mutex>

#include "common.cuh"

namespace cgym {

constexpr int SAMPLE_THREADS = 512;
constexpr int SAMPLE_MAX_PARTS = 16;

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

struct Pick {
  float score;
  int index;
  float mx;  // running maximum of the raw logits
  float sm;  // sum of exp(logit - mx)
};

__device__ __forceinline__ Pick combine(Pick a, Pick b) {
  Pick r = a;
  if (b.score > a.score || (b.score == a.score && b.index < a.index)) { r.score = b.score; r.index = b.index; }
  const float nm = fmaxf(a.mx, b.mx);
  r.sm = (a.mx == -INFINITY ? 0.0f : a.sm * expf(a.mx - nm)) + (b.mx == -INFINITY ? 0.0f : b.sm * expf(b.mx - nm));
  r.mx = nm;
  return r;
}

__device__ __forceinline__ Pick shuffle_xor(Pick p, int o) {
  Pick q;
  q.score = __shfl_xor_sync(0xffffffffu, p.score, o);
  q.index = __shfl_xor_sync(0xffffffffu, p.index, o);
  q.mx = __shfl_xor_sync(0xffffffffu, p.mx, o);
  q.sm = __shfl_xor_sync(0xffffffffu, p.sm, o);
  return q;
}

// eight consecutive logits, 16-byte aligned
__device__ __forceinline__ void load8(const float* p, float* out) {
  const float4 a = *reinterpret_cast<const float4*>(p), b = *reinterpret_cast<const float4*>(p + 4);
  out[0] = a.x; out[1] = a.y; out[2] = a.z; out[3] = a.w;
  out[4] = b.x; out[5] = b.y; out[6] = b.z; out[7] = b.w;
}
__device__ __forceinline__ void load8(const __nv_bfloat16* p, float* out) {
  const uint4 raw = *reinterpret_cast<const uint4*>(p);
  const __nv_bfloat162* pairs = reinterpret_cast<const __nv_bfloat162*>(&raw);
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const float2 f = __bfloat1622float2(pairs[j]);
    out[2 * j] = f.x;
    out[2 * j + 1] = f.y;
  }
}

template <typename T>
__global__ void __launch_bounds__(SAMPLE_THREADS)
sample_kernel(const T* __restrict__ logits, cgym_slot_state st, bool has_state,
              const uint8_t* __restrict__ advance, const int64_t* __restrict__ seeds,
              const int64_t* __restrict__ steps, const float* __restrict__ temperatures,
              const int64_t* __restrict__ rng_offsets, int64_t* __restrict__ sampled_out,
              float* __restrict__ logp_out, int vocab, float* __restrict__ workspace) {
  __shared__ Pick s_pick[SAMPLE_THREADS / 32];
  __shared__ int s_last;
  pdl_trigger();
  pdl_wait();
  const int row = blockIdx.x, part = blockIdx.y, parts = gridDim.y;
  if (has_state) {
    if (threadIdx.x == 0 && part == 0 && advance != nullptr && advance[row]) st.seq_lens[row] += 1;
    if (!st.alive[row]) return;
  }
  const float temperature = temperatures[row];
  const uint64_t key = (static_cast<uint64_t>(seeds[row]) +
                        static_cast<uint64_t>(steps[row]) * 0x9E3779B97F4A7C15ull) & 0x7FFFFFFFFFFFFFFFull;
  const uint32_t k0 = static_cast<uint32_t>(key), k1 = static_cast<uint32_t>(key >> 32);
  const uint32_t base = rng_offsets != nullptr ? static_cast<uint32_t>(rng_offsets[row]) : 0u;
  const T* x = logits + static_cast<int64_t>(row) * vocab;

  Pick mine{-INFINITY, 0x7fffffff, -INFINITY, 0.0f};
  const float t_div = fmaxf(temperature, 1.0e-30f);
  // support of the draw: logits below the row's threshold (top-k / top-p) are never candidates
  const float floor = (has_state && st.min_logits != nullptr) ? st.min_logits[row] : -INFINITY;
  // Gumbel-max score of element i (x / 1 is exact, so the division is skipped at temperature 1)
  // log(-log(u)) of this row, drawn ahead of the logits by gumbel_noise_kernel (same Philox stream, same
  // float operations, so the draw is bit-identical), or evaluated here
  const float* noise = (has_state && st.gumbel_noise != nullptr) ? st.gumbel_noise + static_cast<int64_t>(row) * vocab
                                                                 : nullptr;
  auto consider = [&](int i, float v) {
    if (v < floor) return;
    float score = v;
    if (temperature > 0.0f) {
      float g;
      if (noise != nullptr) {
        g = noise[i];
      } else {
        const float u = fmaxf(uniform_from_word(philox_first_word(base + static_cast<uint32_t>(i), k0, k1)), 1.0e-30f);
        g = logf(-logf(u));
      }
      score = (temperature == 1.0f ? v : __fdiv_rn(v, t_div)) - g;
    }
    if (score > mine.score || (score == mine.score && i < mine.index)) { mine.score = score; mine.index = i; }
  };
  const bool wide = vocab % 8 == 0 && (reinterpret_cast<uintptr_t>(logits) & 15u) == 0;
  if (wide) {
    // eight consecutive logits per thread and step (one or two 16-byte loads): a thread walks its
    // slice in a few memory round trips, and the eight Philox chains of a group run side by side
    const int groups = vocab / 8, per_part = (groups + parts - 1) / parts;
    const int g_end = min(groups, (part + 1) * per_part);
    for (int g = part * per_part + threadIdx.x; g < g_end; g += SAMPLE_THREADS) {
      float v[8];
      load8(x + static_cast<int64_t>(g) * 8, v);
      float top = v[0];
#pragma unroll
      for (int j = 1; j < 8; ++j) top = fmaxf(top, v[j]);
      if (top > mine.mx) {
        mine.sm = mine.mx == -INFINITY ? 0.0f : mine.sm * expf(mine.mx - top);
        mine.mx = top;
      }
      if (mine.mx > -INFINITY) {
#pragma unroll
        for (int j = 0; j < 8; ++j) mine.sm += expf(v[j] - mine.mx);  // exp(-inf) = 0 for masked logits
      }
#pragma unroll
      for (int j = 0; j < 8; ++j) consider(g * 8 + j, v[j]);
    }
  } else {
    const int chunk = (vocab + parts - 1) / parts;
    const int begin = part * chunk, end = min(vocab, begin + chunk);
    for (int i = begin + threadIdx.x; i < end; i += SAMPLE_THREADS) {
      const float v = Elem<T>::load(x + i);
      if (v > mine.mx) {
        mine.sm = (mine.mx == -INFINITY ? 0.0f : mine.sm * expf(mine.mx - v)) + 1.0f;
        mine.mx = v;
      } else if (v > -INFINITY) {
        mine.sm += expf(v - mine.mx);
      }
      consider(i, v);
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) mine = combine(mine, shuffle_xor(mine, o));
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  if (lane == 0) s_pick[warp] = mine;
  __syncthreads();
  if (warp != 0) return;
  mine = lane < SAMPLE_THREADS / 32 ? s_pick[lane] : Pick{-INFINITY, 0x7fffffff, -INFINITY, 0.0f};
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) mine = combine(mine, shuffle_xor(mine, o));

  if (parts > 1) {
    // publish this slice; the last CTA to arrive folds all slices in slice order
    float* slot = workspace + (static_cast<int64_t>(row) * SAMPLE_MAX_PARTS + part) * 4;
    int* counter = reinterpret_cast<int*>(workspace + static_cast<int64_t>(gridDim.x) * SAMPLE_MAX_PARTS * 4) + row;
    if (lane == 0) {
      slot[0] = mine.score;
      slot[1] = __int_as_float(mine.index);
      slot[2] = mine.mx;
      slot[3] = mine.sm;
      __threadfence();
      const int arrived = atomicAdd(counter, 1);
      s_last = arrived == parts - 1;
      if (s_last) *counter = 0;
    }
    __syncwarp();
    if (!s_last) return;
    __threadfence();
    if (lane == 0) {
      const float* all = workspace + static_cast<int64_t>(row) * SAMPLE_MAX_PARTS * 4;
      mine = Pick{__ldcg(all), __float_as_int(__ldcg(all + 1)), __ldcg(all + 2), __ldcg(all + 3)};
      for (int p = 1; p < parts; ++p)
        mine = combine(mine, Pick{__ldcg(all + 4 * p), __float_as_int(__ldcg(all + 4 * p + 1)), __ldcg(all + 4 * p + 2),
                                  __ldcg(all + 4 * p + 3)});
    }
  }
  if (lane != 0) return;

  int token = mine.index < vocab ? mine.index : 0;
  int length = 0;
  if (has_state) {
    length = st.lengths[row];
    if (st.force_eos_at != nullptr && st.force_eos_at[row] == length) token = st.eos_token_id;
  }
  const float logp = Elem<T>::load(x + token) - (mine.mx + logf(mine.sm));
  if (sampled_out != nullptr) sampled_out[row] = token;
  if (logp_out != nullptr) logp_out[row] = logp;
  if (!has_state) return;

  // bookkeeping of the slot scheduler: EOS beats the stop table beats the length limit
  if (length < st.capacity) {
    // a slot's tokens go to its own arena row, or to the row its request was given (device-side slot turnover)
    const int64_t out_row = st.out_rows != nullptr ? st.out_rows[row] : row;
    st.tokens[out_row * st.capacity + length] = token;
    st.logprobs[out_row * st.capacity + length] = logp;
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

// The Gumbel noise of a step does not depend on the step's logits: key and counter come from the row's
// seed, its position and the column. This kernel evaluates log(-log(u)) for every alive, tempered row while
// the layers of the step are still running (it is launched on a side stream at the start of the step: the
// ten Philox rounds per logit are ALU work that fits beside the latency-bound GEMM chain), and the sampler
// then only subtracts it. Grid (rows, parts); eight columns per thread and iteration, 16-byte stores.
__global__ void __launch_bounds__(SAMPLE_THREADS)
gumbel_noise_kernel(float* __restrict__ noise, cgym_slot_state st, int vocab) {
  const int row = blockIdx.x, part = blockIdx.y, parts = gridDim.y;
  if (!st.alive[row] || !(st.temperatures[row] > 0.0f)) return;
  const uint64_t key = (static_cast<uint64_t>(st.seeds[row]) +
                        static_cast<uint64_t>(st.rng_positions[row]) * 0x9E3779B97F4A7C15ull) & 0x7FFFFFFFFFFFFFFFull;
  const uint32_t k0 = static_cast<uint32_t>(key), k1 = static_cast<uint32_t>(key >> 32);
  const uint32_t base = st.rng_offsets != nullptr ? static_cast<uint32_t>(st.rng_offsets[row]) : 0u;
  float* out = noise + static_cast<int64_t>(row) * vocab;
  auto draw = [&](int i) {
    const float u = fmaxf(uniform_from_word(philox_first_word(base + static_cast<uint32_t>(i), k0, k1)), 1.0e-30f);
    return logf(-logf(u));
  };
  if (vocab % 8 == 0 && (reinterpret_cast<uintptr_t>(noise) & 15u) == 0) {
    const int groups = vocab / 8, per_part = (groups + parts - 1) / parts;
    const int g_end = min(groups, (part + 1) * per_part);
    for (int g = part * per_part + threadIdx.x; g < g_end; g += SAMPLE_THREADS) {
      float4 a, b;
      a.x = draw(g * 8), a.y = draw(g * 8 + 1), a.z = draw(g * 8 + 2), a.w = draw(g * 8 + 3);
      b.x = draw(g * 8 + 4), b.y = draw(g * 8 + 5), b.z = draw(g * 8 + 6), b.w = draw(g * 8 + 7);
      reinterpret_cast<float4*>(out + g * 8)[0] = a;
      reinterpret_cast<float4*>(out + g * 8)[1] = b;
    }
  } else {
    const int chunk = (vocab + parts - 1) / parts;
    const int begin = part * chunk, end = min(vocab, begin + chunk);
    for (int i = begin + threadIdx.x; i < end; i += SAMPLE_THREADS) out[i] = draw(i);
  }
}

static int pick_parts(int rows, int vocab, const float* workspace, bool noise_ready = false) {
  if (workspace == nullptr || vocab < 8192) return 1;
  // With the Gumbel noise drawn ahead (gumbel_noise_kernel) a slice is two loads, an exponential and a
  // compare per logit: a CTA's fixed cost (launch, block reductions, the merge through the workspace) then
  // outweighs its share of the row, so take as few slices as still give every resident slot a CTA.
  if (noise_ready) {
    int parts = (2 * 148) / (rows > 0 ? rows : 1);
    if (parts > vocab / 4096) parts = vocab / 4096;
    if (parts > SAMPLE_MAX_PARTS) parts = SAMPLE_MAX_PARTS;
    return parts < 1 ? 1 : parts;
  }
  // Two 512-thread CTAs fit an SM (62 registers per thread), i.e. 296 CTAs run at once. The kernel's time
  // is the number of such waves times a slice's share of the row, so pick the slice count that minimises
  // waves / parts (64 rows: 4 slices fill one wave where 5 would start a second; 256 rows: 8 slices leave
  // a short last wave), with a small charge per slice for its part of the final merge.
  int by_vocab = vocab / 4096;
  if (by_vocab > SAMPLE_MAX_PARTS) by_vocab = SAMPLE_MAX_PARTS;
  int best = 1;
  double best_cost = 1.0e30;
  for (int parts = 1; parts <= by_vocab; ++parts) {
    const int waves = (rows * parts + 2 * 148 - 1) / (2 * 148);
    const double cost = static_cast<double>(waves) / parts + 0.01 * parts;
    if (cost < best_cost) { best_cost = cost; best = parts; }
  }
  return best;
}

// ---- top-k / top-p support thresholds ---------------------------------------------------------------
// Floats map to unsigned keys whose order is the floats' order; the k-th largest logit and the top-p
// cut are then found bit by bit from the most significant bit down, each probe being one pass over
// the row with a fixed-tree block reduction (counts, or tempered softmax mass), so the result does not
// depend on timing. bf16 rows are staged once in shared memory as 16-bit keys (only those 16 bits
// are searched); fp32 rows are re-read from L2 on every probe (test-sized vocabularies).
constexpr int FILTER_THREADS = 1024;

__device__ __forceinline__ uint32_t ordered_key(float v) {
  const uint32_t u = __float_as_uint(v);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}
__device__ __forceinline__ float key_value(uint32_t key) {
  return __uint_as_float((key & 0x80000000u) ? (key ^ 0x80000000u) : ~key);
}
__device__ __forceinline__ uint32_t block_max_u32(uint32_t v, uint32_t* scratch) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nwarps = (blockDim.x + 31) >> 5;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = max(v, __shfl_xor_sync(0xffffffffu, v, o));
  __syncthreads();
  if (lane == 0) scratch[warp] = v;
  __syncthreads();
  uint32_t r = lane < nwarps ? scratch[lane] : 0u;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) r = max(r, __shfl_xor_sync(0xffffffffu, r, o));
  return r;
}

template <typename T>
__global__ void __launch_bounds__(FILTER_THREADS)
filter_threshold_kernel(float* __restrict__ min_logits, const T* __restrict__ logits,
                        const float* __restrict__ temperatures, const int32_t* __restrict__ top_k,
                        const float* __restrict__ top_p, const uint8_t* __restrict__ alive, int vocab) {
  constexpr bool HALF = sizeof(T) == 2;
  constexpr int LOW_BIT = HALF ? 16 : 0;  // bf16 keys have no information below bit 16
  extern __shared__ uint16_t staged[];    // bf16: the row's keys
  __shared__ float scratch[32];
  __shared__ uint32_t uscratch[32];
  pdl_trigger();
  pdl_wait();
  const int row = blockIdx.x;
  const float temperature = temperatures[row];
  const int k = top_k != nullptr ? top_k[row] : 0;
  const float p = top_p != nullptr ? top_p[row] : 1.0f;
  const bool use_k = k > 0 && k < vocab, use_p = p < 1.0f;
  if ((alive != nullptr && !alive[row]) || !(temperature > 0.0f) || (!use_k && !use_p)) {  // uniform per CTA
    if (threadIdx.x == 0) min_logits[row] = -INFINITY;
    return;
  }
  const T* x = logits + static_cast<int64_t>(row) * vocab;
  if (HALF) {
    for (int i = threadIdx.x; i < vocab; i += FILTER_THREADS) staged[i] = static_cast<uint16_t>(ordered_key(Elem<T>::load(x + i)) >> 16);
    __syncthreads();
  }
  auto key_at = [&](int i) -> uint32_t {
    if (HALF) return static_cast<uint32_t>(staged[i]) << 16;
    return ordered_key(Elem<T>::load(x + i));
  };
  // a 16-bit key stands for a bf16 value: keys of negative values are complemented bits, so the 16
  // dropped low bits come back as ones before the key is turned into its float again
  auto value_of = [&](uint32_t key) -> float {
    return key_value((HALF && !(key & 0x80000000u)) ? (key | 0xFFFFu) : key);
  };

  uint32_t tau_k = 0u;  // keys >= tau_k survive top-k
  if (use_k) {
    for (int bit = 31; bit >= LOW_BIT; --bit) {
      const uint32_t probe = tau_k | (1u << bit);
      float count = 0.0f;  // exact: counts stay far below 2^24
      for (int i = threadIdx.x; i < vocab; i += FILTER_THREADS) count += key_at(i) >= probe ? 1.0f : 0.0f;
      if (block_sum(count, scratch) >= static_cast<float>(k)) tau_k = probe;  // the k-th largest key is >= probe
    }
  }
  uint32_t tau = tau_k;
  if (use_p) {
    uint32_t top = 0u;
    for (int i = threadIdx.x; i < vocab; i += FILTER_THREADS) top = max(top, key_at(i));
    top = block_max_u32(top, uscratch);
    const float v_top = value_of(top);
    auto mass_from = [&](uint32_t floor_key) {  // tempered softmax mass (relative to the maximum) of keys >= floor_key
      float mass = 0.0f;
      for (int i = threadIdx.x; i < vocab; i += FILTER_THREADS) {
        const uint32_t key = key_at(i);
        if (key >= floor_key) mass += expf(__fdiv_rn(value_of(key) - v_top, temperature));
      }
      return block_sum(mass, scratch);
    };
    const float budget = p * mass_from(tau_k);
    // the largest key whose tail mass (within the top-k survivors) still exceeds the budget; the
    // predicate holds for every key <= tau_k and never again once it failed, so the bits can be fixed
    // from the top
    uint32_t over = 0u;
    for (int bit = 31; bit >= LOW_BIT; --bit) {
      const uint32_t probe = over | (1u << bit);
      if (mass_from(max(probe, tau_k)) > budget) over = probe;
    }
    // every key above `over` has a tail mass within the budget; the most probable value always stays
    uint32_t tau_p = over + (1u << LOW_BIT);
    if (tau_p < over || tau_p > top) tau_p = top;
    tau = max(tau_k, tau_p);
  }
  if (threadIdx.x == 0) min_logits[row] = tau == 0u ? -INFINITY : value_of(tau);
}

// ---- behaviour head: the k most probable tokens of the unfiltered distribution -----------------------
// Per live row: log Z (max + log-sum-exp), the key of the k-th largest logit by the same bit-wise
// search, the ties at that key resolved towards the lowest token ids (a second search, on the index),
// then exactly k candidates are gathered and sorted by (logit descending, id ascending) with a
// bitonic network in shared memory. Deterministic throughout.
constexpr int HEAD_MAX_K = 128;

template <typename T>
__global__ void __launch_bounds__(FILTER_THREADS)
topk_head_kernel(int32_t* __restrict__ out_ids, float* __restrict__ out_logprobs, const T* __restrict__ logits,
                 const uint8_t* __restrict__ alive, const int32_t* __restrict__ lengths, int vocab, int capacity,
                 int k) {
  constexpr bool HALF = sizeof(T) == 2;
  constexpr int LOW_BIT = HALF ? 16 : 0;
  extern __shared__ uint16_t staged[];
  __shared__ float scratch[32];
  __shared__ unsigned long long picked[HEAD_MAX_K];
  __shared__ int n_picked;
  pdl_trigger();
  pdl_wait();
  const int row = blockIdx.x;
  const int position = lengths != nullptr ? lengths[row] : 0;
  if ((alive != nullptr && !alive[row]) || position >= capacity) return;  // uniform per CTA
  const T* x = logits + static_cast<int64_t>(row) * vocab;
  if (HALF) {
    for (int i = threadIdx.x; i < vocab; i += FILTER_THREADS) staged[i] = static_cast<uint16_t>(ordered_key(Elem<T>::load(x + i)) >> 16);
  }
  if (threadIdx.x < HEAD_MAX_K) picked[threadIdx.x] = 0ull;
  if (threadIdx.x == 0) n_picked = 0;
  __syncthreads();
  auto key_at = [&](int i) -> uint32_t {
    if (HALF) return static_cast<uint32_t>(staged[i]) << 16;
    return ordered_key(Elem<T>::load(x + i));
  };
  // a 16-bit key stands for a bf16 value: keys of negative values are complemented bits, so the 16
  // dropped low bits come back as ones before the key is turned into its float again
  auto value_of = [&](uint32_t key) -> float {
    return key_value((HALF && !(key & 0x80000000u)) ? (key | 0xFFFFu) : key);
  };
  // log Z
  float top = -INFINITY;
  for (int i = threadIdx.x; i < vocab; i += FILTER_THREADS) top = fmaxf(top, value_of(key_at(i)));
  top = block_max(top, scratch);
  float mass = 0.0f;
  for (int i = threadIdx.x; i < vocab; i += FILTER_THREADS) mass += expf(value_of(key_at(i)) - top);
  const float log_z = top + logf(block_sum(mass, scratch));
  // key of the k-th largest logit
  uint32_t tau = 0u;
  for (int bit = 31; bit >= LOW_BIT; --bit) {
    const uint32_t probe = tau | (1u << bit);
    float count = 0.0f;
    for (int i = threadIdx.x; i < vocab; i += FILTER_THREADS) count += key_at(i) >= probe ? 1.0f : 0.0f;
    if (block_sum(count, scratch) >= static_cast<float>(k)) tau = probe;
  }
  float above = 0.0f;
  for (int i = threadIdx.x; i < vocab; i += FILTER_THREADS) above += key_at(i) > tau ? 1.0f : 0.0f;
  const int need = k - static_cast<int>(block_sum(above, scratch));  // ties at tau to take, >= 1
  // the largest index such that at most `need` ties lie at or below it: ties are taken in id order
  int last_tie = 0;
  for (int bit = 30; bit >= 0; --bit) {
    const int probe = last_tie | (1 << bit);
    if (probe >= vocab) continue;
    float below = 0.0f;  // ties with index < probe
    for (int i = threadIdx.x; i < vocab && i < probe; i += FILTER_THREADS) below += key_at(i) == tau ? 1.0f : 0.0f;
    if (block_sum(below, scratch) < static_cast<float>(need)) last_tie = probe;
  }
  // gather exactly k candidates as (key, ~index) so that one descending sort orders ties by ascending id
  for (int i = threadIdx.x; i < vocab; i += FILTER_THREADS) {
    const uint32_t key = key_at(i);
    if (key > tau || (key == tau && i <= last_tie)) {
      const int slot = atomicAdd(&n_picked, 1);
      if (slot < HEAD_MAX_K) picked[slot] = (static_cast<unsigned long long>(key) << 32) | (0xFFFFFFFFu - static_cast<uint32_t>(i));
    }
  }
  __syncthreads();
  // bitonic sort of 128 entries, descending (empty entries are 0 and sink to the end)
  for (int size = 2; size <= HEAD_MAX_K; size <<= 1) {
    for (int stride = size >> 1; stride > 0; stride >>= 1) {
      if (threadIdx.x < HEAD_MAX_K) {
        const int partner = threadIdx.x ^ stride;
        if (partner > static_cast<int>(threadIdx.x)) {
          const bool descending = (threadIdx.x & size) == 0;
          const unsigned long long a = picked[threadIdx.x], b = picked[partner];
          if ((a < b) == descending) { picked[threadIdx.x] = b; picked[partner] = a; }
        }
      }
      __syncthreads();
    }
  }
  if (threadIdx.x < k) {
    const unsigned long long entry = picked[threadIdx.x];
    const int64_t at = (static_cast<int64_t>(row) * capacity + position) * k + threadIdx.x;
    out_ids[at] = static_cast<int32_t>(0xFFFFFFFFu - static_cast<uint32_t>(entry & 0xFFFFFFFFull));
    out_logprobs[at] = value_of(static_cast<uint32_t>(entry >> 32)) - log_z;
  }
}

// ---- repetition penalty ---------------------------------------------------------------------------------
// out[row][i] = fp32 logit, with the logits of tokens the row has seen (its prompt and everything it
// generated) multiplied by the penalty when negative and divided by it otherwise. `seen` is one byte per
// (row, token); the row's latest token (tokens[row][lengths[row] - 1]) is folded in here and marked for
// the steps to come, so the sampler needs no hook of its own. grid (ceil(vocab / 2048), rows).
constexpr int PENALTY_THREADS = 256;

template <typename T>
__global__ void __launch_bounds__(PENALTY_THREADS)
repetition_penalty_kernel(float* __restrict__ out, const T* __restrict__ logits, uint8_t* __restrict__ seen,
                          const int64_t* __restrict__ tokens, const int32_t* __restrict__ lengths,
                          const uint8_t* __restrict__ alive, const float* __restrict__ penalties, int vocab,
                          int capacity) {
  pdl_trigger();
  pdl_wait();
  logits = pdl_fresh(logits);  // written by the kernels before this one: no load may move above the wait
  tokens = pdl_fresh(tokens);
  lengths = pdl_fresh(lengths);
  alive = pdl_fresh(alive);
  const int row = blockIdx.y;
  if (alive != nullptr && !alive[row]) return;
  const float penalty = penalties[row];
  const int length = lengths != nullptr ? min(lengths[row], capacity) : 0;
  const int latest = (tokens != nullptr && length > 0) ? static_cast<int>(tokens[static_cast<int64_t>(row) * capacity + length - 1]) : -1;
  const T* x = logits + static_cast<int64_t>(row) * vocab;
  uint8_t* mark = seen + static_cast<int64_t>(row) * vocab;
  float* y = out + static_cast<int64_t>(row) * vocab;
  auto penalised = [&](int i, float v, uint8_t flag) {
    if (!flag && i != latest) return v;
    return v < 0.0f ? v * penalty : __fdiv_rn(v, penalty);
  };
  const int begin = (blockIdx.x * PENALTY_THREADS + threadIdx.x) * 8;
  if (begin >= vocab) return;
  if ((vocab & 7) == 0) {
    float v[8];
    load8(x + begin, v);
    const uint2 flags = *reinterpret_cast<const uint2*>(mark + begin);
    const uint8_t* f = reinterpret_cast<const uint8_t*>(&flags);
#pragma unroll
    for (int j = 0; j < 8; ++j) v[j] = penalised(begin + j, v[j], f[j]);
    *reinterpret_cast<float4*>(y + begin) = make_float4(v[0], v[1], v[2], v[3]);
    *reinterpret_cast<float4*>(y + begin + 4) = make_float4(v[4], v[5], v[6], v[7]);
  } else {
    for (int i = begin; i < min(vocab, begin + 8); ++i) y[i] = penalised(i, Elem<T>::load(x + i), mark[i]);
  }
  // exactly one thread owns the latest token's byte: it is the one that just read it
  if (latest >= begin && latest < begin + 8 && latest < vocab) mark[latest] = 1;
}

}  // namespace cgym

using namespace cgym;

extern "C" int cgym_repetition_penalty(float* out, const void* logits, uint8_t* seen, const int64_t* tokens,
                                       const int32_t* lengths, const uint8_t* alive, const float* penalties,
                                       int rows, int vocab, int capacity, int dtype, cgym_stream_t stream) {
  CGYM_REQUIRE(out && logits && seen && penalties && rows >= 0 && vocab > 0, "repetition_penalty: bad arguments");
  CGYM_REQUIRE(tokens == nullptr || (lengths != nullptr && capacity > 0),
               "repetition_penalty: tokens need lengths and a capacity");
  if (rows == 0) return 0;
  const dim3 grid((vocab + PENALTY_THREADS * 8 - 1) / (PENALTY_THREADS * 8), rows);
  if (dtype == CGYM_BF16) {
    launch_dependent(repetition_penalty_kernel<__nv_bfloat16>, grid, dim3(PENALTY_THREADS), 0, as_stream(stream), out,
                     static_cast<const __nv_bfloat16*>(logits), seen, tokens, lengths, alive, penalties, vocab, capacity);
  } else if (dtype == CGYM_F32) {
    launch_dependent(repetition_penalty_kernel<float>, grid, dim3(PENALTY_THREADS), 0, as_stream(stream), out,
                     static_cast<const float*>(logits), seen, tokens, lengths, alive, penalties, vocab, capacity);
  } else {
    return fail("repetition_penalty: unsupported logits dtype %d", dtype);
  }
  return check_launch("repetition_penalty");
}

extern "C" int cgym_filter_thresholds(float* min_logits, const void* logits, const float* temperatures,
                                      const int32_t* top_k, const float* top_p, const uint8_t* alive, int rows,
                                      int vocab, int dtype, cgym_stream_t stream) {
  CGYM_REQUIRE(min_logits && logits && temperatures && rows >= 0 && vocab > 0, "filter_thresholds: bad arguments");
  CGYM_REQUIRE(vocab <= FILTER_THREADS * 64, "filter_thresholds: vocabularies up to %d entries", FILTER_THREADS * 64);
  if (rows == 0) return 0;
  if (dtype == CGYM_BF16) {
    const int smem = vocab * static_cast<int>(sizeof(uint16_t));
    static SmemReservation reservation;
    if (int rc = reserve_dynamic_smem(filter_threshold_kernel<__nv_bfloat16>, smem, reservation, "filter_thresholds"))
      return rc;
    launch_dependent(filter_threshold_kernel<__nv_bfloat16>, dim3(rows), dim3(FILTER_THREADS), smem, as_stream(stream),
                     min_logits, static_cast<const __nv_bfloat16*>(logits), temperatures, top_k, top_p, alive, vocab);
  } else if (dtype == CGYM_F32) {
    launch_dependent(filter_threshold_kernel<float>, dim3(rows), dim3(FILTER_THREADS), 0, as_stream(stream), min_logits,
                     static_cast<const float*>(logits), temperatures, top_k, top_p, alive, vocab);
  } else {
    return fail("filter_thresholds: unsupported logits dtype %d", dtype);
  }
  return check_launch("filter_thresholds");
}

extern "C" int cgym_topk_head(int32_t* out_ids, float* out_logprobs, const void* logits, const uint8_t* alive,
                              const int32_t* lengths, int n_slots, int vocab, int capacity, int k, int dtype,
                              cgym_stream_t stream) {
  CGYM_REQUIRE(out_ids && out_logprobs && logits && n_slots >= 0 && vocab > 0 && capacity > 0, "topk_head: bad arguments");
  CGYM_REQUIRE(k > 0 && k <= HEAD_MAX_K && k <= vocab, "topk_head: k must be in [1, min(vocab, %d)]", HEAD_MAX_K);
  CGYM_REQUIRE(vocab <= FILTER_THREADS * 64, "topk_head: vocabularies up to %d entries", FILTER_THREADS * 64);
  if (n_slots == 0) return 0;
  if (dtype == CGYM_BF16) {
    const int smem = vocab * static_cast<int>(sizeof(uint16_t));
    static SmemReservation reservation;
    if (int rc = reserve_dynamic_smem(topk_head_kernel<__nv_bfloat16>, smem, reservation, "topk_head")) return rc;
    launch_dependent(topk_head_kernel<__nv_bfloat16>, dim3(n_slots), dim3(FILTER_THREADS), smem, as_stream(stream), out_ids,
                     out_logprobs, static_cast<const __nv_bfloat16*>(logits), alive, lengths, vocab, capacity, k);
  } else if (dtype == CGYM_F32) {
    launch_dependent(topk_head_kernel<float>, dim3(n_slots), dim3(FILTER_THREADS), 0, as_stream(stream), out_ids,
                     out_logprobs, static_cast<const float*>(logits), alive, lengths, vocab, capacity, k);
  } else {
    return fail("topk_head: unsupported logits dtype %d", dtype);
  }
  return check_launch("topk_head");
}

extern "C" int64_t cgym_sample_workspace_bytes(int rows) {
  return (static_cast<int64_t>(rows) * SAMPLE_MAX_PARTS * 4 + rows) * 4;
}

extern "C" int cgym_sample_record(const void* logits, const cgym_slot_state* state, const uint8_t* advance,
                                  int64_t* sampled_out, float* logp_out, int n_slots, int vocab, int dtype,
                                  float* workspace, cgym_stream_t stream) {
  CGYM_REQUIRE(state != nullptr && n_slots >= 0 && vocab > 0, "sample_record: bad arguments");
  CGYM_REQUIRE(state->seeds && state->temperatures && state->rng_positions && state->lengths && state->alive,
               "sample_record: slot state is incomplete");
  if (n_slots == 0) return 0;
  const dim3 grid(n_slots, pick_parts(n_slots, vocab, workspace, state->gumbel_noise != nullptr));
  if (dtype == CGYM_F32)
    launch_dependent(sample_kernel<float>, grid, dim3(SAMPLE_THREADS), 0, as_stream(stream),
                     static_cast<const float*>(logits), *state, true, advance, state->seeds, state->rng_positions,
                     state->temperatures, state->rng_offsets, sampled_out, logp_out, vocab, workspace);
  else if (dtype == CGYM_BF16)
    launch_dependent(sample_kernel<__nv_bfloat16>, grid, dim3(SAMPLE_THREADS), 0, as_stream(stream),
                     static_cast<const __nv_bfloat16*>(logits), *state, true, advance, state->seeds,
                     state->rng_positions, state->temperatures, state->rng_offsets, sampled_out, logp_out, vocab,
                     workspace);
  else
    return fail("sample_record: unsupported logits dtype %d", dtype);
  return check_launch("sample_record");
}

extern "C" int cgym_gumbel_noise(float* noise, const cgym_slot_state* state, int n_slots, int vocab,
                                 cgym_stream_t stream) {
  CGYM_REQUIRE(noise != nullptr && state != nullptr && n_slots >= 0 && vocab > 0, "gumbel_noise: bad arguments");
  CGYM_REQUIRE(state->seeds && state->temperatures && state->rng_positions && state->alive,
               "gumbel_noise: slot state is incomplete");
  if (n_slots == 0) return 0;
  int parts = vocab / 4096;
  parts = parts < 1 ? 1 : (parts > SAMPLE_MAX_PARTS ? SAMPLE_MAX_PARTS : parts);
  gumbel_noise_kernel<<<dim3(n_slots, parts), SAMPLE_THREADS, 0, as_stream(stream)>>>(noise, *state, vocab);
  return check_launch("gumbel_noise");
}

extern "C" int cgym_sample(int64_t* tokens, float* logprobs, const void* logits, const int64_t* seeds,
                           const int64_t* steps, const float* temperatures, const int64_t* rng_offsets, int rows,
                           int vocab, int dtype, float* workspace, cgym_stream_t stream) {
  CGYM_REQUIRE(rows >= 0 && vocab > 0 && seeds && steps && temperatures && tokens, "sample: bad arguments");
  if (rows == 0) return 0;
  cgym_slot_state none{};
  const dim3 grid(rows, pick_parts(rows, vocab, workspace));
  if (dtype == CGYM_F32)
    sample_kernel<float><<<grid, SAMPLE_THREADS, 0, as_stream(stream)>>>(
        static_cast<const float*>(logits), none, false, nullptr, seeds, steps, temperatures, rng_offsets, tokens,
        logprobs, vocab, workspace);
  else if (dtype == CGYM_BF16)
    sample_kernel<__nv_bfloat16><<<grid, SAMPLE_THREADS, 0, as_stream(stream)>>>(
        static_cast<const __nv_bfloat16*>(logits), none, false, nullptr, seeds, steps, temperatures, rng_offsets,
        tokens, logprobs, vocab, workspace);
  else
    return fail("sample: unsupported logits dtype %d", dtype);
  return check_launch("sample");
}

// ---- sampler whose slice scratch lives in the library image ---------------------------------
// Same kernel and slicing as cgym_sample with a workspace, but the workspace is a fixed array of
// this module, so the call needs no memory from the caller and requests none from the runtime.

constexpr int SAMPLE_STATIC_MAX_ROWS = CGYM_SAMPLE_STATIC_MAX_ROWS;
constexpr int SAMPLE_STATIC_FLOATS = SAMPLE_STATIC_MAX_ROWS * SAMPLE_MAX_PARTS * 4 + SAMPLE_STATIC_MAX_ROWS;  // 130 KiB
constexpr int SAMPLE_STATIC_MAX_DEVICES = 64;

static __device__ __align__(256) float g_sample_scratch[SAMPLE_STATIC_FLOATS];

static std::mutex g_sample_static_mutex;
static float* g_sample_scratch_ptr[SAMPLE_STATIC_MAX_DEVICES] = {};

// Address of this device's copy of the scratch array, resolved once per device with that device
// current (every device that loads the module has its own copy of the array).
static int sample_scratch_for_current_device(float** out) {
  int device = -1;
  cudaError_t err = cudaGetDevice(&device);
  if (err != cudaSuccess) return fail("sample_static: cudaGetDevice failed: %s", cudaGetErrorString(err));
  if (device < 0 || device >= SAMPLE_STATIC_MAX_DEVICES)
    return fail("sample_static: device ordinal %d is beyond the %d this entry point keeps scratch for", device,
                SAMPLE_STATIC_MAX_DEVICES);
  std::lock_guard<std::mutex> lock(g_sample_static_mutex);
  if (g_sample_scratch_ptr[device] == nullptr) {
    float* ptr = nullptr;
    err = cudaGetSymbolAddress(reinterpret_cast<void**>(&ptr), g_sample_scratch);
    if (err != cudaSuccess || ptr == nullptr)
      return fail("sample_static: cudaGetSymbolAddress failed on device %d: %s", device, cudaGetErrorString(err));
    g_sample_scratch_ptr[device] = ptr;
  }
  *out = g_sample_scratch_ptr[device];
  return 0;
}

extern "C" int cgym_sample_static(int64_t* tokens, float* logprobs, const void* logits, const int64_t* seeds,
                                  const int64_t* steps, const float* temperatures, const int64_t* rng_offsets,
                                  int rows, int vocab, int dtype, cgym_stream_t stream) {
  CGYM_REQUIRE(rows >= 0 && vocab > 0, "sample_static: bad arguments");
  if (rows > SAMPLE_STATIC_MAX_ROWS)
    return fail("sample_static: %d rows exceed the built-in scratch (at most %d rows per call); split the batch or "
                "use cgym_sample with a caller-owned workspace", rows, SAMPLE_STATIC_MAX_ROWS);
  CGYM_REQUIRE(dtype == CGYM_F32 || dtype == CGYM_BF16, "sample_static: unsupported logits dtype");
  float* scratch = nullptr;
  if (sample_scratch_for_current_device(&scratch) != 0) return 1;
  if (rows == 0) return 0;  // set-up only
  CGYM_REQUIRE(seeds && steps && temperatures && tokens && logits, "sample_static: bad arguments");
  // the per-row arrival counters must read zero when the kernel starts; the slices need no clearing
  float* counters = scratch + static_cast<int64_t>(rows) * SAMPLE_MAX_PARTS * 4;
  cudaError_t err = cudaMemsetAsync(counters, 0, sizeof(int) * rows, as_stream(stream));
  if (err != cudaSuccess) return fail("sample_static: clearing the counters failed: %s", cudaGetErrorString(err));
  cgym_slot_state none{};
  const dim3 grid(rows, pick_parts(rows, vocab, scratch));
  if (dtype == CGYM_F32)
    sample_kernel<float><<<grid, SAMPLE_THREADS, 0, as_stream(stream)>>>(
        static_cast<const float*>(logits), none, false, nullptr, seeds, steps, temperatures, rng_offsets, tokens,
        logprobs, vocab, scratch);
  else
    sample_kernel<__nv_bfloat16><<<grid, SAMPLE_THREADS, 0, as_stream(stream)>>>(
        static_cast<const __nv_bfloat16*>(logits), none, false, nullptr, seeds, steps, temperatures, rng_offsets,
        tokens, logprobs, vocab, scratch);
  return check_launch("sample_static");
}
