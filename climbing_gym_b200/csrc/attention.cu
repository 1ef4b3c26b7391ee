// Paged grouped-query attention over the block-table KV cache.
//
// One kernel serves decode rows (one query at the end of its sequence) and prefill rows (query
// t of a packed prompt attends to cache positions [0, t]): row r reads positions [0, kv_lens[r])
// of its slot. Grid (rows, kv_heads, splits); each of the four warps of a CTA streams a strided
// share of the split's tokens with its own online-softmax state (fp32, running max), the warps
// are merged through shared memory, and splits through a small fp32 workspace + combine kernel.
// Scores are fp32 dot products of the model-dtype q and k; P is rounded to the model dtype before
// P.V (for e4m3 caches the per-token K scale multiplies the score and the V scale multiplies P
// before that rounding), accumulation is fp32, the result is rounded once on store.
#include "common.cuh"

namespace cgym {

constexpr int ATT_WARPS = 4;
constexpr int ATT_MAX_ACC = 32;  // G * D / 32 accumulators per lane

template <typename KV>
__device__ __forceinline__ float kv_load(const KV* p) { return Elem<KV>::load(p); }
template <>
__device__ __forceinline__ float kv_load<uint8_t>(const uint8_t* p) { return from_e4m3(*p); }

template <typename TQ, typename KV, int PER_LANE>
__global__ void __launch_bounds__(ATT_WARPS * 32)
paged_attention_kernel(TQ* __restrict__ out, const TQ* __restrict__ q, const int32_t* __restrict__ kv_lens,
                       const int32_t* __restrict__ slots, const uint8_t* __restrict__ active,
                       cgym_kv_layout kv, int layer, int n_q_heads, float scale, int n_splits,
                       float* __restrict__ workspace) {
  extern __shared__ float smem[];
  const int D = kv.head_dim, G = n_q_heads / kv.n_kv_heads, GD = G * D;
  float* qs = smem;                           // [G][D]
  float* w_acc = qs + GD;                     // [ATT_WARPS][G][D]
  float* w_m = w_acc + ATT_WARPS * GD;        // [ATT_WARPS][G]
  float* w_l = w_m + ATT_WARPS * G;           // [ATT_WARPS][G]
  const int row = blockIdx.x, kh = blockIdx.y, split = blockIdx.z;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int slot = slots != nullptr ? slots[row] : row;
  int len = kv_lens[row];
  if ((active != nullptr && !active[row]) || slot < 0 || len < 0) len = 0;
  for (int i = threadIdx.x; i < GD; i += blockDim.x)
    qs[i] = Elem<TQ>::load(q + (static_cast<int64_t>(row) * n_q_heads + kh * G) * D + i);
  __syncthreads();

  // this split's token range, in whole pages
  const int P = kv.page_size;
  const int n_blocks = (len + P - 1) / P;
  const int blocks_per_split = (n_blocks + n_splits - 1) / n_splits;
  const int t_begin = min(len, split * blocks_per_split * P);
  const int t_end = min(len, (split + 1) * blocks_per_split * P);

  constexpr int per_lane = PER_LANE;  // head_dim / 32
  float m[8], l[8], acc[8 * PER_LANE];
#pragma unroll
  for (int g = 0; g < 8; ++g) { m[g] = -INFINITY; l[g] = 0.0f; }
#pragma unroll
  for (int i = 0; i < 8 * PER_LANE; ++i) acc[i] = 0.0f;
  const KV* pool = static_cast<const KV*>(kv.kv_pool);
  const int32_t* table = kv.block_table + static_cast<int64_t>(slot < 0 ? 0 : slot) * kv.max_blocks;

  for (int t0 = t_begin + warp * 32; t0 < t_end; t0 += ATT_WARPS * 32) {
    const int tok = t0 + lane;
    const bool valid = tok < t_end;
    int page = 0;
    if (valid) page = table[tok / P];
    const bool ok = valid && page >= 0 && page < kv.n_pages;
    float s[8];
    float v_scale = 1.0f;
    if (ok) {
      const KV* block = pool + kv_block_offset(kv, layer, page, kh);
#pragma unroll
      for (int g = 0; g < 8; ++g) s[g] = 0.0f;
      for (int d = 0; d < D; ++d) {
        const float kd = kv_load<KV>(block + kv_row_index(tok % P, d, D, static_cast<int>(sizeof(KV))));
#pragma unroll
        for (int g = 0; g < 8; ++g)
          if (g < G) s[g] = fmaf(qs[g * D + d], kd, s[g]);
      }
      float k_scale = scale;
      if constexpr (sizeof(KV) == 1) {
        k_scale *= kv.kv_scales[kv_scale_offset(kv, layer, page, 0, kh, tok % P)];
        v_scale = kv.kv_scales[kv_scale_offset(kv, layer, page, 1, kh, tok % P)];
      }
#pragma unroll
      for (int g = 0; g < 8; ++g) s[g] *= k_scale;
    } else {
#pragma unroll
      for (int g = 0; g < 8; ++g) s[g] = -INFINITY;
    }
    float p[8];
#pragma unroll
    for (int g = 0; g < 8; ++g) {
      p[g] = 0.0f;
      if (g < G) {
        const float m_new = fmaxf(m[g], warp_max(s[g]));  // finite: lane 0 of a started chunk is valid
        const float alpha = (m[g] == -INFINITY) ? 0.0f : expf(m[g] - m_new);
        const float e = (ok && m_new > -INFINITY) ? expf(s[g] - m_new) : 0.0f;
        l[g] = l[g] * alpha + warp_sum(e);
        p[g] = Elem<TQ>::round(e * v_scale);
        m[g] = m_new;
#pragma unroll
        for (int j = 0; j < per_lane; ++j) acc[g * per_lane + j] *= alpha;
      }
    }
    const int n_here = min(32, t_end - t0);
    for (int tt = 0; tt < n_here; ++tt) {
      const int pg = __shfl_sync(0xffffffffu, page, tt);
      if (pg < 0 || pg >= kv.n_pages) continue;  // uniform across the warp
      const KV* vt = pool + kv_block_offset(kv, layer, pg, kh) + P * D;  // V^T part: row = dim
      float vv[PER_LANE];
#pragma unroll
      for (int j = 0; j < per_lane; ++j)
        vv[j] = kv_load<KV>(vt + kv_row_index(lane + 32 * j, (t0 + tt) % P, P, static_cast<int>(sizeof(KV))));
#pragma unroll
      for (int g = 0; g < 8; ++g) {
        if (g < G) {
          const float pg_val = __shfl_sync(0xffffffffu, p[g], tt);
#pragma unroll
          for (int j = 0; j < per_lane; ++j) acc[g * per_lane + j] = fmaf(pg_val, vv[j], acc[g * per_lane + j]);
        }
      }
    }
  }

  // merge the warps
#pragma unroll
  for (int g = 0; g < 8; ++g) {
    if (g < G) {
      if (lane == 0) { w_m[warp * G + g] = m[g]; w_l[warp * G + g] = l[g]; }
#pragma unroll
      for (int j = 0; j < per_lane; ++j) w_acc[(warp * G + g) * D + lane + 32 * j] = acc[g * per_lane + j];
    }
  }
  __syncthreads();
  for (int i = threadIdx.x; i < GD; i += blockDim.x) {
    const int g = i / D;
    float mm = -INFINITY;
    for (int w = 0; w < ATT_WARPS; ++w) mm = fmaxf(mm, w_m[w * G + g]);
    float total = 0.0f, value = 0.0f;
    for (int w = 0; w < ATT_WARPS; ++w) {
      const float f = (w_m[w * G + g] == -INFINITY) ? 0.0f : expf(w_m[w * G + g] - mm);
      total += f * w_l[w * G + g];
      value += f * w_acc[(w * G + g) * D + (i % D)];
    }
    const int head = kh * G + g;
    if (n_splits == 1) {
      Elem<TQ>::store(out + (static_cast<int64_t>(row) * n_q_heads + head) * D + (i % D),
                      value / fmaxf(total, 1.0e-20f));
    } else {
      const int64_t part = (static_cast<int64_t>(row) * n_q_heads + head) * n_splits + split;
      const int64_t n_parts = static_cast<int64_t>(gridDim.x) * n_q_heads * n_splits;
      workspace[part * D + (i % D)] = value;
      if ((i % D) == 0) {
        workspace[n_parts * D + part] = mm;
        workspace[n_parts * (D + 1) + part] = total;
      }
    }
  }
}

template <typename TQ>
__global__ void attention_combine_kernel(TQ* __restrict__ out, const float* __restrict__ workspace, int rows,
                                         int n_q_heads, int D, int n_splits) {
  const int row = blockIdx.x, head = blockIdx.y, d = threadIdx.x;
  const int64_t n_parts = static_cast<int64_t>(rows) * n_q_heads * n_splits;
  const int64_t part0 = (static_cast<int64_t>(row) * n_q_heads + head) * n_splits;
  float mm = -INFINITY;
  for (int s = 0; s < n_splits; ++s) mm = fmaxf(mm, workspace[n_parts * D + part0 + s]);
  float total = 0.0f, value = 0.0f;
  for (int s = 0; s < n_splits; ++s) {
    const float ms = workspace[n_parts * D + part0 + s];
    const float f = (ms == -INFINITY) ? 0.0f : expf(ms - mm);
    total += f * workspace[n_parts * (D + 1) + part0 + s];
    value += f * workspace[(part0 + s) * D + d];
  }
  Elem<TQ>::store(out + (static_cast<int64_t>(row) * n_q_heads + head) * D + d, value / fmaxf(total, 1.0e-20f));
}

}  // namespace cgym

using namespace cgym;

namespace cgym {
bool attention_mma_supported(const cgym_kv_layout* kv, int n_q_heads, int dtype);
int launch_decode_attention_mma(void* out, const void* q, const int32_t* kv_lens, const int32_t* slots,
                                const uint8_t* active, const cgym_kv_layout* kv, int layer, int rows, int n_q_heads,
                                float scale, int n_splits, float* workspace, int32_t* status, cudaStream_t stream);
int launch_prefill_attention_mma(void* out, const void* q, const int32_t* tile_row0, const int32_t* tile_ntok,
                                 const int32_t* tile_slot, const int32_t* tile_pos0, const cgym_kv_layout* kv, int layer,
                                 int n_tiles, int n_q_heads, float scale, int32_t* status, cudaStream_t stream);
}  // namespace cgym

extern "C" int cgym_prefill_attention(void* out, const void* q, const int32_t* tile_row0, const int32_t* tile_ntok,
                                      const int32_t* tile_slot, const int32_t* tile_pos0, const cgym_kv_layout* kv,
                                      int layer, int n_tiles, int n_q_heads, float scale, int dtype, int32_t* status,
                                      cgym_stream_t stream) {
  CGYM_REQUIRE(kv != nullptr && status != nullptr, "prefill_attention: kv layout and status are required");
  CGYM_REQUIRE(tile_row0 && tile_ntok && tile_slot && tile_pos0, "prefill_attention: tile lists are required");
  CGYM_REQUIRE(kv->n_kv_heads > 0 && n_q_heads % kv->n_kv_heads == 0, "prefill_attention: heads must group evenly");
  CGYM_REQUIRE(attention_mma_supported(kv, n_q_heads, dtype),
               "prefill_attention: needs bf16 activations, a bf16 or e4m3 cache, head_dim 64, 64-token pages, group <= 16");
  CGYM_REQUIRE(kv->kv_dtype != CGYM_E4M3 || kv->kv_scales != nullptr, "e4m3 KV needs a scale pool");
  if (n_tiles == 0) return 0;
  if (int rc = launch_prefill_attention_mma(out, q, tile_row0, tile_ntok, tile_slot, tile_pos0, kv, layer, n_tiles,
                                            n_q_heads, scale, status, as_stream(stream)))
    return rc;
  return check_launch("prefill_attention");
}

extern "C" int cgym_paged_attention(void* out, const void* q, const int32_t* kv_lens, const int32_t* slots,
                                    const uint8_t* active, const cgym_kv_layout* kv, int layer, int rows,
                                    int n_q_heads, float scale, int n_splits, float* workspace, int dtype,
                                    int impl, int32_t* status, cgym_stream_t stream) {
  CGYM_REQUIRE(kv != nullptr, "paged_attention: kv layout is required");
  const int D = kv->head_dim;
  CGYM_REQUIRE(D == 32 || D == 64 || D == 128 || D == 256, "paged_attention: head_dim must be 32, 64, 128 or 256");
  CGYM_REQUIRE(kv->n_kv_heads > 0 && n_q_heads % kv->n_kv_heads == 0, "paged_attention: heads must group evenly");
  const int G = n_q_heads / kv->n_kv_heads;
  CGYM_REQUIRE(n_splits >= 1 && n_splits <= 64, "paged_attention: n_splits must be in [1, 64]");
  CGYM_REQUIRE(n_splits == 1 || workspace != nullptr, "paged_attention: split-KV needs a workspace");
  CGYM_REQUIRE(kv->kv_dtype != CGYM_E4M3 || kv->kv_scales != nullptr, "e4m3 KV needs a scale pool");
  CGYM_REQUIRE(impl >= 0 && impl <= 2, "paged_attention: impl must be 0 (auto), 1 (CUDA cores) or 2 (tensor cores)");
  if (rows == 0) return 0;
  CGYM_REQUIRE(kv->n_kv_heads <= 65535 && n_q_heads <= 65535, "too many heads");
  const bool mma_ok = status != nullptr && attention_mma_supported(kv, n_q_heads, dtype);
  CGYM_REQUIRE(impl != 2 || mma_ok, "paged_attention: the tensor-core kernel needs bf16 activations, a bf16 or e4m3 "
                                    "cache, head_dim 64, 64-token pages, group <= 16 and a status word");
  if (impl == 2 || (impl == 0 && mma_ok)) {
    if (int rc = launch_decode_attention_mma(out, q, kv_lens, slots, active, kv, layer, rows, n_q_heads, scale, n_splits,
                                             workspace, status, as_stream(stream)))
      return rc;
    if (n_splits > 1) {
      if (dtype == CGYM_BF16)
        attention_combine_kernel<__nv_bfloat16><<<dim3(rows, n_q_heads), D, 0, as_stream(stream)>>>(
            static_cast<__nv_bfloat16*>(out), workspace, rows, n_q_heads, D, n_splits);
    }
    return check_launch("paged_attention", n_splits > 1 ? 2 : 1);
  }
  CGYM_REQUIRE(G <= 8 && G * D <= 32 * ATT_MAX_ACC, "paged_attention: group too large (G <= 8, G*D <= 1024)");
  dim3 grid(rows, kv->n_kv_heads, n_splits);
  const size_t smem = (static_cast<size_t>(G) * D * (1 + ATT_WARPS) + 2 * ATT_WARPS * G) * sizeof(float);
#define LAUNCH_ATT_D(TQ, KV, PL)                                                                         \
  paged_attention_kernel<TQ, KV, PL><<<grid, ATT_WARPS * 32, smem, as_stream(stream)>>>(                 \
      static_cast<TQ*>(out), static_cast<const TQ*>(q), kv_lens, slots, active, *kv, layer, n_q_heads,   \
      scale, n_splits, workspace)
#define LAUNCH_ATT(TQ, KV)                                                                               \
  do {                                                                                                   \
    if (D == 32) LAUNCH_ATT_D(TQ, KV, 1);                                                                \
    else if (D == 64) LAUNCH_ATT_D(TQ, KV, 2);                                                           \
    else if (D == 128) LAUNCH_ATT_D(TQ, KV, 4);                                                          \
    else LAUNCH_ATT_D(TQ, KV, 8);                                                                        \
    if (n_splits > 1)                                                                                    \
      attention_combine_kernel<TQ><<<dim3(rows, n_q_heads), D, 0, as_stream(stream)>>>(                  \
          static_cast<TQ*>(out), workspace, rows, n_q_heads, D, n_splits);                               \
  } while (0)
  if (dtype == CGYM_F32 && kv->kv_dtype == CGYM_F32) LAUNCH_ATT(float, float);
  else if (dtype == CGYM_BF16 && kv->kv_dtype == CGYM_BF16) LAUNCH_ATT(__nv_bfloat16, __nv_bfloat16);
  else if (dtype == CGYM_BF16 && kv->kv_dtype == CGYM_E4M3) LAUNCH_ATT(__nv_bfloat16, uint8_t);
  else return fail("paged_attention: unsupported dtype pair (%d, kv %d)", dtype, kv->kv_dtype);
#undef LAUNCH_ATT
#undef LAUNCH_ATT_D
  return check_launch("paged_attention", n_splits > 1 ? 2 : 1);
}
