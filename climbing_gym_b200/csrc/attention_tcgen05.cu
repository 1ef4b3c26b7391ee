// Prefill attention on the Blackwell tensor cores (tcgen05.mma, accumulators in TMEM), for bf16 KV caches
// with head_dim 64 and 64-token pages. Replaces flash_attn_func on the prompt path of the reference
// (src/climbing_gym/inference/lfm25_engine.py:1387-1389, 1415-1417); the e4m3 cache keeps the mma.sync kernel
// of attention_mma.cu (its operands need widening in registers).
//
// Tile: up to 128 (token, head) rows - 128 / G consecutive query tokens of one sequence times the G query
// heads of one KV head - against the causal range of pages of that sequence. Per page:
//     S  [128 x 64 tokens] = Q [128 x 64 dims] . K^T      tcgen05.mma, S in TMEM
//     P  = exp2(scale * S - running max), rounded to bf16  one thread per row (a TMEM lane is a row, so the
//                                                          row max and row sum need no shuffles), written to
//                                                          shared memory in the 128-byte-swizzled operand layout
//     O  [128 x 64 dims]  += P [128 x 64 tokens] . V       tcgen05.mma, O accumulates in TMEM over the pages
// The cache stores a (page, head) block as K [token][dim] followed by V^T [dim][token], rows of 128 bytes whose
// 16-byte chunks are XOR-ed with the row index: exactly the shared-memory image of a K-major SWIZZLE_128B
// operand, so a block is staged with ONE linear cp.async.bulk and used as the B operand of both products
// without any rearrangement. S is double-buffered in TMEM and P in shared memory, so the tensor pipe computes
// S of page i + 1 and P.V of page i while the softmax threads work on S of page i + 1.
//
// O stays in TMEM for the whole tile: P is taken relative to a reference maximum per row that is only moved
// when the row's running maximum has outgrown it by more than 2^8 (P <= 256 is exact enough in bf16 and far
// from overflow), so the usual per-page rescaling of O disappears. When a row does move its reference, its
// thread waits for the P.V products in flight (they write every row), rescales ITS lane of O in place
// (tcgen05.ld / tcgen05.st; the next P.V cannot start before this thread has delivered its P row) and goes on.
//
// Warp roles (192 threads): 0 = page producer, 1 = MMA issuer + TMEM owner, 2..5 = one row per thread.
// Every mbarrier wait is bounded (two seconds of %globaltimer): on expiry the CTA raises
// CGYM_STATUS_WAIT_TIMEOUT, lets its copies land, frees its TMEM and returns.
#include "common.cuh"

namespace cgym {

namespace fa {

constexpr int D = 64, P = 64, ROWS = 128;
constexpr int THREADS = 192;
constexpr int KV_STAGES = 3;                // 97 KB of shared memory per CTA: two CTAs share an SM
constexpr int PAGE_BYTES = 2 * P * D * 2;   // K + V^T of one (page, head), bf16
constexpr int Q_BYTES = ROWS * D * 2;       // 16 KB
constexpr int P_BYTES = ROWS * P * 2;       // 16 KB
constexpr int SMEM_BYTES = 1024 + Q_BYTES + 2 * P_BYTES + KV_STAGES * PAGE_BYTES;
constexpr int TMEM_COLS = 256;              // S0, S1, O: 64 fp32 columns each (allocations are powers of two)
constexpr float RESCALE_SLACK = 8.0f;       // log2 of the largest P a row may reach before its reference moves
constexpr unsigned long long WAIT_LIMIT_NS = 2000000000ull;

__device__ __forceinline__ uint32_t smem_u32(const void* p) { return static_cast<uint32_t>(__cvta_generic_to_shared(p)); }
__device__ __forceinline__ unsigned long long timer() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
  return t;
}
__device__ __forceinline__ void bar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}
__device__ __forceinline__ void bar_expect(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
}
__device__ __forceinline__ void bar_arrive(uint32_t bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}
__device__ __forceinline__ bool bar_try(uint32_t bar, uint32_t parity) {
  uint32_t done;
  asm volatile(
      "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\tselp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(done) : "r"(bar), "r"(parity) : "memory");
  return done != 0;
}
__device__ __forceinline__ bool bar_wait(uint32_t bar, uint32_t parity, volatile int* abort_flag) {
  if (bar_try(bar, parity)) return true;
  const unsigned long long start = timer();
  for (uint32_t spin = 1;; ++spin) {
    if (bar_try(bar, parity)) return true;
    if ((spin & 63u) == 0u) {
      if (*abort_flag) return false;
      if (timer() - start > WAIT_LIMIT_NS) {
        *abort_flag = 1;
        return false;
      }
    }
  }
}
__device__ __forceinline__ void bulk_copy(uint32_t dst, const void* src, uint32_t bytes, uint32_t bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
               ::"r"(dst), "l"(src), "r"(bytes), "r"(bar) : "memory");
}
// K-major operand of 128-byte rows, SWIZZLE_128B: 8-row groups 1024 bytes apart
__device__ __forceinline__ uint64_t operand_desc(uint32_t addr) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((addr >> 4) & 0x3FFF);
  d |= static_cast<uint64_t>(1) << 16;
  d |= static_cast<uint64_t>(1024 >> 4) << 32;
  d |= static_cast<uint64_t>(1) << 46;
  d |= static_cast<uint64_t>(2) << 61;
  return d;
}
__device__ __forceinline__ void mma_bf16(uint32_t tmem_d, uint64_t da, uint64_t db, uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}"
      ::"r"(tmem_d), "l"(da), "l"(db), "r"(idesc), "r"(accumulate)
      : "memory");
}
__device__ __forceinline__ void mma_commit(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar) : "memory");
}
// the 64 fp32 columns of this thread's TMEM lane, two loads in flight, one wait
__device__ __forceinline__ void tmem_load_row(uint32_t taddr, float (&v)[64]) {
  uint32_t r[64];
#pragma unroll
  for (int h = 0; h < 2; ++h)
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
        "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
        "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
        : "=r"(r[32 * h + 0]), "=r"(r[32 * h + 1]), "=r"(r[32 * h + 2]), "=r"(r[32 * h + 3]), "=r"(r[32 * h + 4]),
          "=r"(r[32 * h + 5]), "=r"(r[32 * h + 6]), "=r"(r[32 * h + 7]), "=r"(r[32 * h + 8]), "=r"(r[32 * h + 9]),
          "=r"(r[32 * h + 10]), "=r"(r[32 * h + 11]), "=r"(r[32 * h + 12]), "=r"(r[32 * h + 13]), "=r"(r[32 * h + 14]),
          "=r"(r[32 * h + 15]), "=r"(r[32 * h + 16]), "=r"(r[32 * h + 17]), "=r"(r[32 * h + 18]), "=r"(r[32 * h + 19]),
          "=r"(r[32 * h + 20]), "=r"(r[32 * h + 21]), "=r"(r[32 * h + 22]), "=r"(r[32 * h + 23]), "=r"(r[32 * h + 24]),
          "=r"(r[32 * h + 25]), "=r"(r[32 * h + 26]), "=r"(r[32 * h + 27]), "=r"(r[32 * h + 28]), "=r"(r[32 * h + 29]),
          "=r"(r[32 * h + 30]), "=r"(r[32 * h + 31])
        : "r"(taddr + 32 * h));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int j = 0; j < 64; ++j) v[j] = __uint_as_float(r[j]);
}
__device__ __forceinline__ void tmem_store_row(uint32_t taddr, const float (&v)[64]) {
#pragma unroll
  for (int h = 0; h < 2; ++h)
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
        "{%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16, "
        "%17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32};"
        ::"r"(taddr + 32 * h), "r"(__float_as_uint(v[32 * h + 0])), "r"(__float_as_uint(v[32 * h + 1])),
          "r"(__float_as_uint(v[32 * h + 2])), "r"(__float_as_uint(v[32 * h + 3])), "r"(__float_as_uint(v[32 * h + 4])),
          "r"(__float_as_uint(v[32 * h + 5])), "r"(__float_as_uint(v[32 * h + 6])), "r"(__float_as_uint(v[32 * h + 7])),
          "r"(__float_as_uint(v[32 * h + 8])), "r"(__float_as_uint(v[32 * h + 9])), "r"(__float_as_uint(v[32 * h + 10])),
          "r"(__float_as_uint(v[32 * h + 11])), "r"(__float_as_uint(v[32 * h + 12])), "r"(__float_as_uint(v[32 * h + 13])),
          "r"(__float_as_uint(v[32 * h + 14])), "r"(__float_as_uint(v[32 * h + 15])), "r"(__float_as_uint(v[32 * h + 16])),
          "r"(__float_as_uint(v[32 * h + 17])), "r"(__float_as_uint(v[32 * h + 18])), "r"(__float_as_uint(v[32 * h + 19])),
          "r"(__float_as_uint(v[32 * h + 20])), "r"(__float_as_uint(v[32 * h + 21])), "r"(__float_as_uint(v[32 * h + 22])),
          "r"(__float_as_uint(v[32 * h + 23])), "r"(__float_as_uint(v[32 * h + 24])), "r"(__float_as_uint(v[32 * h + 25])),
          "r"(__float_as_uint(v[32 * h + 26])), "r"(__float_as_uint(v[32 * h + 27])), "r"(__float_as_uint(v[32 * h + 28])),
          "r"(__float_as_uint(v[32 * h + 29])), "r"(__float_as_uint(v[32 * h + 30])), "r"(__float_as_uint(v[32 * h + 31]))
        : "memory");
  asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ float fast_exp2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

struct Tiles {
  const int32_t* row0;   // packed row of the tile's first query token
  const int32_t* ntok;   // query tokens in the tile (<= 128 / G)
  const int32_t* slot;   // cache slot of the sequence
  const int32_t* pos0;   // cache position of the tile's first query token
};

// byte offset of 16-byte chunk `chunk` of row `row` in a [rows][128 B] SWIZZLE_128B operand tile
__device__ __forceinline__ uint32_t swizzled(int row, int chunk) { return row * 128 + ((chunk ^ (row & 7)) << 4); }

__global__ void __launch_bounds__(THREADS, 2)
prefill_attention_tcgen05_kernel(__nv_bfloat16* __restrict__ out, const __nv_bfloat16* __restrict__ q, Tiles tiles,
                                 cgym_kv_layout kv, int layer, int n_q_heads, float scale,
                                 int32_t* __restrict__ status) {
  extern __shared__ uint8_t smem_raw[];
  __shared__ __align__(8) uint64_t bar_q, bar_kv_full[KV_STAGES], bar_kv_empty[KV_STAGES];
  __shared__ __align__(8) uint64_t bar_s_full[2], bar_s_free[2], bar_p_full[2], bar_pv_done[2];
  __shared__ uint32_t tmem_slot;
  __shared__ int abort_flag;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int tile = blockIdx.x, kh = blockIdx.y;
  const int G = n_q_heads / kv.n_kv_heads;
  const int row0 = tiles.row0[tile], ntok = tiles.ntok[tile], slot = tiles.slot[tile], pos0 = tiles.pos0[tile];
  const int n_rows = ntok * G;                      // (token, head) rows of this tile, <= 128
  const int n_pages = (pos0 + ntok + P - 1) / P;    // causal range of the tile's last token
  const uint32_t base = (smem_u32(smem_raw) + 1023u) & ~1023u;
  const uint32_t q_tile = base, p_tile = base + Q_BYTES, kv_ring = base + Q_BYTES + 2 * P_BYTES;

  if (threadIdx.x == 0) {
    abort_flag = 0;
    bar_init(smem_u32(&bar_q), 128);
    for (int s = 0; s < KV_STAGES; ++s) { bar_init(smem_u32(&bar_kv_full[s]), 1); bar_init(smem_u32(&bar_kv_empty[s]), 1); }
    for (int b = 0; b < 2; ++b) {
      bar_init(smem_u32(&bar_s_full[b]), 1);
      bar_init(smem_u32(&bar_s_free[b]), 128);
      bar_init(smem_u32(&bar_p_full[b]), 128);
      bar_init(smem_u32(&bar_pv_done[b]), 1);
    }
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&tmem_slot)),
                 "r"(TMEM_COLS) : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  const uint32_t tmem = tmem_slot;
  const uint32_t tmem_s[2] = {tmem, tmem + 64}, tmem_o = tmem + 128;

  if (warp == 0) {
    // ---- page producer: one linear bulk copy per (page, head) block ----
    if (lane == 0) {
      const int32_t* table = kv.block_table + static_cast<int64_t>(slot) * kv.max_blocks;
      const uint8_t* pool = static_cast<const uint8_t*>(kv.kv_pool);
      int issued = 0;
      for (int i = 0; i < n_pages; ++i) {
        const int s = i % KV_STAGES;
        if (i >= KV_STAGES && !bar_wait(smem_u32(&bar_kv_empty[s]), ((i / KV_STAGES) & 1) ^ 1, &abort_flag)) break;
        int page = table[i];
        if (page < 0 || page >= kv.n_pages) { atomicOr(status, CGYM_STATUS_BAD_PAGE); page = 0; }
        const uint32_t full = smem_u32(&bar_kv_full[s]);
        bar_expect(full, PAGE_BYTES);
        bulk_copy(kv_ring + s * PAGE_BYTES, pool + kv_block_offset(kv, layer, page, kh) * 2, PAGE_BYTES, full);
        issued = i + 1;
      }
      if (abort_flag)
        for (int i = max(0, issued - KV_STAGES); i < issued; ++i)
          bar_wait(smem_u32(&bar_kv_full[i % KV_STAGES]), (i / KV_STAGES) & 1, &abort_flag);
    }
  } else if (warp == 1) {
    // ---- MMA issuer ----
    if (lane == 0) {
      // fp32 accumulate, bf16 K-major operands, N = 64, M = 128
      const uint32_t idesc = (1u << 4) | (1u << 7) | (1u << 10) | (static_cast<uint32_t>(64 >> 3) << 17) |
                             (static_cast<uint32_t>(128 >> 4) << 24);
      const uint64_t dq = operand_desc(q_tile);
      bool ok = bar_wait(smem_u32(&bar_q), 0, &abort_flag);
      auto issue_pv = [&](int i) {  // O += P[i % 2] . V of page i
        const int b = i & 1, s = i % KV_STAGES;
        if (!bar_wait(smem_u32(&bar_p_full[b]), (i >> 1) & 1, &abort_flag)) return false;
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        const uint64_t dp = operand_desc(p_tile + b * P_BYTES), dv = operand_desc(kv_ring + s * PAGE_BYTES + P * D * 2);
#pragma unroll
        for (int k = 0; k < P / 16; ++k) mma_bf16(tmem_o, dp + 2 * k, dv + 2 * k, idesc, (i > 0 || k > 0) ? 1u : 0u);
        mma_commit(smem_u32(&bar_pv_done[b]));
        mma_commit(smem_u32(&bar_kv_empty[s]));  // the page is free once both products have read it
        return true;
      };
      for (int i = 0; ok && i < n_pages; ++i) {
        const int b = i & 1, s = i % KV_STAGES;
        if (!bar_wait(smem_u32(&bar_kv_full[s]), (i / KV_STAGES) & 1, &abort_flag)) { ok = false; break; }
        if (i >= 2 && !bar_wait(smem_u32(&bar_s_free[b]), ((i >> 1) & 1) ^ 1, &abort_flag)) { ok = false; break; }
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        const uint64_t dk = operand_desc(kv_ring + s * PAGE_BYTES);
#pragma unroll
        for (int k = 0; k < D / 16; ++k) mma_bf16(tmem_s[b], dq + 2 * k, dk + 2 * k, idesc, k > 0 ? 1u : 0u);
        mma_commit(smem_u32(&bar_s_full[b]));
        if (i >= 1) ok = issue_pv(i - 1);
      }
      if (ok && n_pages > 0) issue_pv(n_pages - 1);
    }
  } else {
    // ---- one (token, head) row per thread ----
    const int quarter = warp & 3;                       // TMEM lanes [32 quarter, +32) belong to this warp
    const int r = quarter * 32 + lane;                  // row of the tile
    const bool valid = r < n_rows;
    const int limit = valid ? pos0 + r / G + 1 : 0;     // the row attends to cache positions [0, limit)
    const uint32_t lane_addr = static_cast<uint32_t>(quarter * 32) << 16;
    // Q row -> shared memory, in the operand layout (rows beyond the tile are zero)
    {
      const uint4* src = reinterpret_cast<const uint4*>(
          q + (static_cast<int64_t>(row0 + (valid ? r / G : 0)) * n_q_heads + kh * G + (valid ? r % G : 0)) * D);
#pragma unroll
      for (int c = 0; c < 8; ++c) {
        const uint4 v = valid ? src[c] : make_uint4(0, 0, 0, 0);
        asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(q_tile + swizzled(r, c)), "r"(v.x), "r"(v.y),
                     "r"(v.z), "r"(v.w) : "memory");
      }
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      bar_arrive(smem_u32(&bar_q));
    }
    float ref = -INFINITY, l = 0.0f;  // reference maximum (log2 domain) the row's P values are taken against
    const float scale_log2 = scale * 1.4426950408889634f;
    bool ok = true;
    for (int i = 0; i < n_pages; ++i) {
      const int b = i & 1;
      if (!bar_wait(smem_u32(&bar_s_full[b]), (i >> 1) & 1, &abort_flag)) { ok = false; break; }
      asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
      float s[P];
      tmem_load_row(tmem_s[b] + lane_addr, s);
      asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
      bar_arrive(smem_u32(&bar_s_free[b]));
      // causal mask (only the pages that straddle the row's limit need it), maximum of the raw scores
      const int first = i * P;
      if (first + P > limit) {
#pragma unroll
        for (int j = 0; j < P; ++j)
          if (first + j >= limit) s[j] = -INFINITY;
      }
      float row_max = s[0];
#pragma unroll
      for (int j = 1; j < P; ++j) row_max = fmaxf(row_max, s[j]);
      row_max *= scale_log2;  // scale > 0: scaling commutes with the maximum
      // P buffer b was last read by the P.V of page i - 2: it must have completed before the row is overwritten
      if (i >= 2 && !bar_wait(smem_u32(&bar_pv_done[b]), ((i - 2) >> 1) & 1, &abort_flag)) { ok = false; break; }
      if (row_max > ref + RESCALE_SLACK || (ref == -INFINITY && row_max > -INFINITY)) {
        // move the reference; what the row has accumulated so far is rescaled in place
        if (i >= 1 && ref > -INFINITY) {
          if (!bar_wait(smem_u32(&bar_pv_done[(i - 1) & 1]), ((i - 1) >> 1) & 1, &abort_flag)) { ok = false; break; }
          asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
          const float factor = fast_exp2(ref - row_max);
          float acc[D];
          tmem_load_row(tmem_o + lane_addr, acc);
#pragma unroll
          for (int d = 0; d < D; ++d) acc[d] *= factor;
          tmem_store_row(tmem_o + lane_addr, acc);
          asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
          l *= factor;
        }
        ref = row_max;
      }
      const bool empty = ref == -INFINITY;  // nothing to attend to (rows beyond the tile)
      const float shift = empty ? 0.0f : -ref;
      float sum = 0.0f;
      uint32_t packed[P / 2];
#pragma unroll
      for (int j = 0; j < P; j += 2) {
        // masked scores are -inf: fma(-inf, scale, shift) = -inf and exp2(-inf) = 0
        const float p0 = empty ? 0.0f : fast_exp2(fmaf(s[j], scale_log2, shift));
        const float p1 = empty ? 0.0f : fast_exp2(fmaf(s[j + 1], scale_log2, shift));
        const __nv_bfloat162 pair = __floats2bfloat162_rn(p0, p1);
        sum += p0 + p1;  // the row sum adds the fp32 values; only the tensor-core operand is rounded
        packed[j / 2] = *reinterpret_cast<const uint32_t*>(&pair);
      }
      l += sum;
#pragma unroll
      for (int c = 0; c < 8; ++c)
        asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(p_tile + b * P_BYTES + swizzled(r, c)),
                     "r"(packed[4 * c]), "r"(packed[4 * c + 1]), "r"(packed[4 * c + 2]), "r"(packed[4 * c + 3]) : "memory");
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      bar_arrive(smem_u32(&bar_p_full[b]));
    }
    float o[D];
    if (ok && n_pages > 0) {
      if (bar_wait(smem_u32(&bar_pv_done[(n_pages - 1) & 1]), ((n_pages - 1) >> 1) & 1, &abort_flag)) {
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        tmem_load_row(tmem_o + lane_addr, o);
      } else {
        ok = false;
      }
    }
    if (ok && valid) {
      const float inv = 1.0f / fmaxf(l, 1.0e-20f);
      uint4* dst = reinterpret_cast<uint4*>(out + (static_cast<int64_t>(row0 + r / G) * n_q_heads + kh * G + (r % G)) * D);
#pragma unroll
      for (int c = 0; c < 8; ++c) {
        uint4 v;
        __nv_bfloat162 a = __floats2bfloat162_rn(o[8 * c] * inv, o[8 * c + 1] * inv);
        __nv_bfloat162 bb = __floats2bfloat162_rn(o[8 * c + 2] * inv, o[8 * c + 3] * inv);
        __nv_bfloat162 cc = __floats2bfloat162_rn(o[8 * c + 4] * inv, o[8 * c + 5] * inv);
        __nv_bfloat162 dd = __floats2bfloat162_rn(o[8 * c + 6] * inv, o[8 * c + 7] * inv);
        v.x = *reinterpret_cast<uint32_t*>(&a);
        v.y = *reinterpret_cast<uint32_t*>(&bb);
        v.z = *reinterpret_cast<uint32_t*>(&cc);
        v.w = *reinterpret_cast<uint32_t*>(&dd);
        dst[c] = v;
      }
    }
  }

  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  if (threadIdx.x == 0 && abort_flag) atomicOr(status, CGYM_STATUS_WAIT_TIMEOUT);
  if (warp == 1) {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(TMEM_COLS) : "memory");
  }
}

}  // namespace fa

bool prefill_attention_tcgen05_supported(const cgym_kv_layout* kv, int n_q_heads) {
  if (kv->kv_dtype != CGYM_BF16 || kv->page_size != 64 || kv->head_dim != 64) return false;
  const int G = n_q_heads / kv->n_kv_heads;
  return G >= 1 && G <= 16 && n_q_heads % kv->n_kv_heads == 0;
}

int launch_prefill_attention_tcgen05(void* out, const void* q, const int32_t* tile_row0, const int32_t* tile_ntok,
                                     const int32_t* tile_slot, const int32_t* tile_pos0, const cgym_kv_layout* kv,
                                     int layer, int n_tiles, int n_q_heads, float scale, int32_t* status,
                                     cudaStream_t stream) {
  CGYM_REQUIRE((reinterpret_cast<uintptr_t>(q) & 15u) == 0 && (reinterpret_cast<uintptr_t>(out) & 15u) == 0,
               "prefill_attention(tcgen05): q and out must be 16-byte aligned");
  static SmemReservation reservation;
  if (int rc = reserve_dynamic_smem(fa::prefill_attention_tcgen05_kernel, fa::SMEM_BYTES, reservation,
                                    "prefill_attention(tcgen05)"))
    return rc;
  const fa::Tiles tiles{tile_row0, tile_ntok, tile_slot, tile_pos0};
  fa::prefill_attention_tcgen05_kernel<<<dim3(n_tiles, kv->n_kv_heads), fa::THREADS, fa::SMEM_BYTES, stream>>>(
      static_cast<__nv_bfloat16*>(out), static_cast<const __nv_bfloat16*>(q), tiles, *kv, layer, n_q_heads, scale, status);
  return 0;
}

}  // namespace cgym
