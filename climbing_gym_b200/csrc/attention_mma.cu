// Tensor-core paged attention for bf16 and e4m3 KV caches (head_dim 64, 64-token pages).
//
// Data movement: a (page, kv_head) block of the cache - K as [token][dim] followed by V^T as
// [dim][token], 16-byte chunks already XOR-swizzled in global memory - is brought into shared memory
// by ONE cp.async.bulk (TMA bulk copy, mbarrier completion), e4m3 caches add one 512-byte copy of the
// per-token scales. Fragment loads are bank-conflict free: ldmatrix.x4 on bf16 pages, one 16-byte load
// per K row / V^T row on e4m3 pages (32-bit loads remain where registers are short).
//
// Math: S = Q.K^T and O += P.V on mma.sync m16n8k16 with fp32 accumulation; an m-tile is 16
// (token, head) rows of one GQA group, so the G query heads that share a KV head reuse every staged
// byte. Softmax is online in fp32 (exp2 domain, running max). P is rounded to the MMA input type
// before P.V: bf16 for bf16 caches; for e4m3 caches K and V are widened to fp16 (exact) and the
// per-token K scale multiplies the score, the V scale multiplies P before its rounding.
//
// decode kernel : one query token per row, grid (rows, kv_heads, splits); the four warps of a CTA
//                 take pages round-robin, each with its own 1- to 3-page bulk-copy ring and softmax
//                 state, merged through shared memory (and splits through an fp32 workspace).
// prefill kernel: a CTA owns up to 128 / G consecutive query tokens of one sequence for one KV head;
//                 a producer warp streams the causal range of pages through a 4-stage ring that the
//                 eight consumer warps (one m-tile each) share.
// Every mbarrier wait is bounded; on expiry the CTA flags CGYM_STATUS_WAIT_TIMEOUT and drains.
#include <cuda_fp16.h>

#include "common.cuh"

namespace cgym {

constexpr unsigned long long ATT_WAIT_LIMIT_NS = 2000000000ull;

__device__ __forceinline__ uint32_t att_smem_u32(const void* p) { return static_cast<uint32_t>(__cvta_generic_to_shared(p)); }
__device__ __forceinline__ unsigned long long att_timer() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
  return t;
}
__device__ __forceinline__ void att_bar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}
__device__ __forceinline__ void att_bar_expect(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
}
__device__ __forceinline__ void att_bar_arrive(uint32_t bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}
__device__ __forceinline__ bool att_bar_try(uint32_t bar, uint32_t parity) {
  uint32_t done;
  asm volatile(
      "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\tselp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(done) : "r"(bar), "r"(parity) : "memory");
  return done != 0;
}
__device__ __forceinline__ bool att_bar_wait(uint32_t bar, uint32_t parity, volatile int* abort_flag) {
  if (att_bar_try(bar, parity)) return true;
  const unsigned long long start = att_timer();
  for (uint32_t spin = 1;; ++spin) {
    if (att_bar_try(bar, parity)) return true;
    if ((spin & 63u) == 0u) {
      if (*abort_flag) return false;
      if (att_timer() - start > ATT_WAIT_LIMIT_NS) {
        *abort_flag = 1;
        return false;
      }
    }
  }
}
// linear global -> shared bulk copy; both addresses 16-byte aligned, size a multiple of 16
__device__ __forceinline__ void att_bulk_copy(uint32_t dst, const void* src, uint32_t bytes, uint32_t bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
               ::"r"(dst), "l"(src), "r"(bytes), "r"(bar) : "memory");
}
__device__ __forceinline__ uint32_t att_lds32(uint32_t addr) {
  uint32_t v;
  asm volatile("ld.shared.b32 %0, [%1];" : "=r"(v) : "r"(addr));
  return v;
}
__device__ __forceinline__ void att_lds128(uint32_t addr, uint32_t (&v)[4]) {
  asm volatile("ld.shared.v4.b32 {%0, %1, %2, %3}, [%4];" : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]) : "r"(addr));
}
__device__ __forceinline__ void att_lds128f(uint32_t addr, float (&v)[4]) {
  asm volatile("ld.shared.v4.f32 {%0, %1, %2, %3}, [%4];" : "=f"(v[0]), "=f"(v[1]), "=f"(v[2]), "=f"(v[3]) : "r"(addr));
}
// four 8 x 8 b16 matrices; lane l supplies the address of row l % 8 of matrix l / 8
__device__ __forceinline__ void att_ldmatrix_x4(uint32_t addr, uint32_t (&v)[4]) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]) : "r"(addr));
}
__device__ __forceinline__ float att_lds_f32(uint32_t addr) {
  float v;
  asm volatile("ld.shared.f32 %0, [%1];" : "=f"(v) : "r"(addr));
  return v;
}

template <bool F16>
__device__ __forceinline__ void att_mma(float (&c)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  if constexpr (F16) {
    asm volatile("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
                 : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
                 : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
  } else {
    asm volatile("mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
                 : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
                 : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
  }
}

template <bool F16>
__device__ __forceinline__ uint32_t att_pack(float lo, float hi) {
  if constexpr (F16) {
    const __half2 h = __floats2half2_rn(lo, hi);
    return *reinterpret_cast<const uint32_t*>(&h);
  } else {
    const __nv_bfloat162 h = __floats2bfloat162_rn(lo, hi);
    return *reinterpret_cast<const uint32_t*>(&h);
  }
}
// two e4m3 codes (low 16 bits) -> packed fp16x2 (exact)
__device__ __forceinline__ uint32_t att_e4m3x2_to_f16x2(uint32_t two_codes) {
  uint32_t out;
  asm volatile("{\n\t.reg .b16 t;\n\tcvt.u16.u32 t, %1;\n\tcvt.rn.f16x2.e4m3x2 %0, t;\n\t}" : "=r"(out) : "r"(two_codes));
  return out;
}

// four e4m3 codes -> two packed fp16x2 (exact): codes 0, 1 and codes 2, 3
__device__ __forceinline__ void att_e4m3x4_to_f16x4(uint32_t four_codes, uint32_t& lo, uint32_t& hi) {
  asm("{\n\t.reg .b16 a, b;\n\tmov.b32 {a, b}, %2;\n\tcvt.rn.f16x2.e4m3x2 %0, a;\n\tcvt.rn.f16x2.e4m3x2 %1, b;\n\t}"
      : "=r"(lo), "=r"(hi) : "r"(four_codes));
}

// Geometry of one staged (page, head) block for cache element size EB, head_dim D, page size P.
template <int EB, int D, int P>
struct BlockGeom {
  static constexpr int K_ROW = D * EB;          // bytes per K row (one token)
  static constexpr int V_ROW = P * EB;          // bytes per V^T row (one dim)
  static constexpr int K_CPR = K_ROW / 16;
  static constexpr int V_CPR = V_ROW / 16;
  static constexpr int K_BYTES = P * K_ROW;
  static constexpr int BLOCK_BYTES = 2 * P * D * EB;
  static constexpr int SCALE_BYTES = (EB == 1) ? 2 * P * 4 : 0;
  static constexpr int STAGE_BYTES = BLOCK_BYTES + SCALE_BYTES;
  // token held in column c of S n-tile t (see the fragment notes in the file header of the C ABI docs)
  static __device__ __forceinline__ int token_of(int t, int c) {
    if constexpr (EB == 1) return 16 * (c >> 1) + 4 * (t >> 1) + 2 * (t & 1) + (c & 1);
    else return 8 * t + c;
  }
};

// Loads the A fragments of one m-tile of Q. Row R of the tile is (token R / G, head R % G).
template <int EB, int D, typename TQ>
__device__ __forceinline__ void load_q_frags(uint32_t (&qa)[D / 16][4], const TQ* __restrict__ q_base, int row_lo,
                                             int row_hi, int n_rows, int G, int n_q_heads, int head0, int lane) {
  constexpr bool F16 = EB == 1;
  const int j = lane & 3;
  const int rows[2] = {row_lo, row_hi};
#pragma unroll
  for (int s = 0; s < D / 16; ++s) {
#pragma unroll
    for (int half = 0; half < 2; ++half) {
      const int R = rows[half];
      float v[4] = {0.f, 0.f, 0.f, 0.f};
      if (R < n_rows) {
        const TQ* src = q_base + (static_cast<int64_t>(R / G) * n_q_heads + head0 + (R % G)) * D;
        // bf16 path: k = 16s + 2j + {0,1} and + 8; e4m3 path: dims 16j + 4s + {0,1} and {2,3}
        const int d0 = F16 ? 16 * j + 4 * s : 16 * s + 2 * j;
        const int d1 = F16 ? d0 + 2 : d0 + 8;
        v[0] = Elem<TQ>::load(src + d0); v[1] = Elem<TQ>::load(src + d0 + 1);
        v[2] = Elem<TQ>::load(src + d1); v[3] = Elem<TQ>::load(src + d1 + 1);
      }
      qa[s][half] = att_pack<F16>(v[0], v[1]);      // a0a1 (row_lo) / a2a3 (row_hi)
      qa[s][2 + half] = att_pack<F16>(v[2], v[3]);  // a4a5 / a6a7
    }
  }
}

// One page for one m-tile: S = Q K^T (scaled, masked), online softmax update, O += P V.
// limit_lo / limit_hi: number of cache positions rows row_lo / row_hi may see (0 masks the row).
// HI = false: rows 8..15 of the m-tile are padding (a decode row with at most 8 query heads per KV
// head), so their softmax arithmetic is skipped and their P fragments are zero.
//
// e4m3 pages: a lane reads one whole 16-byte chunk of a K row (or V^T row) per n-tile (or output
// tile) and feeds the four K steps from its four words; the contraction index of an MMA is only a
// label, so Q is loaded with dims 16 j + 4 s + {0..3} in K step s to match, and the token a score
// column stands for (BlockGeom::token_of) is chosen such that the P fragments line up with 16
// consecutive tokens of a V^T row. The per-token scales of a lane's columns are then four
// consecutive floats: one 16-byte load per pair of n-tiles.
template <int EB, int D, int P, bool HI, bool LDM = !HI>
__device__ __forceinline__ void attend_page(const uint32_t (&qa)[D / 16][4], float (&o)[D / 8][4], float (&m)[2],
                                            float (&l)[2], uint32_t stage, int page_token0, int limit_lo,
                                            int limit_hi, float scale_log2, int lane) {
  using Geo = BlockGeom<EB, D, P>;
  constexpr bool F16 = EB == 1;
  constexpr int NT = P / 8, KS = D / 16, OT = D / 8, PS = P / 16;
  static_assert(!F16 || (D == 64 && P == 64), "the e4m3 fragment layout is built for 64 x 64 blocks");
  const int c8 = lane >> 2, j = lane & 3;
  float s[NT][4];
#pragma unroll
  for (int t = 0; t < NT; ++t) s[t][0] = s[t][1] = s[t][2] = s[t][3] = 0.f;
  if constexpr (F16) {
#pragma unroll
    for (int t0 = 0; t0 < NT; t0 += 4) {  // four n-tiles at a time: independent accumulators between dependent MMAs
      uint32_t kw[4][4];
#pragma unroll
      for (int tt = 0; tt < 4; ++tt) {
        const int tok = Geo::token_of(t0 + tt, c8);  // K row this thread feeds for column c8
        att_lds128(stage + tok * Geo::K_ROW + kv_swizzle(tok, j, Geo::K_CPR) * 16, kw[tt]);
      }
#pragma unroll
      for (int k = 0; k < KS; ++k) {
#pragma unroll
        for (int tt = 0; tt < 4; ++tt) {
          uint32_t b0, b1;
          att_e4m3x4_to_f16x4(kw[tt][k], b0, b1);
          att_mma<F16>(s[t0 + tt], qa[k], b0, b1);
        }
      }
    }
  } else if constexpr (!LDM) {
    // bf16 pages, plain 32-bit fragment loads (kept for callers whose register budget the ldmatrix form
    // below would overflow: two m-tiles per warp)
#pragma unroll
    for (int t = 0; t < NT; ++t) {
      const int tok = Geo::token_of(t, c8);
      const uint32_t row_addr = stage + tok * Geo::K_ROW;
#pragma unroll
      for (int k = 0; k < KS; ++k) {
        const uint32_t b0 = att_lds32(row_addr + kv_swizzle(tok, 2 * k, Geo::K_CPR) * 16 + 4 * j);
        const uint32_t b1 = att_lds32(row_addr + kv_swizzle(tok, 2 * k + 1, Geo::K_CPR) * 16 + 4 * j);
        att_mma<F16>(s[t], qa[k], b0, b1);
      }
    }
  } else {
    // bf16 pages: ldmatrix.x4 fetches the B fragments of two K steps of one n-tile at once (matrix m of
    // the four = 16-byte chunk 4 h + m of the K rows 8 t .. 8 t + 7, one row address per lane)
    static_assert(KS % 2 == 0 && NT % 2 == 0, "fragment loads pair K steps and n-tiles");
    const int lrow = lane & 7, lmat = lane >> 3;
    constexpr int TG = HI ? 1 : 2;  // n-tiles in flight: independent accumulators between dependent MMAs
#pragma unroll
    for (int t0 = 0; t0 < NT; t0 += TG) {
      uint32_t kb[TG][KS / 2][4];
#pragma unroll
      for (int tt = 0; tt < TG; ++tt) {
        const int tok = 8 * (t0 + tt) + lrow;
#pragma unroll
        for (int h = 0; h < KS / 2; ++h)
          att_ldmatrix_x4(stage + tok * Geo::K_ROW + kv_swizzle(tok, 4 * h + lmat, Geo::K_CPR) * 16, kb[tt][h]);
      }
#pragma unroll
      for (int k = 0; k < KS; ++k) {
#pragma unroll
        for (int tt = 0; tt < TG; ++tt)
          att_mma<F16>(s[t0 + tt], qa[k], kb[tt][k >> 1][2 * (k & 1)], kb[tt][k >> 1][2 * (k & 1) + 1]);
      }
    }
  }
  // scale (x per-token K scale for e4m3), causal / length mask, page maximum per row
  const bool masked = page_token0 + P > (HI ? min(limit_lo, limit_hi) : limit_lo);  // warp-uniform per m-tile row pair
  float mx[2] = {-INFINITY, -INFINITY};
#pragma unroll
  for (int a = 0; a < NT / 2; ++a) {
    float ks4[4] = {scale_log2, scale_log2, scale_log2, scale_log2};
    if constexpr (F16) {
      att_lds128f(stage + Geo::BLOCK_BYTES + 4 * (16 * j + 4 * a), ks4);  // tokens 16 j + 4 a + {0..3}
#pragma unroll
      for (int q = 0; q < 4; ++q) ks4[q] *= scale_log2;
    }
#pragma unroll
    for (int e = 0; e < 2; ++e) {
      const int t = 2 * a + e;
#pragma unroll
      for (int i = 0; i < 2; ++i) {
        const float ks = ks4[2 * e + i];
        s[t][i] *= ks;
        if constexpr (HI) s[t][2 + i] *= ks;
        if (masked) {
          const int pos = page_token0 + Geo::token_of(t, 2 * j + i);
          if (pos >= limit_lo) s[t][i] = -INFINITY;
          if constexpr (HI) { if (pos >= limit_hi) s[t][2 + i] = -INFINITY; }
        }
        mx[0] = fmaxf(mx[0], s[t][i]);
        if constexpr (HI) mx[1] = fmaxf(mx[1], s[t][2 + i]);
      }
    }
  }
  float alpha[2] = {1.f, 1.f};
#pragma unroll
  for (int h = 0; h < (HI ? 2 : 1); ++h) {
    mx[h] = fmaxf(mx[h], __shfl_xor_sync(0xffffffffu, mx[h], 1));
    mx[h] = fmaxf(mx[h], __shfl_xor_sync(0xffffffffu, mx[h], 2));
    const float m_new = fmaxf(m[h], mx[h]);
    alpha[h] = (m[h] == -INFINITY) ? 0.f : exp2f(m[h] - m_new);
    m[h] = m_new;
    l[h] *= alpha[h];
  }
#pragma unroll
  for (int u = 0; u < OT; ++u) {
    o[u][0] *= alpha[0]; o[u][1] *= alpha[0];
    if constexpr (HI) { o[u][2] *= alpha[1]; o[u][3] *= alpha[1]; }
  }
  // P = exp2(S - m); fp32 row sums; P (x V scale) rounded to the MMA input type
  const float m0 = (m[0] == -INFINITY) ? 0.f : m[0], m1 = (m[1] == -INFINITY) ? 0.f : m[1];
  uint32_t pa[PS][4];
#pragma unroll
  for (int a = 0; a < NT / 2; ++a) {
    float vs4[4] = {1.f, 1.f, 1.f, 1.f};
    if constexpr (F16) att_lds128f(stage + Geo::BLOCK_BYTES + 4 * P + 4 * (16 * j + 4 * a), vs4);
    float p_lo[4], p_hi[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int q = 0; q < 4; ++q) {  // q = 2 e + i: n-tile 2 a + e, column 2 j + i
      const int t = 2 * a + (q >> 1), i = q & 1;
      const float p0 = exp2f(s[t][i] - m0);  // exp2(-inf) = 0 for masked entries
      l[0] += p0;
      p_lo[q] = F16 ? p0 * vs4[q] : p0;
      if constexpr (HI) {
        const float p1 = exp2f(s[t][2 + i] - m1);
        l[1] += p1;
        p_hi[q] = F16 ? p1 * vs4[q] : p1;
      }
    }
    pa[a][0] = att_pack<F16>(p_lo[0], p_lo[1]);
    pa[a][2] = att_pack<F16>(p_lo[2], p_lo[3]);
    pa[a][1] = HI ? att_pack<F16>(p_hi[0], p_hi[1]) : 0u;
    pa[a][3] = HI ? att_pack<F16>(p_hi[2], p_hi[3]) : 0u;
  }
  const uint32_t vt = stage + Geo::K_BYTES;
  if constexpr (F16) {
#pragma unroll
    for (int u0 = 0; u0 < OT; u0 += 4) {
      uint32_t vw[4][4];
#pragma unroll
      for (int uu = 0; uu < 4; ++uu) {
        const int dim = 8 * (u0 + uu) + c8;  // V^T row this thread feeds for output column c8
        att_lds128(vt + dim * Geo::V_ROW + kv_swizzle(dim, j, Geo::V_CPR) * 16, vw[uu]);
      }
#pragma unroll
      for (int k = 0; k < PS; ++k) {
#pragma unroll
        for (int uu = 0; uu < 4; ++uu) {
          uint32_t b0, b1;
          att_e4m3x4_to_f16x4(vw[uu][k], b0, b1);
          att_mma<F16>(o[u0 + uu], pa[k], b0, b1);
        }
      }
    }
  } else if constexpr (!LDM) {
#pragma unroll
    for (int k = 0; k < PS; ++k) {
#pragma unroll
      for (int u = 0; u < OT; ++u) {
        const int dim = 8 * u + c8;  // V^T row this thread feeds for output column c8
        const uint32_t row_addr = vt + dim * Geo::V_ROW;
        const uint32_t b0 = att_lds32(row_addr + kv_swizzle(dim, 2 * k, Geo::V_CPR) * 16 + 4 * j);
        const uint32_t b1 = att_lds32(row_addr + kv_swizzle(dim, 2 * k + 1, Geo::V_CPR) * 16 + 4 * j);
        att_mma<F16>(o[u], pa[k], b0, b1);
      }
    }
  } else {
    static_assert(PS % 2 == 0 && OT % 2 == 0, "fragment loads pair K steps and output tiles");
    const int lrow = lane & 7, lmat = lane >> 3;
    constexpr int UG = HI ? 1 : 2;
#pragma unroll
    for (int u0 = 0; u0 < OT; u0 += UG) {
      uint32_t vb[UG][PS / 2][4];
#pragma unroll
      for (int uu = 0; uu < UG; ++uu) {
        const int dim = 8 * (u0 + uu) + lrow;  // V^T row (one head dim), 16-byte chunks of 8 tokens
#pragma unroll
        for (int h = 0; h < PS / 2; ++h)
          att_ldmatrix_x4(vt + dim * Geo::V_ROW + kv_swizzle(dim, 4 * h + lmat, Geo::V_CPR) * 16, vb[uu][h]);
      }
#pragma unroll
      for (int k = 0; k < PS; ++k) {
#pragma unroll
        for (int uu = 0; uu < UG; ++uu)
          att_mma<F16>(o[u0 + uu], pa[k], vb[uu][k >> 1][2 * (k & 1)], vb[uu][k >> 1][2 * (k & 1) + 1]);
      }
    }
  }
}

__device__ __forceinline__ void stage_block(uint32_t dst, uint32_t bar, const uint8_t* pool, const float* scales,
                                            int64_t block_byte_offset, int64_t scale_offset, int block_bytes,
                                            int scale_bytes) {
  att_bar_expect(bar, block_bytes + scale_bytes);
  att_bulk_copy(dst, pool + block_byte_offset, block_bytes, bar);
  if (scale_bytes) att_bulk_copy(dst + block_bytes, scales + scale_offset, scale_bytes, bar);
}

// ------------------------------------------------------------------------------------------ decode
// NST = pages in flight per warp. A CTA spends about 3 us outside its page loop (q and block-table
// fetch, first page latency, merge, store), so the SM is better used by several short-ring CTAs whose
// fixed phases overlap than by one CTA with a deep ring: NST = 1 -> 64 KB (bf16) and 3 CTAs per SM.
// e4m3 pages are half the size, so two of them per warp still leave room for 3 CTAs per SM (NST = 2).
template <int EB, int NST>
constexpr int decode_ctas_per_sm() { return (NST == 1 || (EB == 1 && NST == 2)) ? 3 : 1; }

template <typename TQ, int EB, int D, int P, int NST, bool HI>
__global__ void __launch_bounds__(128, decode_ctas_per_sm<EB, NST>())
decode_attention_mma_kernel(TQ* __restrict__ out, const TQ* __restrict__ q, const int32_t* __restrict__ kv_lens,
                            const int32_t* __restrict__ slots, const uint8_t* __restrict__ active,
                            cgym_kv_layout kv, int layer, int n_q_heads, float scale, int n_splits,
                            float* __restrict__ workspace, int32_t* __restrict__ status) {
  using Geo = BlockGeom<EB, D, P>;
  constexpr int OT = D / 8;
  extern __shared__ __align__(128) uint8_t att_smem[];
  __shared__ __align__(8) uint64_t bars[4][NST];
  __shared__ int abort_flag;
  pdl_trigger();
  // Under programmatic dependent launch this CTA may run before the kernel just ahead of it (the
  // QK-norm / RoPE / append) has finished. That kernel writes q and ONE cache position per row, in
  // the row's last page; kv_lens, slots, active and the block table are fixed since the start of the
  // step. So the pages before the last one are fetched right away and only q and the last page wait.
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int row = blockIdx.x, kh = blockIdx.y, split = blockIdx.z;
  const int G = n_q_heads / kv.n_kv_heads;
  const int slot = slots != nullptr ? slots[row] : row;
  int len = kv_lens[row];
  if ((active != nullptr && !active[row]) || slot < 0 || len < 0) len = 0;
  if (threadIdx.x == 0) {
    abort_flag = 0;
    for (int w = 0; w < 4; ++w)
      for (int st = 0; st < NST; ++st) att_bar_init(att_smem_u32(&bars[w][st]), 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncthreads();

  const int total_pages = (len + P - 1) / P;
  const int per_split = (total_pages + n_splits - 1) / n_splits;
  const int page_begin = min(total_pages, split * per_split), page_end = min(total_pages, page_begin + per_split);
  const int n_mine = (page_end - page_begin - warp + 3) / 4;  // pages page_begin + warp + 4 i
  const int32_t* table = kv.block_table + static_cast<int64_t>(slot < 0 ? 0 : slot) * kv.max_blocks;
  const uint8_t* pool = static_cast<const uint8_t*>(kv.kv_pool);
  const uint32_t ring = att_smem_u32(att_smem) + warp * NST * Geo::STAGE_BYTES;

  auto issue = [&](int i) {
    if (lane == 0) {
      int page = table[page_begin + warp + 4 * i];
      if (page < 0 || page >= kv.n_pages) { atomicOr(status, CGYM_STATUS_BAD_PAGE); page = 0; }
      stage_block(ring + (i % NST) * Geo::STAGE_BYTES, att_smem_u32(&bars[warp][i % NST]), pool, kv.kv_scales,
                  kv_block_offset(kv, layer, page, kh) * EB, kv_scale_offset(kv, layer, page, 0, kh, 0),
                  Geo::BLOCK_BYTES, Geo::SCALE_BYTES);
    }
  };
  int issued = 0;
  const int last_page = total_pages - 1;  // holds the position the append kernel writes this step
  while (issued < n_mine && issued < NST && page_begin + warp + 4 * issued != last_page) issue(issued++);
  pdl_wait();
  q = pdl_fresh(q);
  uint32_t qa[D / 16][4];
  load_q_frags<EB, D, TQ>(qa, q + static_cast<int64_t>(row) * n_q_heads * D, lane >> 2, (lane >> 2) + 8, G, G,
                          n_q_heads, kh * G, lane);
  float o[OT][4], m[2] = {-INFINITY, -INFINITY}, l[2] = {0.f, 0.f};
#pragma unroll
  for (int u = 0; u < OT; ++u) o[u][0] = o[u][1] = o[u][2] = o[u][3] = 0.f;
  const float scale_log2 = scale * 1.4426950408889634f;
  for (; issued < n_mine && issued < NST; ++issued) issue(issued);  // fill the rest of the warp's ring
  for (int i = 0; i < n_mine; ++i) {
    if (!att_bar_wait(att_smem_u32(&bars[warp][i % NST]), (i / NST) & 1, &abort_flag)) break;
    const int token0 = (page_begin + warp + 4 * i) * P;
    attend_page<EB, D, P, HI>(qa, o, m, l, ring + (i % NST) * Geo::STAGE_BYTES, token0, len, len, scale_log2, lane);
    __syncwarp();  // every lane is done reading this stage before lane 0 refills it
    if (issued < n_mine) { issue(issued); ++issued; }
  }
  if (abort_flag && lane == 0) {  // let copies in flight land before shared memory is reused / released
    for (int i = max(0, issued - NST); i < issued; ++i)
      att_bar_wait(att_smem_u32(&bars[warp][i % NST]), (i / NST) & 1, &abort_flag);
  }
  __syncthreads();
  if (threadIdx.x == 0 && abort_flag) atomicOr(status, CGYM_STATUS_WAIT_TIMEOUT);

  // merge the four warps through shared memory (the rings are free now)
  float* w_o = reinterpret_cast<float*>(att_smem);          // [4][16][D]
  float* w_m = w_o + 4 * 16 * D;                            // [4][16]
  float* w_l = w_m + 4 * 16;                                // [4][16]
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    l[h] += __shfl_xor_sync(0xffffffffu, l[h], 1);
    l[h] += __shfl_xor_sync(0xffffffffu, l[h], 2);
  }
  {
    const int r0 = lane >> 2, j = lane & 3;
    if (j == 0) {
      w_m[warp * 16 + r0] = m[0]; w_m[warp * 16 + r0 + 8] = m[1];
      w_l[warp * 16 + r0] = l[0]; w_l[warp * 16 + r0 + 8] = l[1];
    }
#pragma unroll
    for (int u = 0; u < OT; ++u) {
      float* dst = w_o + (warp * 16 + r0) * D + 8 * u + 2 * j;
      dst[0] = o[u][0]; dst[1] = o[u][1];
      dst[8 * D] = o[u][2]; dst[8 * D + 1] = o[u][3];
    }
  }
  __syncthreads();
  for (int i = threadIdx.x; i < G * D; i += blockDim.x) {
    const int g = i / D, d = i % D;
    float mm = -INFINITY;
    for (int w = 0; w < 4; ++w) mm = fmaxf(mm, w_m[w * 16 + g]);
    float total = 0.f, value = 0.f;
    for (int w = 0; w < 4; ++w) {
      const float mw = w_m[w * 16 + g];
      const float f = (mw == -INFINITY) ? 0.f : exp2f(mw - mm);
      total += f * w_l[w * 16 + g];
      value += f * w_o[(w * 16 + g) * D + d];
    }
    const int head = kh * G + g;
    if (n_splits == 1) {
      Elem<TQ>::store(out + (static_cast<int64_t>(row) * n_q_heads + head) * D + d, value / fmaxf(total, 1.0e-20f));
    } else {
      const int64_t part = (static_cast<int64_t>(row) * n_q_heads + head) * n_splits + split;
      const int64_t n_parts = static_cast<int64_t>(gridDim.x) * n_q_heads * n_splits;
      workspace[part * D + d] = value;
      if (d == 0) {
        workspace[n_parts * D + part] = mm * 0.6931471805599453f;  // the combine kernel works in the natural-log domain
        workspace[n_parts * (D + 1) + part] = total;
      }
    }
  }
}

// ------------------------------------------------------------------------------------------ prefill
struct PrefillTiles {
  const int32_t* row0;   // packed row of the tile's first query token
  const int32_t* ntok;   // query tokens in the tile (<= 128 / G)
  const int32_t* slot;   // cache slot of the sequence
  const int32_t* pos0;   // cache position of the tile's first query token
};

// MT = m-tiles (16 rows) per consumer warp; the 128 rows of a CTA take 8 / MT consumer warps plus the producer.
template <typename TQ, int EB, int D, int P, int MT>
__global__ void __launch_bounds__(32 * (8 / MT + 1), 1)
prefill_attention_mma_kernel(TQ* __restrict__ out, const TQ* __restrict__ q, PrefillTiles tiles, cgym_kv_layout kv,
                             int layer, int n_q_heads, float scale, int32_t* __restrict__ status) {
  using Geo = BlockGeom<EB, D, P>;
  constexpr int OT = D / 8, STAGES = 4, CW = 8 / MT;  // CW consumer warps
  extern __shared__ __align__(128) uint8_t att_smem[];
  __shared__ __align__(8) uint64_t bar_full[STAGES];
  __shared__ __align__(8) uint64_t bar_empty[STAGES];
  __shared__ int abort_flag;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int tile = blockIdx.x, kh = blockIdx.y;
  const int G = n_q_heads / kv.n_kv_heads;
  const int row0 = tiles.row0[tile], ntok = tiles.ntok[tile], slot = tiles.slot[tile], pos0 = tiles.pos0[tile];
  const int n_rows = ntok * G;                 // (token, head) rows of this tile, <= 128
  const int n_pages = (pos0 + ntok + P - 1) / P;  // causal range of the tile's last token
  if (threadIdx.x == 0) {
    abort_flag = 0;
    for (int s = 0; s < STAGES; ++s) { att_bar_init(att_smem_u32(&bar_full[s]), 1); att_bar_init(att_smem_u32(&bar_empty[s]), CW); }
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncthreads();
  const uint32_t ring = att_smem_u32(att_smem);
  const int32_t* table = kv.block_table + static_cast<int64_t>(slot) * kv.max_blocks;

  if (warp == CW) {
    // ---- producer ----
    if (lane == 0) {
      const uint8_t* pool = static_cast<const uint8_t*>(kv.kv_pool);
      int issued = 0;
      for (int i = 0; i < n_pages; ++i) {
        const int s = i % STAGES;
        if (!att_bar_wait(att_smem_u32(&bar_empty[s]), ((i / STAGES) & 1) ^ 1, &abort_flag)) break;
        int page = table[i];
        if (page < 0 || page >= kv.n_pages) { atomicOr(status, CGYM_STATUS_BAD_PAGE); page = 0; }
        stage_block(ring + s * Geo::STAGE_BYTES, att_smem_u32(&bar_full[s]), pool, kv.kv_scales,
                    kv_block_offset(kv, layer, page, kh) * EB, kv_scale_offset(kv, layer, page, 0, kh, 0),
                    Geo::BLOCK_BYTES, Geo::SCALE_BYTES);
        issued = i + 1;
      }
      if (abort_flag)
        for (int i = max(0, issued - STAGES); i < issued; ++i)
          att_bar_wait(att_smem_u32(&bar_full[i % STAGES]), (i / STAGES) & 1, &abort_flag);
    }
  } else {
    // ---- consumers: warp w owns rows [16 MT w, 16 MT (w + 1)) as MT m-tiles ----
    uint32_t qa[MT][D / 16][4];
    float o[MT][OT][4], m[MT][2], l[MT][2];
    int limit[MT][2];
    const TQ* q_base = q + static_cast<int64_t>(row0) * n_q_heads * D;
    int warp_limit = 0;
#pragma unroll
    for (int t = 0; t < MT; ++t) {
      const int r_lo = warp * (16 * MT) + t * 16 + (lane >> 2), r_hi = r_lo + 8;
      load_q_frags<EB, D, TQ>(qa[t], q_base, r_lo, r_hi, n_rows, G, n_q_heads, kh * G, lane);
      limit[t][0] = r_lo < n_rows ? pos0 + r_lo / G + 1 : 0;
      limit[t][1] = r_hi < n_rows ? pos0 + r_hi / G + 1 : 0;
      warp_limit = max(warp_limit, max(limit[t][0], limit[t][1]));
      m[t][0] = m[t][1] = -INFINITY;
      l[t][0] = l[t][1] = 0.f;
#pragma unroll
      for (int u = 0; u < OT; ++u) o[t][u][0] = o[t][u][1] = o[t][u][2] = o[t][u][3] = 0.f;
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) warp_limit = max(warp_limit, __shfl_xor_sync(0xffffffffu, warp_limit, off));
    const float scale_log2 = scale * 1.4426950408889634f;
    for (int i = 0; i < n_pages; ++i) {
      const int s = i % STAGES;
      if (!att_bar_wait(att_smem_u32(&bar_full[s]), (i / STAGES) & 1, &abort_flag)) break;
      if (i * P < warp_limit) {
#pragma unroll
        for (int t = 0; t < MT; ++t)
          attend_page<EB, D, P, true, MT == 1>(qa[t], o[t], m[t], l[t], ring + s * Geo::STAGE_BYTES, i * P, limit[t][0], limit[t][1],
                                scale_log2, lane);
      }
      __syncwarp();
      if (lane == 0) att_bar_arrive(att_smem_u32(&bar_empty[s]));
    }
    // normalise and store: fragment (row, dims 8u + 2j + {0,1})
    const int j = lane & 3;
#pragma unroll
    for (int t = 0; t < MT; ++t) {
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        float sum = l[t][h];
        sum += __shfl_xor_sync(0xffffffffu, sum, 1);
        sum += __shfl_xor_sync(0xffffffffu, sum, 2);
        const int R = warp * (16 * MT) + t * 16 + (lane >> 2) + 8 * h;
        if (R < n_rows) {
          const float inv = 1.0f / fmaxf(sum, 1.0e-20f);
          TQ* dst = out + (static_cast<int64_t>(row0 + R / G) * n_q_heads + kh * G + (R % G)) * D;
#pragma unroll
          for (int u = 0; u < OT; ++u) {
            Elem<TQ>::store(dst + 8 * u + 2 * j, o[t][u][2 * h] * inv);
            Elem<TQ>::store(dst + 8 * u + 2 * j + 1, o[t][u][2 * h + 1] * inv);
          }
        }
      }
    }
  }
  __syncthreads();
  if (threadIdx.x == 0 && abort_flag) atomicOr(status, CGYM_STATUS_WAIT_TIMEOUT);
}

// ------------------------------------------------------------------------------------------ launchers
bool attention_mma_supported(const cgym_kv_layout* kv, int n_q_heads, int dtype) {
  if (dtype != CGYM_BF16) return false;
  if (kv->kv_dtype != CGYM_BF16 && kv->kv_dtype != CGYM_E4M3) return false;
  if (kv->page_size != 64 || kv->head_dim != 64) return false;
  const int G = n_q_heads / kv->n_kv_heads;
  return G >= 1 && G <= 16 && n_q_heads % kv->n_kv_heads == 0;
}

template <int EB, int D, int NST, bool HI>
static int launch_decode(void* out, const void* q, const int32_t* kv_lens, const int32_t* slots, const uint8_t* active,
                         const cgym_kv_layout* kv, int layer, int rows, int n_q_heads, float scale, int n_splits,
                         float* workspace, int32_t* status, cudaStream_t stream) {
  using T = __nv_bfloat16;
  using Geo = BlockGeom<EB, D, 64>;
  constexpr int ring = 4 * NST * Geo::STAGE_BYTES, merge = (4 * 16 * D + 2 * 4 * 16) * 4;
  constexpr int smem = ring > merge ? ring : merge;
  auto kernel = decode_attention_mma_kernel<T, EB, D, 64, NST, HI>;
  static SmemReservation reservation;
  if (int rc = reserve_dynamic_smem(kernel, smem, reservation, "paged_attention")) return rc;
  const cudaError_t rc = launch_dependent(kernel, dim3(rows, kv->n_kv_heads, n_splits), dim3(128), smem, stream,
                                          static_cast<T*>(out), static_cast<const T*>(q), kv_lens, slots, active, *kv,
                                          layer, n_q_heads, scale, n_splits, workspace, status);
  CGYM_REQUIRE(rc == cudaSuccess, "paged_attention: launch failed: %s", cudaGetErrorString(rc));
  return 0;
}

int launch_decode_attention_mma(void* out, const void* q, const int32_t* kv_lens, const int32_t* slots,
                                const uint8_t* active, const cgym_kv_layout* kv, int layer, int rows, int n_q_heads,
                                float scale, int n_splits, float* workspace, int32_t* status, cudaStream_t stream) {
  const bool fp8 = kv->kv_dtype == CGYM_E4M3;
  // More CTAs than one per SM: short rings, several CTAs per SM. Fewer: one deep ring per SM.
  const bool shallow = static_cast<int64_t>(rows) * kv->n_kv_heads * n_splits > 148;
  // rows 8..15 of the 16-row MMA tile carry query heads only when more than 8 heads share a KV head
  const bool hi = n_q_heads / kv->n_kv_heads > 8;
#define CGYM_DECODE(EB, NST)                                                                                          \
  (hi ? launch_decode<EB, 64, NST, true>(out, q, kv_lens, slots, active, kv, layer, rows, n_q_heads, scale, n_splits, \
                                         workspace, status, stream)                                                   \
      : launch_decode<EB, 64, NST, false>(out, q, kv_lens, slots, active, kv, layer, rows, n_q_heads, scale, n_splits, \
                                          workspace, status, stream))
  if (fp8) return shallow ? CGYM_DECODE(1, 2) : CGYM_DECODE(1, 3);
  return shallow ? CGYM_DECODE(2, 1) : CGYM_DECODE(2, 3);
#undef CGYM_DECODE
}

template <int EB, int D>
static int launch_prefill(void* out, const void* q, const PrefillTiles& tiles, const cgym_kv_layout* kv, int layer,
                          int n_tiles, int n_q_heads, float scale, int32_t* status, cudaStream_t stream) {
  using T = __nv_bfloat16;
  using Geo = BlockGeom<EB, D, 64>;
  constexpr int smem = 4 * Geo::STAGE_BYTES;
  // eight consumer warps of one 16-row m-tile each (four warps of two m-tiles measured slower on long prompts)
  auto kernel = prefill_attention_mma_kernel<T, EB, D, 64, 1>;
  static SmemReservation reservation;
  if (int rc = reserve_dynamic_smem(kernel, smem, reservation, "prefill_attention")) return rc;
  kernel<<<dim3(n_tiles, kv->n_kv_heads), 288, smem, stream>>>(static_cast<T*>(out), static_cast<const T*>(q), tiles, *kv,
                                                               layer, n_q_heads, scale, status);
  return 0;
}

bool prefill_attention_tcgen05_supported(const cgym_kv_layout* kv, int n_q_heads);
int launch_prefill_attention_tcgen05(void* out, const void* q, const int32_t* tile_row0, const int32_t* tile_ntok,
                                     const int32_t* tile_slot, const int32_t* tile_pos0, const cgym_kv_layout* kv,
                                     int layer, int n_tiles, int n_q_heads, float scale, int32_t* status,
                                     cudaStream_t stream);

// bf16 caches take the tcgen05 / TMEM kernel (attention_tcgen05.cu); e4m3 caches, whose operands are widened to
// fp16 in registers, stay on the mma.sync kernel above.
int launch_prefill_attention_mma(void* out, const void* q, const int32_t* tile_row0, const int32_t* tile_ntok,
                                 const int32_t* tile_slot, const int32_t* tile_pos0, const cgym_kv_layout* kv, int layer,
                                 int n_tiles, int n_q_heads, float scale, int32_t* status, cudaStream_t stream) {
  if (prefill_attention_tcgen05_supported(kv, n_q_heads))
    return launch_prefill_attention_tcgen05(out, q, tile_row0, tile_ntok, tile_slot, tile_pos0, kv, layer, n_tiles,
                                            n_q_heads, scale, status, stream);
  const PrefillTiles tiles{tile_row0, tile_ntok, tile_slot, tile_pos0};
  const bool fp8 = kv->kv_dtype == CGYM_E4M3;
  return fp8 ? launch_prefill<1, 64>(out, q, tiles, kv, layer, n_tiles, n_q_heads, scale, status, stream)
             : launch_prefill<2, 64>(out, q, tiles, kv, layer, n_tiles, n_q_heads, scale, status, stream);
}

}  // namespace cgym
