// Blackwell tensor-core GEMM for the projections and the LM head:
//   y[M, N] = x[M, K] . w[N, K]^T      (bf16 x bf16, or e4m3 x e4m3 with per-row / per-channel scales)
//
// The weight matrix is the streamed operand (decode reads every weight once per step and M is
// small), so the kernel is "swap-AB": a CTA owns 128 output features (the MMA M dimension, one TMEM
// lane each) and a tile of UN tokens (the MMA N dimension, one TMEM column each). Per 128-byte K
// slice, TMA brings a [128 x 128B] weight tile and a [UN x 128B] activation tile into shared memory
// with the 128-byte swizzle the UMMA descriptors expect; one elected thread issues tcgen05.mma
// (fp32 accumulate in TMEM), tcgen05.commit releases the stage, and four epilogue warps read the
// accumulator back with tcgen05.ld, turn it (lane = feature) into token rows through shared memory and
// write y in 16-byte row segments, applying scales / row mask / row map. While the MMAs run, the same
// warps resolve where each token row of the tile goes (row mask, row map, M edge) and its activation
// scale into shared memory and fetch the weight scales, so nothing between the accumulator and the
// store depends on global memory.
// Warp roles: 0 = TMA producer, 1 = MMA issuer + TMEM owner, 2..5 = epilogue.
//
// Split-K (grid.z <= 8) runs as a thread-block cluster: each CTA parks its fp32 partial tile - in the
// caller's workspace (L2) when one is given, else in its own shared memory - and after a cluster
// barrier every CTA sums its share of the tile's rows over all partials in split order, so results
// are deterministic and no second launch is needed. Every mbarrier wait is bounded (about two
// seconds of %globaltimer): on expiry the CTA raises CGYM_STATUS_WAIT_TIMEOUT, drains its own TMA
// copies with the same bound, frees its TMEM and returns.
#include <cuda.h>

#include <mutex>

#include "common.cuh"

namespace cgym {

constexpr int UM = 128;           // output features per CTA
constexpr int SLICE_BYTES = 128;  // K bytes per pipeline stage (one swizzle atom wide)
constexpr int GEMM_THREADS = 192;
constexpr unsigned long long WAIT_LIMIT_NS = 2000000000ull;

// TEST HOOK (cgym_test_gemm_wait): a shorter limit for the waits that decide to give up, and a switch that
// makes the producer arm its barriers without issuing the copies, so that a wait nothing satisfies runs out
// and the give-up path (status word, TMEM freed, kernel returns) can be exercised without a fault or a hang.
// Both keep their defaults in production; waits that drain copies already in flight always use the full limit.
__device__ unsigned long long g_wait_limit_ns = WAIT_LIMIT_NS;
__device__ int g_drop_loads = 0;

__device__ __forceinline__ uint32_t smem_u32(const void* p) { return static_cast<uint32_t>(__cvta_generic_to_shared(p)); }

__device__ __forceinline__ unsigned long long global_timer() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
}
__device__ __forceinline__ bool mbar_try(uint32_t bar, uint32_t parity) {
  uint32_t done;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(done)
      : "r"(bar), "r"(parity)
      : "memory");
  return done != 0;
}
// bounded wait: false when the limit expired or another role already gave up
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity, volatile int* abort_flag,
                                          bool draining = false) {
  if (mbar_try(bar, parity)) return true;
  const unsigned long long start = global_timer();
  unsigned long long limit = 2000000000ull;  // WAIT_LIMIT_NS
  if (!draining) limit = *const_cast<volatile unsigned long long*>(&g_wait_limit_ns);
  for (uint32_t spin = 1;; ++spin) {
    if (mbar_try(bar, parity)) return true;
    if ((spin & 63u) == 0u) {
      if (*abort_flag && !draining) return false;
      if (global_timer() - start > limit) {
        *abort_flag = 1;
        return false;
      }
    }
  }
}

__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap* map, uint32_t bar, int x, int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];"
      ::"r"(dst), "l"(reinterpret_cast<uint64_t>(map)), "r"(bar), "r"(x), "r"(y)
      : "memory");
}

// K-major, 128-byte-swizzled operand tile: rows are 128 B apart, 8-row groups 1024 B apart
__device__ __forceinline__ uint64_t umma_smem_desc(uint32_t addr) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((addr >> 4) & 0x3FFF);   // start address
  d |= static_cast<uint64_t>(1) << 16;                // leading byte offset (unused with swizzle)
  d |= static_cast<uint64_t>(1024 >> 4) << 32;        // stride byte offset between 8-row groups
  d |= static_cast<uint64_t>(1) << 46;                // descriptor version (Blackwell)
  d |= static_cast<uint64_t>(2) << 61;                // SWIZZLE_128B
  return d;
}

__device__ __forceinline__ void umma_bf16(uint32_t tmem_d, uint64_t da, uint64_t db, uint32_t idesc, uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}"
      ::"r"(tmem_d), "l"(da), "l"(db), "r"(idesc), "r"(acc)
      : "memory");
}
__device__ __forceinline__ void umma_fp8(uint32_t tmem_d, uint64_t da, uint64_t db, uint32_t idesc, uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f8f6f4 [%0], %1, %2, %3, p;\n\t}"
      ::"r"(tmem_d), "l"(da), "l"(db), "r"(idesc), "r"(acc)
      : "memory");
}
__device__ __forceinline__ void umma_commit(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar) : "memory");
}
__device__ __forceinline__ void tmem_issue32(uint32_t taddr, uint32_t (&v)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
      "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
      : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]),
        "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15]),
        "=r"(v[16]), "=r"(v[17]), "=r"(v[18]), "=r"(v[19]), "=r"(v[20]), "=r"(v[21]), "=r"(v[22]), "=r"(v[23]),
        "=r"(v[24]), "=r"(v[25]), "=r"(v[26]), "=r"(v[27]), "=r"(v[28]), "=r"(v[29]), "=r"(v[30]), "=r"(v[31])
      : "r"(taddr));
}
// Completes every TMEM load of this thread. The registers of the load being waited for pass through the
// statement, so no use of them can be scheduled ahead of the wait.
__device__ __forceinline__ void tmem_wait32(uint32_t (&v)[32]) {
  asm volatile("tcgen05.wait::ld.sync.aligned;"
               : "+r"(v[0]), "+r"(v[1]), "+r"(v[2]), "+r"(v[3]), "+r"(v[4]), "+r"(v[5]), "+r"(v[6]), "+r"(v[7]),
                 "+r"(v[8]), "+r"(v[9]), "+r"(v[10]), "+r"(v[11]), "+r"(v[12]), "+r"(v[13]), "+r"(v[14]), "+r"(v[15]),
                 "+r"(v[16]), "+r"(v[17]), "+r"(v[18]), "+r"(v[19]), "+r"(v[20]), "+r"(v[21]), "+r"(v[22]), "+r"(v[23]),
                 "+r"(v[24]), "+r"(v[25]), "+r"(v[26]), "+r"(v[27]), "+r"(v[28]), "+r"(v[29]), "+r"(v[30]), "+r"(v[31])
               :
               : "memory");
}

struct GemmEpilogue {
  __nv_bfloat16* y;        // bf16 [M, N]
  const float* x_scales;   // per token, fp8 only
  const float* w_scales;   // per output feature, fp8 only
  const uint8_t* row_mask; // optional
  const int32_t* row_map;  // optional: token row m is written to output row row_map[m] (negative: not written)
  int32_t* status;
  int M, N, K;
  int partial;             // 1: split-K over a cluster of gridDim.z CTAs
  float* split_ws;         // split-K partial tiles [tile][split][UN][128] fp32; NULL = exchange through DSMEM
};


// Cluster split-K reduction of the parked [UN][128] fp32 tiles. CTA `rank` owns the token rows
// ml = rank, rank + SPLITS, ...; epilogue warp `quarter` takes every fourth of them, and one 16-byte
// load per lane fetches a whole 128-feature row of one peer's tile over distributed shared memory
// (lane l holds features 4l .. 4l+3). All loads of a thread are issued before the first add; the
// sum runs in split order, so the result does not depend on timing. Where a token row goes (row mask, row
// map, M edge) and its activation scale were staged in shared memory while the MMAs ran (row_out /
// row_scale), so no load from global memory sits between the partial sums and the store.
//
// GLOBAL = true is the same reduction with the partial tiles parked in a global fp32 workspace
// ([split][UN][128] per output tile, L2-resident) instead of shared memory: the SM-to-SM network
// moves about 15 GB/s per SM, an order of magnitude below what an SM draws from L2, so the exchange
// is faster through L2 and needs no barrier after it (nobody reads a peer's shared memory).
template <int SPLITS, int UN, bool GLOBAL>
__device__ __forceinline__ void cluster_reduce_rows(const GemmEpilogue& ep, uint32_t tile, const float* ws_tile,
                                                    uint32_t rank, int quarter, int lane, int n0,
                                                    const int32_t* row_out, const float* row_scale,
                                                    const float (&ws)[4]) {
  constexpr int ROWS = UN / SPLITS;  // rows this CTA reduces (a multiple of 4: UN >= 32, SPLITS <= 8)
  constexpr int MINE = ROWS / 4;     // rows per warp
  static_assert(ROWS % 4 == 0, "each epilogue warp reduces ROWS / 4 rows");
  const uint32_t column = tile + static_cast<uint32_t>(lane) * 16u;
  uint32_t peer[SPLITS];
  if (!GLOBAL) {
#pragma unroll
    for (int sp = 0; sp < SPLITS; ++sp)
      asm("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(peer[sp]) : "r"(column), "r"(sp));
  }
  const int n = n0 + 4 * lane;
  constexpr int BATCH = MINE * SPLITS <= 16 ? MINE : 16 / SPLITS;  // at most 16 loads of 16 bytes in flight
#pragma unroll 1
  for (int first = 0; first < MINE; first += BATCH) {
  float4 value[BATCH][SPLITS];
#pragma unroll
  for (int b = 0; b < BATCH; ++b) {
    const int i = first + b;
    const uint32_t ml = rank + static_cast<uint32_t>(quarter + 4 * i) * SPLITS;
#pragma unroll
    for (int sp = 0; sp < SPLITS; ++sp) {
      if (GLOBAL)
        value[b][sp] = __ldcg(reinterpret_cast<const float4*>(ws_tile + (static_cast<size_t>(sp) * UN + ml) * UM) + lane);
      else
        asm volatile("ld.shared::cluster.v4.f32 {%0, %1, %2, %3}, [%4];"
                     : "=f"(value[b][sp].x), "=f"(value[b][sp].y), "=f"(value[b][sp].z), "=f"(value[b][sp].w)
                     : "r"(peer[sp] + ml * (UM * 4u)));
    }
  }
#pragma unroll
  for (int b = 0; b < BATCH; ++b) {
    const int i = first + b;
    const int ml = static_cast<int>(rank) + (quarter + 4 * i) * SPLITS;
    const int out_row = row_out[ml];  // negative: beyond M, masked or unmapped
    if (out_row < 0) continue;
    float total[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll
    for (int sp = 0; sp < SPLITS; ++sp) {
      total[0] = __fadd_rn(total[0], value[b][sp].x);
      total[1] = __fadd_rn(total[1], value[b][sp].y);
      total[2] = __fadd_rn(total[2], value[b][sp].z);
      total[3] = __fadd_rn(total[3], value[b][sp].w);
    }
    if (ep.x_scales != nullptr) {
      const float xs = row_scale[ml];
#pragma unroll
      for (int j = 0; j < 4; ++j) total[j] = __fmul_rn(__fmul_rn(total[j], xs), ws[j]);
    }
    __nv_bfloat16* dst = ep.y + static_cast<int64_t>(out_row) * ep.N + n;
    if (n + 3 < ep.N && (ep.N & 3) == 0) {
      uint2 packed;
      *reinterpret_cast<__nv_bfloat162*>(&packed.x) = __floats2bfloat162_rn(total[0], total[1]);
      *reinterpret_cast<__nv_bfloat162*>(&packed.y) = __floats2bfloat162_rn(total[2], total[3]);
      *reinterpret_cast<uint2*>(dst) = packed;
    } else {
#pragma unroll
      for (int j = 0; j < 4; ++j)
        if (n + j < ep.N) dst[j] = __float2bfloat16_rn(total[j]);
    }
  }
  }
}

// RING_KB bounds the TMA ring: 192 fills the SM for one CTA (large token tiles); 96 lets two CTAs
// share an SM, so the CTAs of the NEXT kernel of a dependent-launch chain become resident - and
// stream their first weight tiles - while this kernel's CTAs are still computing.
// FM = feature sub-tiles of 128 per CTA. FM = 2 (unsplit GEMMs over more than 128 tokens) runs two MMAs
// per K step against the same token tile, into two TMEM accumulators: the activation tile is fetched
// once for 256 features, which halves its share of the L2 -> shared-memory traffic that bounds these
// shapes.
template <int UN, bool FP8, int RING_KB, int FM = 1>
__global__ void __launch_bounds__(GEMM_THREADS, RING_KB <= 96 ? 2 : 1)
gemm_tcgen05_kernel(const __grid_constant__ CUtensorMap tmap_w, const __grid_constant__ CUtensorMap tmap_x,
                    GemmEpilogue ep) {
  constexpr int W_BYTES = FM * UM * SLICE_BYTES;  // weight part of a stage; the token tile follows it
  constexpr int STAGE_BYTES = W_BYTES + UN * SLICE_BYTES;
  constexpr int STAGES = (RING_KB * 1024 / STAGE_BYTES) > 8 ? 8 : (RING_KB * 1024 / STAGE_BYTES);
  constexpr int ELEMS_PER_SLICE = FP8 ? 128 : 64;
  constexpr int TMEM_COLS = FM * UN < 32 ? 32 : FM * UN;
  static_assert(TMEM_COLS <= 512, "two accumulators of UN columns must fit the 512 TMEM columns");
  extern __shared__ uint8_t smem_raw[];
  __shared__ __align__(8) uint64_t bar_full[STAGES];
  __shared__ __align__(8) uint64_t bar_empty[STAGES];
  __shared__ __align__(8) uint64_t bar_acc;
  __shared__ uint32_t tmem_slot;
  __shared__ int abort_flag;
  __shared__ int32_t row_out[UN];   // output row of token row ml of this tile; negative = not written
  __shared__ __align__(16) float row_scale[UN];  // its activation scale (1 without scales)

  pdl_trigger();  // the next kernel may be scheduled now; it waits for this grid before touching y
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t tiles = (smem_u32(smem_raw) + 1023u) & ~1023u;
  const int n0 = blockIdx.x * (UM * FM), m0 = blockIdx.y * UN;
  const int total_kb = (ep.K + ELEMS_PER_SLICE - 1) / ELEMS_PER_SLICE;
  const int per_split = (total_kb + gridDim.z - 1) / gridDim.z;
  const int kb_begin = blockIdx.z * per_split;
  const int kb_end = min(total_kb, kb_begin + per_split);
  const int n_kb = max(0, kb_end - kb_begin);

  if (threadIdx.x == 0) {
    abort_flag = 0;
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(smem_u32(&bar_full[s]), 1);
      mbar_init(smem_u32(&bar_empty[s]), 1);
    }
    mbar_init(smem_u32(&bar_acc), 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&tmem_slot)),
                 "r"(TMEM_COLS)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  const uint32_t tmem_acc = tmem_slot;
  float ws_reduce[4] = {1.0f, 1.0f, 1.0f, 1.0f};  // epilogue warps: weight scales of the features a lane reduces

  if (warp == 0 && lane == 0) {
    // ---- TMA producer ----
    int issued = 0;
    const bool drop = *const_cast<volatile int*>(&g_drop_loads) != 0;  // test hook: arm the barriers, copy nothing
    // Weights never depend on the previous kernel: fill the ring with weight tiles right away, and
    // only then wait for the kernel that produces the activations (programmatic dependent launch).
    const int prefetch = n_kb < STAGES ? n_kb : STAGES;
    for (int i = 0; i < prefetch; ++i) {
      const uint32_t full = smem_u32(&bar_full[i]);
      mbar_expect_tx(full, STAGE_BYTES);
#pragma unroll
      for (int f = 0; f < FM; ++f)
        if (!drop)
          tma_load_2d(tiles + i * STAGE_BYTES + f * UM * SLICE_BYTES, &tmap_w, full, (kb_begin + i) * ELEMS_PER_SLICE,
                      n0 + f * UM);
    }
    pdl_wait();
    for (int i = 0; i < prefetch; ++i) {
      if (!drop)
        tma_load_2d(tiles + i * STAGE_BYTES + W_BYTES, &tmap_x, smem_u32(&bar_full[i]),
                    (kb_begin + i) * ELEMS_PER_SLICE, m0);
      issued = i + 1;
    }
    for (int i = prefetch; i < n_kb; ++i) {
      const int s = i % STAGES;
      const uint32_t parity = ((i / STAGES) & 1) ^ 1;
      if (!mbar_wait(smem_u32(&bar_empty[s]), parity, &abort_flag)) break;
      const uint32_t full = smem_u32(&bar_full[s]);
      mbar_expect_tx(full, STAGE_BYTES);
      const uint32_t a_dst = tiles + s * STAGE_BYTES, b_dst = a_dst + W_BYTES;
      const int k_elem = (kb_begin + i) * ELEMS_PER_SLICE;
      if (!drop) {
#pragma unroll
        for (int f = 0; f < FM; ++f) tma_load_2d(a_dst + f * UM * SLICE_BYTES, &tmap_w, full, k_elem, n0 + f * UM);
        tma_load_2d(b_dst, &tmap_x, full, k_elem, m0);
      }
      issued = i + 1;
    }
    if (abort_flag && !drop) {
      // let copies already in flight land before the CTA's shared memory is released
      for (int i = max(0, issued - STAGES); i < issued; ++i)
        mbar_wait(smem_u32(&bar_full[i % STAGES]), (i / STAGES) & 1, &abort_flag, true);
    }
  } else if (warp == 1 && lane == 0) {
    // ---- MMA issuer ----
    // instruction descriptor: fp32 accumulate, K-major A and B, N = UN, M = 128
    uint32_t idesc = (1u << 4) | (static_cast<uint32_t>(UN >> 3) << 17) | (static_cast<uint32_t>(UM >> 4) << 24);
    if (!FP8) idesc |= (1u << 7) | (1u << 10);  // bf16 operands (e4m3 is format 0)
    for (int i = 0; i < n_kb; ++i) {
      const int s = i % STAGES;
      if (!mbar_wait(smem_u32(&bar_full[s]), (i / STAGES) & 1, &abort_flag)) break;
      asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
      const uint32_t a_src = tiles + s * STAGE_BYTES, b_src = a_src + W_BYTES;
      const uint64_t da = umma_smem_desc(a_src), db = umma_smem_desc(b_src);
#pragma unroll
      for (int k = 0; k < SLICE_BYTES / 32; ++k) {  // one MMA consumes 32 bytes of K per row
        const uint32_t acc = (i > 0 || k > 0) ? 1u : 0u;
#pragma unroll
        for (int f = 0; f < FM; ++f) {  // feature sub-tile f: its weight rows, its accumulator columns
          const uint64_t dw = da + static_cast<uint64_t>(f * (UM * SLICE_BYTES / 16) + 2 * k);
          if (FP8) umma_fp8(tmem_acc + f * UN, dw, db + 2 * k, idesc, acc);
          else umma_bf16(tmem_acc + f * UN, dw, db + 2 * k, idesc, acc);
        }
      }
      umma_commit(smem_u32(&bar_empty[s]));
    }
    umma_commit(smem_u32(&bar_acc));
  } else if (warp >= 2) {
    // ---- epilogue: TMEM lane = output feature, column = token ----
    const int quarter = warp & 3;  // a warp may only touch TMEM lanes [32 * (warp % 4), +32)
    // Weight scales are constants of the model: fetch them before the wait, in the layout the final store
    // uses (split-K: lane l reduces features 4l .. 4l+3; else lane = feature of each sub-tile). A load issued
    // after the main loop would queue behind the other CTAs' tile traffic.
    float ws_direct[FM];
#pragma unroll
    for (int f = 0; f < FM; ++f) {
      const int n = n0 + f * UM + quarter * 32 + lane;
      ws_direct[f] = (!ep.partial && ep.w_scales != nullptr && n < ep.N) ? ep.w_scales[n] : 1.0f;
    }
    if (ep.partial && ep.w_scales != nullptr) {
#pragma unroll
      for (int j = 0; j < 4; ++j) ws_reduce[j] = n0 + 4 * lane + j < ep.N ? ep.w_scales[n0 + 4 * lane + j] : 1.0f;
    }
    pdl_wait();  // activation scales / row mask come from earlier kernels of the step
    // While the MMAs run: resolve where each token row of the tile goes and what scales it. The loops
    // below then depend on shared memory alone (one load from global memory per row and lane, between the
    // accumulator and the store, made the epilogue longer than the main loop).
    for (int ml = static_cast<int>(threadIdx.x) - 64; ml < UN; ml += 128) {
      const int m = m0 + ml;
      int out = -1;
      float xs = 1.0f;
      if (m < ep.M && (ep.row_mask == nullptr || ep.row_mask[m])) {
        out = ep.row_map != nullptr ? ep.row_map[m] : m;
        if (ep.x_scales != nullptr) xs = ep.x_scales[m];
      }
      row_out[ml] = out;
      row_scale[ml] = xs;
    }
    if (n_kb > 0) mbar_wait(smem_u32(&bar_acc), 0, &abort_flag);
    asm volatile("bar.sync 1, 128;" ::: "memory");  // the four epilogue warps agree on abort_flag and see the rows
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    if (abort_flag == 0 || ep.partial) {
      // rows of 8 features are stored as one 16-byte word when the tile lies inside y and rows are aligned
      const bool wide = !ep.partial && (ep.N & 7) == 0 && n0 + FM * UM <= ep.N;
      const bool scaled = ep.x_scales != nullptr;
      const bool live = n_kb > 0 && abort_flag == 0;  // else the accumulator was never written: the tile is zero
      // per warp: a [32 tokens][32 features] bf16 block of the idle ring turns the accumulator (lane =
      // feature) into token rows
      __nv_bfloat16* stage = reinterpret_cast<__nv_bfloat16*>(smem_raw + (tiles - smem_u32(smem_raw))) + quarter * 1024;
      // partial tile [UN][128]: in this CTA's shared memory (the ring is idle now) or in the workspace
      float* part = reinterpret_cast<float*>(smem_raw + (tiles - smem_u32(smem_raw)));
      if (ep.partial && ep.split_ws != nullptr)
        part = ep.split_ws + ((static_cast<size_t>(blockIdx.y) * gridDim.x + blockIdx.x) * gridDim.z + blockIdx.z) * (UN * UM);
      const int n_local = quarter * 32 + lane;
      constexpr int CHUNKS = UN / 32, TOTAL = FM * CHUNKS;  // blocks of 32 token columns, sub-tile major
      auto chunk_addr = [&](int i) {
        return tmem_acc + (static_cast<uint32_t>(quarter * 32) << 16) + static_cast<uint32_t>((i / CHUNKS) * UN + (i % CHUNKS) * 32);
      };
      auto emit = [&](int i, const uint32_t (&v)[32]) {
        const int f = i / CHUNKS, c = i % CHUNKS, n = n0 + f * UM + n_local;
        const float ws = (FM > 1 && f == 1) ? ws_direct[FM - 1] : ws_direct[0];
        if (ep.partial) {
#pragma unroll
          for (int j = 0; j < 32; ++j) part[(c * 32 + j) * UM + n_local] = live ? __uint_as_float(v[j]) : 0.0f;
        } else {
          store_block(ep, v, c, n, n0 + f * UM + quarter * 32, lane, wide, scaled, ws, stage, row_out, row_scale);
        }
      };
      // A TMEM load and its wait cost about half a microsecond back to back, whatever the width. A CTA that
      // owns its SM fetches 128 columns (four blocks) per wait. The half-SM kernels of the decode step fetch one
      // block at a time: their registers decide how early the CTAs of the NEXT kernel of the chain become
      // resident beside them, which is worth more there than a shorter epilogue.
      constexpr int GROUP = RING_KB > 96 ? (TOTAL < 4 ? TOTAL : 4) : 1;
      static_assert(TOTAL % GROUP == 0, "token tiles are 32, 64, 128 or 256 columns");
#pragma unroll 1
      for (int i = 0; i < TOTAL; i += GROUP) {
        uint32_t v[GROUP][32];
#pragma unroll
        for (int g = 0; g < GROUP; ++g) {
          if (live) {
            tmem_issue32(chunk_addr(i + g), v[g]);
          } else {
#pragma unroll
            for (int j = 0; j < 32; ++j) v[g][j] = 0u;
          }
        }
        if (live) {
#pragma unroll
          for (int g = 0; g < GROUP; ++g) tmem_wait32(v[g]);  // the first completes all; the rest tie the registers
        }
#pragma unroll
        for (int g = 0; g < GROUP; ++g) emit(i + g, v[g]);
      }
    }
  }

  if (ep.partial) {
    // Split-K across a thread-block cluster (one CTA per K range, cluster = grid.z): every CTA has
    // parked its fp32 partial tile in its own shared memory; after a cluster barrier CTA r sums, in
    // split order, the token rows m with m % splits == r straight out of its peers' shared memory
    // (distributed shared memory), applies scales / mask and writes y. Deterministic, no HBM round trip.
    __syncwarp();  // the producer / MMA lanes rejoin their warps before the aligned cluster barrier
    asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
    if (warp >= 2) {
      const int quarter = warp & 3;
      const uint32_t splits = gridDim.z, rank = blockIdx.z;
      if (ep.split_ws != nullptr) {
        const float* ws_tile =
            ep.split_ws + (static_cast<size_t>(blockIdx.y) * gridDim.x + blockIdx.x) * gridDim.z * (UN * UM);
        if (splits == 2) cluster_reduce_rows<2, UN, true>(ep, tiles, ws_tile, rank, quarter, lane, n0, row_out, row_scale, ws_reduce);
        else if (splits == 4) cluster_reduce_rows<4, UN, true>(ep, tiles, ws_tile, rank, quarter, lane, n0, row_out, row_scale, ws_reduce);
        else cluster_reduce_rows<8, UN, true>(ep, tiles, ws_tile, rank, quarter, lane, n0, row_out, row_scale, ws_reduce);
      } else {
        if (splits == 2) cluster_reduce_rows<2, UN, false>(ep, tiles, nullptr, rank, quarter, lane, n0, row_out, row_scale, ws_reduce);
        else if (splits == 4) cluster_reduce_rows<4, UN, false>(ep, tiles, nullptr, rank, quarter, lane, n0, row_out, row_scale, ws_reduce);
        else cluster_reduce_rows<8, UN, false>(ep, tiles, nullptr, rank, quarter, lane, n0, row_out, row_scale, ws_reduce);
      }
    }
    if (ep.split_ws == nullptr) {
      // nobody leaves (and frees its shared memory) while a peer may still be reading it
      __syncwarp();
      asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
    }
  }

  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  if (threadIdx.x == 0 && abort_flag) atomicOr(ep.status, CGYM_STATUS_WAIT_TIMEOUT);
  if (warp == 1) {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem_acc), "r"(TMEM_COLS) : "memory");
  }
}

// ---- CTA-pair form (tcgen05.mma.cta_group::2) --------------------------------------------------
// Two CTAs of a cluster (an SM pair) compute one [256 features x 256 tokens] tile: each stages its own 128
// weight rows and HALF of the token tile (128 rows), the leader (cluster rank 0) issues one MMA of M = 256,
// N = 256 per K step that reads both CTAs' shared memory and writes 128 accumulator lanes x 256 columns into
// EACH CTA's TMEM, and every CTA runs the epilogue for its own 128 features. Per FLOP a CTA moves the bytes of
// the single-CTA 256 x 256 tile, but it needs only 256 TMEM columns and a half-SM ring, so two pairs share an
// SM pair and one CTA's epilogue runs under the other's main loop.
// Protocol: both CTAs' copies complete on the LEADER's full barrier (the peer names it with mapa; the leader
// expects both stages' bytes); the leader's
// MMA thread commits every stage twice: to its own `done` barrier and, through the peer's mapped address, to
// the peer's `empty` barrier (a relay by remote arrive from the leader's producer added a microsecond and
// a half to the peer's refill loop and left the pair at 60 % of the tensor pipe); the accumulator barrier
// likewise. Every copy is a plain per-CTA TMA load. TMEM is allocated and freed by
// warp 1 of both CTAs with the cta_group::2 forms, the free after a cluster barrier.
__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
__device__ __forceinline__ uint32_t map_to_cta(uint32_t local_addr, uint32_t rank) {
  uint32_t out;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(out) : "r"(local_addr), "r"(rank));
  return out;
}
__device__ __forceinline__ void tma_load_2d_pair(uint32_t dst, const CUtensorMap* map, uint32_t leader_bar, int x, int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];"
      ::"r"(dst), "l"(reinterpret_cast<uint64_t>(map)), "r"(leader_bar), "r"(x), "r"(y)
      : "memory");
}
__device__ __forceinline__ void umma_pair(uint32_t tmem_d, uint64_t da, uint64_t db, uint32_t idesc, uint32_t acc, bool fp8) {
  if (fp8)
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::2.kind::f8f6f4 [%0], %1, %2, %3, p;\n\t}"
        ::"r"(tmem_d), "l"(da), "l"(db), "r"(idesc), "r"(acc)
        : "memory");
  else
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}"
        ::"r"(tmem_d), "l"(da), "l"(db), "r"(idesc), "r"(acc)
        : "memory");
}
__device__ __forceinline__ void umma_commit_pair(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar) : "memory");
}

// One block of 32 token columns of an accumulator (lane = feature n, v[j] = token row c * 32 + j of the tile) to y:
// scaled, rounded to bf16, transposed through a [32 tokens][32 features] staging block of the warp and written as
// 16-byte row segments when `wide` (the tile lies inside y and rows are 16-byte aligned), element by element
// otherwise. row_out / row_scale are the tile's staged row metadata (shared memory).
__device__ __forceinline__ void store_block(const GemmEpilogue& ep, const uint32_t (&v)[32], int c, int n, int n_base,
                                            int lane, bool wide, bool scaled, float ws, __nv_bfloat16* stage,
                                            const int32_t* row_out, const float* row_scale) {
  if (wide) {
#pragma unroll
    for (int j0 = 0; j0 < 32; j0 += 8) {
      // the scales of eight rows are read before the first store of the group: the compiler cannot tell that
      // the stores below leave row_scale alone, and would order every read behind the store before it
      float xs[8];
      *reinterpret_cast<float4*>(&xs[0]) = *reinterpret_cast<const float4*>(&row_scale[c * 32 + j0]);
      *reinterpret_cast<float4*>(&xs[4]) = *reinterpret_cast<const float4*>(&row_scale[c * 32 + j0 + 4]);
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        float val = __uint_as_float(v[j0 + j]);
        if (scaled) val = __fmul_rn(__fmul_rn(val, xs[j]), ws);
        stage[(j0 + j) * 32 + lane] = __float2bfloat16_rn(val);
      }
    }
    __syncwarp();
    // four lanes per token row (8 features = 16 bytes each), eight rows per pass
#pragma unroll
    for (int pass = 0; pass < 4; ++pass) {
      const int row = pass * 8 + (lane >> 2);
      const uint4 word = *reinterpret_cast<const uint4*>(stage + row * 32 + (lane & 3) * 8);
      const int out_row = row_out[c * 32 + row];
      if (out_row >= 0)
        *reinterpret_cast<uint4*>(ep.y + static_cast<int64_t>(out_row) * ep.N + n_base + (lane & 3) * 8) = word;
    }
    __syncwarp();
  } else if (n < ep.N) {
#pragma unroll
    for (int j = 0; j < 32; ++j) {
      const int out_row = row_out[c * 32 + j];
      if (out_row < 0) continue;
      float val = __uint_as_float(v[j]);
      if (scaled) val = __fmul_rn(__fmul_rn(val, row_scale[c * 32 + j]), ws);
      ep.y[static_cast<int64_t>(out_row) * ep.N + n] = __float2bfloat16_rn(val);
    }
  }
}

constexpr int PAIR_TOKENS = 256;  // token tile of a pair
constexpr int PAIR_HALF = 128;    // token rows a CTA stages
constexpr int PAIR_STAGES = 3;
constexpr int PAIR_EPILOGUE_GROUP = 2;

template <bool FP8>
__global__ void __launch_bounds__(GEMM_THREADS, 2)
gemm_pair_kernel(const __grid_constant__ CUtensorMap tmap_w, const __grid_constant__ CUtensorMap tmap_x,
                 GemmEpilogue ep) {
  constexpr int UN = PAIR_TOKENS, STAGES = PAIR_STAGES;
  constexpr int W_BYTES = UM * SLICE_BYTES, STAGE_BYTES = W_BYTES + PAIR_HALF * SLICE_BYTES;
  constexpr int ELEMS_PER_SLICE = FP8 ? 128 : 64;
  constexpr int TMEM_COLS = UN;
  extern __shared__ uint8_t smem_raw[];
  __shared__ __align__(8) uint64_t bar_full[STAGES];   // leader: both CTAs' copies of a stage have landed
  __shared__ __align__(8) uint64_t bar_done[STAGES];   // leader: the MMAs that read a stage have completed
  __shared__ __align__(8) uint64_t bar_empty[STAGES];  // peer: the leader passed `done` on
  __shared__ __align__(8) uint64_t bar_acc;            // the accumulator is complete (peer: passed on by the leader)
  __shared__ uint32_t tmem_slot;
  __shared__ int abort_flag;
  __shared__ int32_t row_out[UN];
  __shared__ __align__(16) float row_scale[UN];

  // No early griddepcontrol.launch_dependents here: a pair needs the SAME free TMEM columns on both of its SMs,
  // and clusters can become resident late (the stragglers seen with split-K clusters). A successor GEMM of a
  // dependent-launch chain that became resident early would allocate TMEM columns and then wait for this grid,
  // while a late pair of this grid waits for those columns: a cycle of two unbounded waits. Without the trigger
  // the successor starts when every CTA of this grid has exited. (w13 of a 256-row decode step routed through
  // this kernel with the trigger hung; this cycle is the explanation that fits.)
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = cluster_rank();
  const bool leader = rank == 0;
  const uint32_t tiles = (smem_u32(smem_raw) + 1023u) & ~1023u;
  const int n0 = blockIdx.x * UM, m0 = blockIdx.y * UN;
  const int n_kb = (ep.K + ELEMS_PER_SLICE - 1) / ELEMS_PER_SLICE;

  if (threadIdx.x == 0) {
    abort_flag = 0;
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(smem_u32(&bar_full[s]), 1);
      mbar_init(smem_u32(&bar_done[s]), 1);
      mbar_init(smem_u32(&bar_empty[s]), 1);
    }
    mbar_init(smem_u32(&bar_acc), 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&tmem_slot)),
                 "r"(TMEM_COLS)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  // both CTAs' barriers exist before either touches the other's
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  const uint32_t tmem_acc = tmem_slot;

  if (warp == 0 && lane == 0) {
    // ---- TMA producer (both CTAs) ----
    const int x_row = m0 + static_cast<int>(rank) * PAIR_HALF;
    const uint32_t full0 = leader ? smem_u32(&bar_full[0]) : map_to_cta(smem_u32(&bar_full[0]), 0);
    auto load = [&](uint32_t dst, const CUtensorMap* map, uint32_t full, int x, int y) {
      if (leader) tma_load_2d(dst, map, full, x, y);
      else tma_load_2d_pair(dst, map, full, x, y);  // completes on the leader's barrier
    };
    // weights never depend on the previous kernel: the first ring of weight tiles goes out before the wait
    const int prefetch = n_kb < STAGES ? n_kb : STAGES;
    for (int i = 0; i < prefetch; ++i) {
      const uint32_t full = full0 + static_cast<uint32_t>(i) * 8u;
      if (leader) mbar_expect_tx(full, 2 * STAGE_BYTES);
      load(tiles + i * STAGE_BYTES, &tmap_w, full, i * ELEMS_PER_SLICE, n0);
    }
    pdl_wait();
    for (int i = 0; i < prefetch; ++i)
      load(tiles + i * STAGE_BYTES + W_BYTES, &tmap_x, full0 + static_cast<uint32_t>(i) * 8u, i * ELEMS_PER_SLICE, x_row);
    for (int i = prefetch; i < n_kb; ++i) {
      const int s = i % STAGES;
      // leader: the MMAs that read the stage have completed; peer: the leader's MMA thread said so
      const uint32_t freed = smem_u32(leader ? &bar_done[s] : &bar_empty[s]);
      if (!mbar_wait(freed, ((i / STAGES) & 1) ^ 1, &abort_flag)) break;
      const uint32_t full = full0 + static_cast<uint32_t>(s) * 8u;
      if (leader) mbar_expect_tx(full, 2 * STAGE_BYTES);
      const uint32_t a_dst = tiles + s * STAGE_BYTES;
      load(a_dst, &tmap_w, full, i * ELEMS_PER_SLICE, n0);
      load(a_dst + W_BYTES, &tmap_x, full, i * ELEMS_PER_SLICE, x_row);
    }
  } else if (warp == 1 && lane == 0 && leader) {
    // ---- MMA issuer (leader only): M = 256 (128 features per CTA), N = 256 tokens (128 staged per CTA) ----
    uint32_t idesc = (1u << 4) | (static_cast<uint32_t>(UN >> 3) << 17) | (static_cast<uint32_t>(256 >> 4) << 24);
    if (!FP8) idesc |= (1u << 7) | (1u << 10);
    const uint32_t peer_empty = map_to_cta(smem_u32(&bar_empty[0]), 1);
    for (int i = 0; i < n_kb; ++i) {
      const int s = i % STAGES;
      if (!mbar_wait(smem_u32(&bar_full[s]), (i / STAGES) & 1, &abort_flag)) break;
      asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
      const uint32_t a_src = tiles + s * STAGE_BYTES, b_src = a_src + W_BYTES;
      const uint64_t da = umma_smem_desc(a_src), db = umma_smem_desc(b_src);
#pragma unroll
      for (int k = 0; k < SLICE_BYTES / 32; ++k)
        umma_pair(tmem_acc, da + 2 * k, db + 2 * k, idesc, (i > 0 || k > 0) ? 1u : 0u, FP8);
      umma_commit_pair(smem_u32(&bar_done[s]));
      umma_commit_pair(peer_empty + static_cast<uint32_t>(s) * 8u);  // the peer may refill its half of the stage
    }
    umma_commit_pair(smem_u32(&bar_acc));
    umma_commit_pair(map_to_cta(smem_u32(&bar_acc), 1));
  } else if (warp >= 2) {
    // ---- epilogue (both CTAs): TMEM lane = one of this CTA's 128 features, column = token of the pair's tile ----
    const int quarter = warp & 3;
    const int n_local = quarter * 32 + lane, n = n0 + n_local;
    const float ws = (ep.w_scales != nullptr && n < ep.N) ? ep.w_scales[n] : 1.0f;
    pdl_wait();  // activation scales / row mask come from earlier kernels of the step
    for (int ml = static_cast<int>(threadIdx.x) - 64; ml < UN; ml += 128) {
      const int m = m0 + ml;
      int out = -1;
      float xs = 1.0f;
      if (m < ep.M && (ep.row_mask == nullptr || ep.row_mask[m])) {
        out = ep.row_map != nullptr ? ep.row_map[m] : m;
        if (ep.x_scales != nullptr) xs = ep.x_scales[m];
      }
      row_out[ml] = out;
      row_scale[ml] = xs;
    }
    if (n_kb > 0) mbar_wait(smem_u32(&bar_acc), 0, &abort_flag);
    asm volatile("bar.sync 1, 128;" ::: "memory");
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    if (abort_flag == 0) {
      const bool wide = (ep.N & 7) == 0 && n0 + UM <= ep.N;
      const bool scaled = ep.x_scales != nullptr;
      const bool live = n_kb > 0;
      __nv_bfloat16* stage = reinterpret_cast<__nv_bfloat16*>(smem_raw + (tiles - smem_u32(smem_raw))) + quarter * 1024;
      auto emit = [&](int c, const uint32_t (&v)[32]) {
        store_block(ep, v, c, n, n0 + quarter * 32, lane, wide, scaled, ws, stage, row_out, row_scale);
      };
      constexpr int GROUP = PAIR_EPILOGUE_GROUP;  // blocks of 32 columns fetched per TMEM wait
#pragma unroll 1
      for (int c0 = 0; c0 < UN / 32; c0 += GROUP) {
        uint32_t v[GROUP][32];
#pragma unroll
        for (int g = 0; g < GROUP; ++g) {
#pragma unroll
          for (int j = 0; j < 32; ++j) v[g][j] = 0u;
          if (live) tmem_issue32(tmem_acc + (static_cast<uint32_t>(quarter * 32) << 16) + static_cast<uint32_t>((c0 + g) * 32), v[g]);
        }
        if (live) {
#pragma unroll
          for (int g = 0; g < GROUP; ++g) tmem_wait32(v[g]);
        }
#pragma unroll
        for (int g = 0; g < GROUP; ++g) emit(c0 + g, v[g]);
      }
    }
  }

  // neither CTA frees its half of the pair's TMEM, or leaves, while the other may still use it
  __syncwarp();
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
  if (threadIdx.x == 0 && abort_flag) atomicOr(ep.status, CGYM_STATUS_WAIT_TIMEOUT);
  if (warp == 1) {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem_acc), "r"(TMEM_COLS) : "memory");
  }
}

// Persistent CTA-pair form for prefill-sized token counts: one pair per SM pair walks over the output tiles
// (tile t, t + pairs, ...), a six-stage ring (192 KB) streams without a break from one tile into the next, and
// the 512 TMEM columns hold TWO accumulators of 256 columns, so the epilogue of tile j (TMEM -> bf16 rows ->
// global, through a staging block of its own) runs under the main loop of tile j + 1 in the same CTA. Barriers
// beyond the one-tile form: acc_full[2] (leader commits to its own and to the peer's) and, in the leader,
// acc_empty[2] with two arrivals per use: the leader's and the peer's epilogue have both read the buffer.
constexpr int PP_STAGES = 6;

template <bool FP8>
__global__ void __launch_bounds__(GEMM_THREADS, 1)
gemm_pair_persistent_kernel(const __grid_constant__ CUtensorMap tmap_w, const __grid_constant__ CUtensorMap tmap_x,
                            GemmEpilogue ep, int pairs_n, int n_tiles_total) {
  constexpr int UN = PAIR_TOKENS, STAGES = PP_STAGES;
  constexpr int W_BYTES = UM * SLICE_BYTES, STAGE_BYTES = W_BYTES + PAIR_HALF * SLICE_BYTES;
  constexpr int ELEMS_PER_SLICE = FP8 ? 128 : 64;
  constexpr int TMEM_COLS = 2 * UN;
  extern __shared__ uint8_t smem_raw[];
  __shared__ __align__(8) uint64_t bar_full[STAGES], bar_done[STAGES], bar_empty[STAGES];
  __shared__ __align__(8) uint64_t bar_acc_full[2], bar_acc_empty[2];
  __shared__ uint32_t tmem_slot;
  __shared__ int abort_flag;
  __shared__ int32_t row_out[UN];
  __shared__ __align__(16) float row_scale[UN];

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = cluster_rank();
  const bool leader = rank == 0;
  const uint32_t tiles = (smem_u32(smem_raw) + 1023u) & ~1023u;
  const uint32_t stage_block = tiles + STAGES * STAGE_BYTES;  // 4 x 2 KB of epilogue staging behind the ring
  const int n_kb = (ep.K + ELEMS_PER_SLICE - 1) / ELEMS_PER_SLICE;
  const int pair_id = blockIdx.x >> 1, n_pairs = gridDim.x >> 1;
  const int my_tiles = pair_id < n_tiles_total ? (n_tiles_total - pair_id + n_pairs - 1) / n_pairs : 0;

  if (threadIdx.x == 0) {
    abort_flag = 0;
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(smem_u32(&bar_full[s]), 1);
      mbar_init(smem_u32(&bar_done[s]), 1);
      mbar_init(smem_u32(&bar_empty[s]), 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(smem_u32(&bar_acc_full[b]), 1);
      mbar_init(smem_u32(&bar_acc_empty[b]), 2);
    }
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&tmem_slot)),
                 "r"(TMEM_COLS)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  const uint32_t tmem_acc = tmem_slot;

  if (warp == 0 && lane == 0) {
    // ---- TMA producer (both CTAs): one stream of K slices over all of the pair's tiles ----
    const uint32_t full0 = leader ? smem_u32(&bar_full[0]) : map_to_cta(smem_u32(&bar_full[0]), 0);
    pdl_wait();
    int g = 0;
    bool ok = true;
    for (int j = 0; ok && j < my_tiles; ++j) {
      const int t = pair_id + j * n_pairs;
      const int n0 = ((t % pairs_n) * 2 + static_cast<int>(rank)) * UM;
      const int x_row = (t / pairs_n) * UN + static_cast<int>(rank) * PAIR_HALF;
      for (int i = 0; i < n_kb; ++i, ++g) {
        const int s = g % STAGES;
        if (g >= STAGES) {
          const uint32_t freed = smem_u32(leader ? &bar_done[s] : &bar_empty[s]);
          if (!mbar_wait(freed, ((g / STAGES) & 1) ^ 1, &abort_flag)) { ok = false; break; }
        }
        const uint32_t full = full0 + static_cast<uint32_t>(s) * 8u;
        const uint32_t a_dst = tiles + s * STAGE_BYTES;
        if (leader) {
          mbar_expect_tx(full, 2 * STAGE_BYTES);
          tma_load_2d(a_dst, &tmap_w, full, i * ELEMS_PER_SLICE, n0);
          tma_load_2d(a_dst + W_BYTES, &tmap_x, full, i * ELEMS_PER_SLICE, x_row);
        } else {
          tma_load_2d_pair(a_dst, &tmap_w, full, i * ELEMS_PER_SLICE, n0);
          tma_load_2d_pair(a_dst + W_BYTES, &tmap_x, full, i * ELEMS_PER_SLICE, x_row);
        }
      }
    }
  } else if (warp == 1 && lane == 0 && leader) {
    // ---- MMA issuer (leader only) ----
    uint32_t idesc = (1u << 4) | (static_cast<uint32_t>(UN >> 3) << 17) | (static_cast<uint32_t>(256 >> 4) << 24);
    if (!FP8) idesc |= (1u << 7) | (1u << 10);
    const uint32_t peer_empty = map_to_cta(smem_u32(&bar_empty[0]), 1);
    const uint32_t peer_acc_full = map_to_cta(smem_u32(&bar_acc_full[0]), 1);
    int g = 0;
    bool ok = true;
    for (int j = 0; ok && j < my_tiles; ++j) {
      const int b = j & 1;
      // both epilogues have read what tile j - 2 left in this buffer
      if (j >= 2 && !mbar_wait(smem_u32(&bar_acc_empty[b]), ((j >> 1) & 1) ^ 1, &abort_flag)) break;
      asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
      for (int i = 0; i < n_kb; ++i, ++g) {
        const int s = g % STAGES;
        if (!mbar_wait(smem_u32(&bar_full[s]), (g / STAGES) & 1, &abort_flag)) { ok = false; break; }
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        const uint32_t a_src = tiles + s * STAGE_BYTES, b_src = a_src + W_BYTES;
        const uint64_t da = umma_smem_desc(a_src), db = umma_smem_desc(b_src);
#pragma unroll
        for (int k = 0; k < SLICE_BYTES / 32; ++k)
          umma_pair(tmem_acc + static_cast<uint32_t>(b * UN), da + 2 * k, db + 2 * k, idesc, (i > 0 || k > 0) ? 1u : 0u, FP8);
        umma_commit_pair(smem_u32(&bar_done[s]));
        umma_commit_pair(peer_empty + static_cast<uint32_t>(s) * 8u);
      }
      if (!ok) break;
      umma_commit_pair(smem_u32(&bar_acc_full[b]));
      umma_commit_pair(peer_acc_full + static_cast<uint32_t>(b) * 8u);
    }
  } else if (warp >= 2) {
    // ---- epilogue (both CTAs), one tile behind the MMAs ----
    const int quarter = warp & 3;
    const uint32_t leader_acc_empty = map_to_cta(smem_u32(&bar_acc_empty[0]), 0);
    pdl_wait();
    const bool scaled = ep.x_scales != nullptr;
    __nv_bfloat16* stage = reinterpret_cast<__nv_bfloat16*>(smem_raw + (stage_block - smem_u32(smem_raw))) + quarter * 1024;
    for (int j = 0; j < my_tiles; ++j) {
      const int b = j & 1, t = pair_id + j * n_pairs;
      const int n0 = ((t % pairs_n) * 2 + static_cast<int>(rank)) * UM, m0 = (t / pairs_n) * UN;
      const int n = n0 + quarter * 32 + lane;
      const float ws = (ep.w_scales != nullptr && n < ep.N) ? ep.w_scales[n] : 1.0f;
      asm volatile("bar.sync 1, 128;" ::: "memory");  // the previous tile's rows are no longer read
      for (int ml = static_cast<int>(threadIdx.x) - 64; ml < UN; ml += 128) {
        const int m = m0 + ml;
        int out = -1;
        float xs = 1.0f;
        if (m < ep.M && (ep.row_mask == nullptr || ep.row_mask[m])) {
          out = ep.row_map != nullptr ? ep.row_map[m] : m;
          if (scaled) xs = ep.x_scales[m];
        }
        row_out[ml] = out;
        row_scale[ml] = xs;
      }
      const bool got = mbar_wait(smem_u32(&bar_acc_full[b]), (j >> 1) & 1, &abort_flag);
      asm volatile("bar.sync 1, 128;" ::: "memory");
      asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
      if (!got || abort_flag) break;
      const bool wide = (ep.N & 7) == 0 && n0 + UM <= ep.N;
#pragma unroll 1
      for (int c = 0; c < UN / 32; ++c) {
        uint32_t v[32];
        tmem_issue32(tmem_acc + (static_cast<uint32_t>(quarter * 32) << 16) + static_cast<uint32_t>(b * UN + c * 32), v);
        tmem_wait32(v);
        store_block(ep, v, c, n, n0 + quarter * 32, lane, wide, scaled, ws, stage, row_out, row_scale);
      }
      // this CTA's four warps have read the buffer: one arrival per CTA on the leader's barrier
      asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
      asm volatile("bar.sync 1, 128;" ::: "memory");
      if (threadIdx.x == 64)
        asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(leader_acc_empty + static_cast<uint32_t>(b) * 8u) : "memory");
    }
  }

  __syncwarp();
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
  if (threadIdx.x == 0 && abort_flag) atomicOr(ep.status, CGYM_STATUS_WAIT_TIMEOUT);
  if (warp == 1) {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem_acc), "r"(TMEM_COLS) : "memory");
  }
}

// ---- host side -------------------------------------------------------------------------------
using EncodeFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                              const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                              CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeFn tensor_map_encoder() {
  static EncodeFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* sym = nullptr;
    cudaDriverEntryPointQueryResult result;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &sym, cudaEnableDefault, &result) == cudaSuccess &&
        result == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeFn>(sym);
  });
  return fn;
}

static int make_map(CUtensorMap* map, const void* base, int rows, int k, int box_rows, bool fp8) {
  EncodeFn encode = tensor_map_encoder();
  CGYM_REQUIRE(encode != nullptr, "gemm: cuTensorMapEncodeTiled is not available from the driver");
  const cuuint64_t dims[2] = {static_cast<cuuint64_t>(k), static_cast<cuuint64_t>(rows)};
  const cuuint64_t strides[1] = {static_cast<cuuint64_t>(k) * (fp8 ? 1 : 2)};
  const cuuint32_t box[2] = {static_cast<cuuint32_t>(fp8 ? 128 : 64), static_cast<cuuint32_t>(box_rows)};
  const cuuint32_t elem_strides[2] = {1, 1};
  const CUresult rc = encode(map, fp8 ? CU_TENSOR_MAP_DATA_TYPE_UINT8 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2,
                             const_cast<void*>(base), dims, strides, box, elem_strides, CU_TENSOR_MAP_INTERLEAVE_NONE,
                             CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  CGYM_REQUIRE(rc == CUDA_SUCCESS, "gemm: cuTensorMapEncodeTiled failed with code %d", static_cast<int>(rc));
  return 0;
}

template <int UN, bool FP8, int RING_KB, int FM = 1>
static int launch_tile(const CUtensorMap& mw, const CUtensorMap& mx, const GemmEpilogue& ep, dim3 grid,
                       cudaStream_t stream) {
  constexpr int STAGE_BYTES = (UM * FM + UN) * SLICE_BYTES;
  constexpr int STAGES = (RING_KB * 1024 / STAGE_BYTES) > 8 ? 8 : (RING_KB * 1024 / STAGE_BYTES);
  constexpr int SMEM = STAGES * STAGE_BYTES + 1024;
  static_assert(UN * UM * 4 <= STAGES * STAGE_BYTES, "the split-K partial tile must fit in the idle ring");
  static SmemReservation reservation;  // per instantiation
  if (int rc = reserve_dynamic_smem(gemm_tcgen05_kernel<UN, FP8, RING_KB, FM>, SMEM, reservation, "gemm(tcgen05)")) return rc;
  cudaLaunchConfig_t config = {};
  config.gridDim = grid;
  config.blockDim = dim3(GEMM_THREADS);
  config.dynamicSmemBytes = SMEM;
  config.stream = stream;
  cudaLaunchAttribute attrs[2];
  int n_attrs = 0;
  if (g_pdl_enabled) {
    attrs[n_attrs].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attrs[n_attrs].val.programmaticStreamSerializationAllowed = 1;
    ++n_attrs;
  }
  if (grid.z > 1) {  // the K splits of one output tile form a cluster
    attrs[n_attrs].id = cudaLaunchAttributeClusterDimension;
    attrs[n_attrs].val.clusterDim.x = 1;
    attrs[n_attrs].val.clusterDim.y = 1;
    attrs[n_attrs].val.clusterDim.z = grid.z;
    ++n_attrs;
  }
  config.attrs = attrs;
  config.numAttrs = n_attrs;
  const cudaError_t rc = cudaLaunchKernelEx(&config, gemm_tcgen05_kernel<UN, FP8, RING_KB, FM>, mw, mx, ep);
  CGYM_REQUIRE(rc == cudaSuccess, "gemm(tcgen05): launch failed: %s", cudaGetErrorString(rc));
  return 0;
}


template <bool FP8>
static int launch_pair(const CUtensorMap& mw, const CUtensorMap& mx, const GemmEpilogue& ep, dim3 grid,
                       cudaStream_t stream) {
  constexpr int SMEM = PAIR_STAGES * (UM + PAIR_HALF) * SLICE_BYTES + 1024;
  static SmemReservation reservation;
  if (int rc = reserve_dynamic_smem(gemm_pair_kernel<FP8>, SMEM, reservation, "gemm(pair)")) return rc;
  cudaLaunchConfig_t config = {};
  config.gridDim = grid;
  config.blockDim = dim3(GEMM_THREADS);
  config.dynamicSmemBytes = SMEM;
  config.stream = stream;
  cudaLaunchAttribute attrs[2];
  int n_attrs = 0;
  attrs[n_attrs].id = cudaLaunchAttributeClusterDimension;  // consecutive feature tiles form the pair
  attrs[n_attrs].val.clusterDim.x = 2;
  attrs[n_attrs].val.clusterDim.y = 1;
  attrs[n_attrs].val.clusterDim.z = 1;
  ++n_attrs;
  if (g_pdl_enabled) {
    attrs[n_attrs].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attrs[n_attrs].val.programmaticStreamSerializationAllowed = 1;
    ++n_attrs;
  }
  config.attrs = attrs;
  config.numAttrs = n_attrs;
  const cudaError_t rc = cudaLaunchKernelEx(&config, gemm_pair_kernel<FP8>, mw, mx, ep);
  CGYM_REQUIRE(rc == cudaSuccess, "gemm(pair): launch failed: %s", cudaGetErrorString(rc));
  return check_launch("gemm_pair");
}

template <bool FP8>
static int launch_pair_persistent(const CUtensorMap& mw, const CUtensorMap& mx, const GemmEpilogue& ep, int pairs_n,
                                  int m_tiles, cudaStream_t stream) {
  constexpr int SMEM = PP_STAGES * (UM + PAIR_HALF) * SLICE_BYTES + 4 * 2048 + 1024;
  static SmemReservation reservation;
  if (int rc = reserve_dynamic_smem(gemm_pair_persistent_kernel<FP8>, SMEM, reservation, "gemm(pair, persistent)")) return rc;
  const int n_tiles_total = pairs_n * m_tiles;
  const int pairs = n_tiles_total < 74 ? n_tiles_total : 74;  // one pair per SM pair
  cudaLaunchConfig_t config = {};
  config.gridDim = dim3(2 * pairs);
  config.blockDim = dim3(GEMM_THREADS);
  config.dynamicSmemBytes = SMEM;
  config.stream = stream;
  cudaLaunchAttribute attrs[2];
  int n_attrs = 0;
  attrs[n_attrs].id = cudaLaunchAttributeClusterDimension;
  attrs[n_attrs].val.clusterDim.x = 2;
  attrs[n_attrs].val.clusterDim.y = 1;
  attrs[n_attrs].val.clusterDim.z = 1;
  ++n_attrs;
  if (g_pdl_enabled) {
    attrs[n_attrs].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attrs[n_attrs].val.programmaticStreamSerializationAllowed = 1;
    ++n_attrs;
  }
  config.attrs = attrs;
  config.numAttrs = n_attrs;
  const cudaError_t rc = cudaLaunchKernelEx(&config, gemm_pair_persistent_kernel<FP8>, mw, mx, ep, pairs_n, n_tiles_total);
  CGYM_REQUIRE(rc == cudaSuccess, "gemm(pair, persistent): launch failed: %s", cudaGetErrorString(rc));
  return check_launch("gemm_pair_persistent");
}

bool gemm_tcgen05_supports(int M, int N, int K, bool fp8, const void* x, const void* w) {
  const int elem = fp8 ? 1 : 2;
  if (M <= 0 || N <= 0 || K <= 0) return false;
  if ((static_cast<int64_t>(K) * elem) % 16 != 0) return false;  // TMA row pitch
  if ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(w)) & 15u) return false;
  return true;
}

// Which kernel, tile and grid a GEMM takes: a pure function of the shape, the operand type, the caller's
// forcing code and whether the launch is part of a dependent-launch chain (a captured decode step).
struct GemmPlan {
  int kind;    // 0 = single-CTA tiles, 1 = CTA pairs (one tile per pair), 2 = persistent CTA pairs
  int un;      // token tile (MMA N)
  int fm;      // 128-feature sub-tiles per CTA (single-CTA tiles only)
  int splits;  // K splits = cluster size along z (single-CTA tiles only)
  int grid_x, grid_y;
};

static GemmPlan plan_gemm(int M, int N, int K, bool fp8, int force_splits, bool pdl) {
  // CTA pairs (256 features x 256 tokens per pair, unsplit) where they measured faster than the single-CTA
  // tiles: prefill-sized token counts with a contraction of up to 4096 (w13, in-projection, qkv: +5..10 % in
  // the persistent form; at K = 8192, 128 tiles, both forms lose to the single CTA by their last round), and
  // the LM head of a full decode batch (+8 %, one-tile form).
  // Inside a dependent-launch chain (a captured decode step) only the LM head of a 129..256-row batch takes
  // pairs: a 512-row decode step whose projections ran as pairs stopped making progress (the step probe did
  // not finish within its 100 s; the GPU stayed usable), and the cause was not found by reading, so that
  // combination stays off. Prefill and scoring launch outside such chains.
  const bool pair_auto = force_splits == 0 && N % (2 * UM) == 0 &&
                         ((M > 256 && K <= 4096 && !pdl) || (M > 128 && M <= 256 && N / (2 * UM) >= 148));
  if (force_splits == -2 || force_splits == -3 || pair_auto) {
    const int grid_x = N / UM, grid_y = (M + PAIR_TOKENS - 1) / PAIR_TOKENS;
    // two rounds or more of tiles over the 74 SM pairs: the persistent form (epilogue under the next tile's main
    // loop); fewer tiles leave it idle in its last round and the one-tile form with two CTAs per SM is as fast
    const bool persistent = force_splits == -3 || (pair_auto && M > 256 && grid_x / 2 * grid_y >= 2 * 74);
    return GemmPlan{persistent ? 2 : 1, PAIR_TOKENS, 1, 1, grid_x, grid_y};
  }
  // Token tile: the smallest that covers M up to 128; up to 256 rows (a full decode batch) tiles of 128
  // or 64 keep the weight-streaming layout (half-SM rings, split-K) - the other tiles' weight loads hit
  // L2 - and only larger M (prefill) takes the 256-token tile that halves L2 -> SM traffic per FLOP.
  int un = M <= 32 ? 32 : (M <= 64 ? 64 : (M <= 256 ? 128 : 256));
  // A full decode batch (129..256 rows) takes 64-token tiles where all of them still fit the GPU's resident
  // slots at once (every projection of the 1.2B model except w13 and the LM head): with four token tiles
  // the K dimension needs half as many splits to fill the SMs, so half as many fp32 partial tiles are written
  // and read back, the clusters are half as large (eight co-resident CTAs in one GPC often had to wait for
  // the previous kernel to drain), and a CTA's epilogue covers 64 columns instead of 128. The weight tiles
  // are fetched by four token tiles instead of two - out of L2, which has the bandwidth to spare here.
  if (M > 128 && M <= 256 && ((N + UM - 1) / UM) * ((M + 63) / 64) <= 2 * 148) un = 64;
  // Two feature sub-tiles per CTA (one fetch of the token tile serves 256 features) for unsplit GEMMs
  // over more than 128 tokens. With 256-token tiles (prefill) it pays unless halving the CTA count costs
  // more in the last, partly filled wave than the saved traffic gains; for a decode batch of 129..256
  // rows only the LM head is large enough, and it then takes the 256-token tile as well.
  bool dual = false;
  if (M > 128 && N % (2 * UM) == 0 && force_splits <= 1) {
    auto wave_fill = [](int ctas) { return static_cast<double>(ctas) / (148.0 * ((ctas + 147) / 148)); };
    if (un == 256) {
      const int single = (N / UM) * ((M + 255) / 256);
      dual = wave_fill(single / 2) >= wave_fill(single) - 0.1;
    } else if (N / (2 * UM) >= 148) {
      un = 256;
      dual = true;
    }
  }
  const int n_tiles = (N + UM - 1) / UM, m_tiles = (M + un - 1) / un;
  const int total_kb = (K + (fp8 ? 128 : 64) - 1) / (fp8 ? 128 : 64);
  // decode-sized token tiles take the half-SM ring (two CTAs per SM), larger ones the full ring
  const bool half_ring = un <= 128;
  // Split-K until the CTAs fill the GPU's resident slots (at most 8: the portable cluster size). A
  // weight stream is bound by the bytes in flight, i.e. by how many rings are filling at once, so a
  // decode GEMM wants about two CTAs on every SM, each owning as little as one ring of K slices.
  constexpr int min_kb = 4;  // fewest K slices per split: one fill of the half-SM ring
  int splits = 1;
  if (force_splits > 0) {
    splits = force_splits;
  } else {
    const int slots = half_ring ? 2 * 148 : 148;
    splits = slots / (n_tiles * m_tiles);
    if (splits > total_kb / min_kb) splits = total_kb / min_kb;
  }
  if (dual) splits = 1;
  if (splits > 8) splits = 8;
  if (splits > total_kb) splits = total_kb;
  splits = splits >= 8 ? 8 : (splits >= 4 ? 4 : (splits >= 2 ? 2 : 1));  // cluster sizes the reduction is built for
  // every split must own at least one K slice
  while (splits > 1 && (splits - 1) * ((total_kb + splits - 1) / splits) >= total_kb) splits /= 2;
  return GemmPlan{0, un, dual ? 2 : 1, splits, dual ? n_tiles / 2 : n_tiles, m_tiles};
}

int launch_gemm_tcgen05(void* y, const void* x, const void* w, const float* x_scales, const float* w_scales,
                        const uint8_t* row_mask, const int32_t* row_map, int M, int N, int K, bool fp8,
                        void* workspace, int64_t workspace_bytes, int32_t* status, int force_splits,
                        cudaStream_t stream) {
  CGYM_REQUIRE(gemm_tcgen05_supports(M, N, K, fp8, x, w),
               "gemm(tcgen05): needs 16-byte aligned operands and a K row pitch that is a multiple of 16 bytes");
  CGYM_REQUIRE(status != nullptr, "gemm(tcgen05): a status word is required");
  const GemmPlan plan = plan_gemm(M, N, K, fp8, force_splits, g_pdl_enabled != 0);
  if (plan.kind != 0) {
    CGYM_REQUIRE(N % (2 * UM) == 0, "gemm(pair): the feature count must be a multiple of 256");
    CUtensorMap mw, mx;
    if (int rc = make_map(&mw, w, N, K, UM, fp8)) return rc;
    if (int rc = make_map(&mx, x, M, K, PAIR_HALF, fp8)) return rc;
    GemmEpilogue ep{static_cast<__nv_bfloat16*>(y), x_scales, w_scales, row_mask, row_map, status, M, N, K, 0, nullptr};
    if (plan.kind == 2)
      return fp8 ? launch_pair_persistent<true>(mw, mx, ep, N / (2 * UM), plan.grid_y, stream)
                 : launch_pair_persistent<false>(mw, mx, ep, N / (2 * UM), plan.grid_y, stream);
    const dim3 grid(plan.grid_x, plan.grid_y, 1);
    return fp8 ? launch_pair<true>(mw, mx, ep, grid, stream) : launch_pair<false>(mw, mx, ep, grid, stream);
  }
  const int un = plan.un, splits = plan.splits;
  const bool dual = plan.fm == 2, half_ring = un <= 128;
  const int n_tiles = (N + UM - 1) / UM, m_tiles = plan.grid_y;
  // partial tiles go through the caller's workspace (L2) when it is large enough, else through DSMEM
  const int64_t split_bytes = static_cast<int64_t>(n_tiles) * m_tiles * splits * un * UM * 4;
  float* split_ws = nullptr;
  if (splits > 1 && workspace != nullptr && workspace_bytes >= split_bytes &&
      (reinterpret_cast<uintptr_t>(workspace) & 15u) == 0)
    split_ws = static_cast<float*>(workspace);

  CUtensorMap mw, mx;
  if (int rc = make_map(&mw, w, N, K, UM, fp8)) return rc;
  if (int rc = make_map(&mx, x, M, K, un, fp8)) return rc;
  GemmEpilogue ep{static_cast<__nv_bfloat16*>(y), x_scales, w_scales, row_mask, row_map, status, M, N, K,
                  splits > 1 ? 1 : 0, split_ws};
  dim3 grid(plan.grid_x, m_tiles, splits);
  int rc = 0;
#define LAUNCH_UN(U, R)                                                                 \
  rc = fp8 ? launch_tile<U, true, R>(mw, mx, ep, grid, stream) : launch_tile<U, false, R>(mw, mx, ep, grid, stream)
#define LAUNCH_DUAL(U)                                                                       \
  rc = fp8 ? launch_tile<U, true, 192, 2>(mw, mx, ep, grid, stream) : launch_tile<U, false, 192, 2>(mw, mx, ep, grid, stream)
  if (dual) { if (un == 128) LAUNCH_DUAL(128); else LAUNCH_DUAL(256); }
  else if (un == 32) { if (half_ring) LAUNCH_UN(32, 96); else LAUNCH_UN(32, 192); }
  else if (un == 64) { if (half_ring) LAUNCH_UN(64, 96); else LAUNCH_UN(64, 192); }
  else if (un == 128) { if (half_ring) LAUNCH_UN(128, 96); else LAUNCH_UN(128, 192); }
  else LAUNCH_UN(256, 192);
#undef LAUNCH_UN
#undef LAUNCH_DUAL
  if (rc) return rc;
  return check_launch("gemm_tcgen05");
}

}  // namespace cgym

extern "C" int cgym_test_gemm_wait(unsigned long long limit_ns, int drop_loads) {
  using namespace cgym;
  const unsigned long long limit = limit_ns == 0 ? WAIT_LIMIT_NS : limit_ns;
  const int drop = drop_loads ? 1 : 0;
  cudaError_t rc = cudaMemcpyToSymbol(g_wait_limit_ns, &limit, sizeof(limit));
  if (rc == cudaSuccess) rc = cudaMemcpyToSymbol(g_drop_loads, &drop, sizeof(drop));
  CGYM_REQUIRE(rc == cudaSuccess, "test_gemm_wait: %s", cudaGetErrorString(rc));
  return 0;
}

extern "C" int cgym_gemm_plan(int M, int N, int K, int fp8, int impl, int in_dependent_chain, int* plan6) {
  using namespace cgym;
  CGYM_REQUIRE(M > 0 && N > 0 && K > 0 && plan6 != nullptr, "gemm_plan: bad arguments");
  CGYM_REQUIRE(impl == 0 || (impl >= 2 && impl <= 5), "gemm_plan: impl must be 0 or 2..5 (the tcgen05 forms)");
  const int force = impl == 3 ? 4 : (impl == 4 ? -2 : (impl == 5 ? -3 : 0));
  CGYM_REQUIRE(force == 0 || force == 4 || N % (2 * UM) == 0, "gemm_plan: pairs need a feature count that is a multiple of 256");
  const GemmPlan plan = plan_gemm(M, N, K, fp8 != 0, force, in_dependent_chain != 0);
  plan6[0] = plan.kind, plan6[1] = plan.un, plan6[2] = plan.fm;
  plan6[3] = plan.splits, plan6[4] = plan.grid_x, plan6[5] = plan.grid_y;
  return 0;
}
