// Shared device/host helpers for the cgym_b200 kernels (sm_100a only).
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp8.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <cstdarg>
#include <cstdio>
#include <mutex>

#include "../../include/cgym_b200.h"

namespace cgym {

// ---- error reporting -------------------------------------------------------------------
// One message buffer per host thread: the adapter calls from executor threads, and an error
// string must not be overwritten by another thread between the failing call and the read.
char* error_buffer();
int fail(const char* fmt, ...);
int check_launch(const char* what, int kernels = 1);

#define CGYM_REQUIRE(cond, ...)             \
  do {                                      \
    if (!(cond)) return ::cgym::fail(__VA_ARGS__); \
  } while (0)

inline cudaStream_t as_stream(cgym_stream_t s) { return reinterpret_cast<cudaStream_t>(s); }

// ---- programmatic dependent launch -------------------------------------------------------
// The decode step is ~150 short kernels; with programmatic stream serialization a kernel may be
// scheduled while its predecessor is still running, so its launch latency, prologue (barrier
// init, TMEM allocation, descriptor fetch) and - for the GEMMs - the first weight tiles overlap
// the predecessor's tail. Contract: a kernel launched through launch_dependent() calls pdl_wait()
// before it touches memory a predecessor may write or still read, and pdl_trigger() once it no
// longer minds the next kernel being scheduled. Every thread of every such kernel calls pdl_wait()
// (so a grid never completes before its predecessor: the wait is transitive along the chain), and
// kernels trigger BEFORE they wait, which lets the kernels several positions ahead become
// resident - the GEMMs among them stream their first weight tiles - while the chain catches up.
// Both are no-ops for ordinary launches.
extern thread_local int g_pdl_enabled;  // per host thread: set by cgym_set_pdl(), read at launch time
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }
// A kernel that does work BEFORE pdl_wait() must reach its predecessor's output only through pointers
// passed through pdl_fresh() after the wait. Inputs are declared `const T* __restrict__`, which tells
// the compiler that nothing changes that memory during the kernel - so it may hoist such loads above
// the wait to batch them with the early ones, and read what the predecessor has not written yet. The
// empty volatile asm makes the pointer's value a product of a statement that follows the wait.
template <typename P>
__device__ __forceinline__ P* pdl_fresh(P* p) {
  asm volatile("" : "+l"(p)::"memory");
  return p;
}

template <typename... Params, typename... Args>
inline cudaError_t launch_dependent(void (*kernel)(Params...), dim3 grid, dim3 block, size_t smem,
                                    cudaStream_t stream, Args&&... args) {
  cudaLaunchConfig_t config = {};
  config.gridDim = grid;
  config.blockDim = block;
  config.dynamicSmemBytes = smem;
  config.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  config.attrs = attr;
  config.numAttrs = g_pdl_enabled ? 1 : 0;
  return cudaLaunchKernelEx(&config, kernel, static_cast<Params>(args)...);
}

// ---- opt-in dynamic shared memory ------------------------------------------------------------
// cudaFuncAttributeMaxDynamicSharedMemorySize belongs to a (kernel, device) pair: a process that drives
// several GPUs must set it once on each. SmemReservation remembers, per device ordinal, the largest size set
// so far for one kernel (declare one `static SmemReservation` beside each kernel's launch); calls from
// several host threads are serialised. Ordinals beyond the table set the attribute on every call.
struct SmemReservation {
  static constexpr int MAX_DEVICES = 64;
  std::mutex mutex;
  int reserved[MAX_DEVICES] = {};
};

template <typename K>
inline int reserve_dynamic_smem(K kernel, int bytes, SmemReservation& seen, const char* what) {
  int device = -1;
  cudaError_t rc = cudaGetDevice(&device);
  if (rc != cudaSuccess) return fail("%s: cudaGetDevice failed: %s", what, cudaGetErrorString(rc));
  std::lock_guard<std::mutex> lock(seen.mutex);
  const bool tracked = device >= 0 && device < SmemReservation::MAX_DEVICES;
  if (tracked && seen.reserved[device] >= bytes) return 0;
  rc = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  if (rc != cudaSuccess)
    return fail("%s: cannot reserve %d bytes of shared memory on device %d: %s", what, bytes, device,
                cudaGetErrorString(rc));
  if (tracked) seen.reserved[device] = bytes;
  return 0;
}

// ---- element types ---------------------------------------------------------------------
// load / store convert through fp32; store rounds to nearest even for bf16 (cvt.rn), which is
// the cast the reference applies at every rounding point.
template <typename T>
struct Elem;
template <>
struct Elem<float> {
  static __device__ __forceinline__ float load(const float* p) { return *p; }
  static __device__ __forceinline__ void store(float* p, float v) { *p = v; }
  static __device__ __forceinline__ float round(float v) { return v; }
};
template <>
struct Elem<__nv_bfloat16> {
  static __device__ __forceinline__ float load(const __nv_bfloat16* p) { return __bfloat162float(*p); }
  static __device__ __forceinline__ void store(__nv_bfloat16* p, float v) { *p = __float2bfloat16_rn(v); }
  static __device__ __forceinline__ float round(float v) { return __bfloat162float(__float2bfloat16_rn(v)); }
};

// fp32 -> e4m3 code, round-to-nearest-even, saturating to +-448 (cvt.rn.satfinite.e4m3x2.f32).
__device__ __forceinline__ uint8_t to_e4m3(float v) {
  return static_cast<uint8_t>(__nv_cvt_float_to_fp8(v, __NV_SATFINITE, __NV_E4M3));
}
__device__ __forceinline__ float from_e4m3(uint8_t code) {
  __half_raw h = __nv_cvt_fp8_to_halfraw(code, __NV_E4M3);
  return __half2float(*reinterpret_cast<__half*>(&h));
}

// ---- reductions ------------------------------------------------------------------------
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}
// Block-wide reductions over <= 1024 threads; `scratch` holds 32 floats. All threads get the result.
__device__ __forceinline__ float block_sum(float v, float* scratch) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nwarps = (blockDim.x + 31) >> 5;
  v = warp_sum(v);
  __syncthreads();
  if (lane == 0) scratch[warp] = v;
  __syncthreads();
  float r = (lane < nwarps) ? scratch[lane] : 0.0f;
  return warp_sum(r);
}
__device__ __forceinline__ float block_max(float v, float* scratch) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nwarps = (blockDim.x + 31) >> 5;
  v = warp_max(v);
  __syncthreads();
  if (lane == 0) scratch[warp] = v;
  __syncthreads();
  float r = (lane < nwarps) ? scratch[lane] : -INFINITY;
  return warp_max(r);
}

// ---- paged KV addressing ---------------------------------------------------------------
// pool[layer][page][kv_head] is one contiguous block of 2 * page_size * head_dim elements:
//   K part   [token][dim]   (row = token, head_dim elements)
//   V^T part [dim][token]   (row = dim,   page_size elements)
// so that both are "contraction-contiguous" B operands for the tensor-core attention kernels and a
// (page, head) block moves with ONE bulk copy. Inside each row the 16-byte chunks are XOR-swizzled
// by the row index, already in global memory: the block lands in shared memory through a linear
// bulk copy and fragment loads of 8 consecutive rows at one column hit 8 different bank groups.
__host__ __device__ __forceinline__ int kv_swizzle(int row, int chunk, int chunks_per_row) {
  if (chunks_per_row >= 8) return chunk ^ (row & 7);
  // fewer than 8 chunks per row: 8 / cpr consecutive rows share a 128-byte line
  const int rows_per_line = 8 / chunks_per_row;  // 2 or 4 (or 8 when cpr == 1: nothing to swizzle)
  return chunk ^ ((row / rows_per_line) & (chunks_per_row - 1));
}
__host__ __device__ __forceinline__ int64_t kv_block_offset(const cgym_kv_layout& kv, int layer, int page, int head) {
  return ((static_cast<int64_t>(layer) * kv.n_pages + page) * kv.n_kv_heads + head) *
         (2ll * kv.page_size * kv.head_dim);
}
// element index inside a row of `row_elems` elements of `elem_bytes` bytes each
__host__ __device__ __forceinline__ int kv_row_index(int row, int col, int row_elems, int elem_bytes) {
  const int per_chunk = 16 / elem_bytes;
  const int chunk = kv_swizzle(row, col / per_chunk, row_elems / per_chunk);
  return row * row_elems + chunk * per_chunk + (col % per_chunk);
}
__host__ __device__ __forceinline__ int64_t kv_k_offset(const cgym_kv_layout& kv, int layer, int page, int head,
                                                        int token, int d, int elem_bytes) {
  return kv_block_offset(kv, layer, page, head) + kv_row_index(token, d, kv.head_dim, elem_bytes);
}
__host__ __device__ __forceinline__ int64_t kv_v_offset(const cgym_kv_layout& kv, int layer, int page, int head,
                                                        int token, int d, int elem_bytes) {
  return kv_block_offset(kv, layer, page, head) + kv.page_size * kv.head_dim +
         kv_row_index(d, token, kv.page_size, elem_bytes);
}
// scales[layer][page][kv_head][k|v][token]
__host__ __device__ __forceinline__ int64_t kv_scale_offset(const cgym_kv_layout& kv, int layer, int page,
                                                            int which, int head, int token) {
  int64_t idx = (((static_cast<int64_t>(layer) * kv.n_pages + page) * kv.n_kv_heads + head) * 2 + which);
  return idx * kv.page_size + token;
}

}  // namespace cgym
