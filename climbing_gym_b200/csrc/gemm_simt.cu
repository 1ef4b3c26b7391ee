// CUDA-core tile GEMM: y[M,N] = x[M,K] . w[N,K]^T with fp32 accumulation.
//
// This is the any-shape, any-dtype (fp32 / bf16 / e4m3 x e4m3 with row and channel scales) kernel:
// it serves fp32 models (the CPU-runnable parity configuration), shapes the tensor-core kernel does
// not take (K not a multiple of 64, tiny N) and is the cross-check for the tcgen05 kernel in the
// GPU tests. 64x64 output tile, 16-wide K slices staged through shared memory, 4x4 micro-tile per
// thread. Accumulation runs over K in ascending order inside one thread, so results are
// deterministic and independent of the grid.
#include "common.cuh"

namespace cgym {

constexpr int ST_BM = 64, ST_BN = 64, ST_BK = 16;

template <typename T>
__device__ __forceinline__ float gemm_load(const T* p) { return Elem<T>::load(p); }
template <>
__device__ __forceinline__ float gemm_load<uint8_t>(const uint8_t* p) { return from_e4m3(*p); }

// TIN: operand element type (float, bf16, uint8 = e4m3); TOUT: output type (float or bf16)
template <typename TIN, typename TOUT>
__global__ void __launch_bounds__(256)
gemm_simt_kernel(TOUT* __restrict__ y, const TIN* __restrict__ x, const TIN* __restrict__ w,
                 const float* __restrict__ x_scales, const float* __restrict__ w_scales,
                 const uint8_t* __restrict__ row_mask, const int32_t* __restrict__ row_map, int M, int N, int K) {
  __shared__ float xs[ST_BK][ST_BM + 1];
  __shared__ float ws[ST_BK][ST_BN + 1];
  const int tx = threadIdx.x % 16, ty = threadIdx.x / 16;
  const int m0 = blockIdx.y * ST_BM, n0 = blockIdx.x * ST_BN;
  float acc[4][4] = {};
  for (int k0 = 0; k0 < K; k0 += ST_BK) {
    for (int i = threadIdx.x; i < ST_BM * ST_BK; i += 256) {
      const int r = i / ST_BK, c = i % ST_BK;
      const int gm = m0 + r, gk = k0 + c;
      xs[c][r] = (gm < M && gk < K) ? gemm_load<TIN>(x + static_cast<int64_t>(gm) * K + gk) : 0.0f;
      const int gn = n0 + r;
      ws[c][r] = (gn < N && gk < K) ? gemm_load<TIN>(w + static_cast<int64_t>(gn) * K + gk) : 0.0f;
    }
    __syncthreads();
#pragma unroll
    for (int k = 0; k < ST_BK; ++k) {
      float a[4], b[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) { a[i] = xs[k][ty * 4 + i]; b[i] = ws[k][tx * 4 + i]; }
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(a[i], b[j], acc[i][j]);
    }
    __syncthreads();
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int gm = m0 + ty * 4 + i;
    if (gm >= M || (row_mask != nullptr && !row_mask[gm])) continue;
    const int out_row = row_map != nullptr ? row_map[gm] : gm;  // scattered output rows; negative: not written
    if (out_row < 0) continue;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int gn = n0 + tx * 4 + j;
      if (gn >= N) continue;
      float v = acc[i][j];
      if (x_scales != nullptr) v = __fmul_rn(__fmul_rn(v, x_scales[gm]), w_scales[gn]);
      Elem<TOUT>::store(y + static_cast<int64_t>(out_row) * N + gn, v);
    }
  }
}

int launch_gemm_simt(void* y, const void* x, const void* w, const float* x_scales, const float* w_scales,
                     const uint8_t* row_mask, const int32_t* row_map, int M, int N, int K, int in_dtype,
                     cudaStream_t stream) {
  dim3 grid((N + ST_BN - 1) / ST_BN, (M + ST_BM - 1) / ST_BM);
  if (in_dtype == CGYM_F32)
    gemm_simt_kernel<float, float><<<grid, 256, 0, stream>>>(static_cast<float*>(y), static_cast<const float*>(x),
                                                             static_cast<const float*>(w), nullptr, nullptr,
                                                             row_mask, row_map, M, N, K);
  else if (in_dtype == CGYM_BF16)
    gemm_simt_kernel<__nv_bfloat16, __nv_bfloat16><<<grid, 256, 0, stream>>>(
        static_cast<__nv_bfloat16*>(y), static_cast<const __nv_bfloat16*>(x), static_cast<const __nv_bfloat16*>(w),
        nullptr, nullptr, row_mask, row_map, M, N, K);
  else if (in_dtype == CGYM_E4M3)
    gemm_simt_kernel<uint8_t, __nv_bfloat16><<<grid, 256, 0, stream>>>(
        static_cast<__nv_bfloat16*>(y), static_cast<const uint8_t*>(x), static_cast<const uint8_t*>(w), x_scales,
        w_scales, row_mask, row_map, M, N, K);
  else
    return fail("gemm: unsupported dtype %d", in_dtype);
  return check_launch("gemm_simt");
}

}  // namespace cgym
