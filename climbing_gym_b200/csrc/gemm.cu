// Entry points of the projection GEMMs: pick the tcgen05/TMEM kernel when the operands allow it and
// the CUDA-core tile kernel otherwise (fp32 models, unaligned K).
#include "common.cuh"

namespace cgym {
int launch_gemm_simt(void* y, const void* x, const void* w, const float* x_scales, const float* w_scales,
                     const uint8_t* row_mask, const int32_t* row_map, int M, int N, int K, int in_dtype,
                     cudaStream_t stream);
int launch_gemm_tcgen05(void* y, const void* x, const void* w, const float* x_scales, const float* w_scales,
                        const uint8_t* row_mask, const int32_t* row_map, int M, int N, int K, bool fp8,
                        void* workspace, int64_t workspace_bytes, int32_t* status, int force_splits,
                        cudaStream_t stream);
bool gemm_tcgen05_supports(int M, int N, int K, bool fp8, const void* x, const void* w);
}  // namespace cgym

using namespace cgym;

extern "C" int cgym_gemm_scatter(void* y, const void* x, const void* w, const uint8_t* row_mask,
                                 const int32_t* row_map, int M, int N, int K, int dtype, int impl, void* workspace,
                                 int64_t workspace_bytes, int32_t* status, cgym_stream_t stream) {
  CGYM_REQUIRE(M >= 0 && N > 0 && K > 0, "gemm: bad shape (%d, %d, %d)", M, N, K);
  CGYM_REQUIRE(y && x && w, "gemm: null operand");
  CGYM_REQUIRE(impl >= 0 && impl <= 5, "gemm: impl must be 0 (auto), 1 (simt), 2 (tcgen05), 3 (forced split-K), 4 (CTA pairs) or 5 (persistent CTA pairs)");
  if (M == 0) return 0;
  if (impl == 0) impl = (dtype == CGYM_BF16 && gemm_tcgen05_supports(M, N, K, false, x, w)) ? 2 : 1;
  if (impl >= 2) {
    CGYM_REQUIRE(dtype == CGYM_BF16, "gemm(tcgen05): bf16 operands only");
    return launch_gemm_tcgen05(y, x, w, nullptr, nullptr, row_mask, row_map, M, N, K, false, workspace,
                               workspace_bytes, status, impl == 3 ? 4 : (impl == 4 ? -2 : (impl == 5 ? -3 : 0)), as_stream(stream));
  }
  return launch_gemm_simt(y, x, w, nullptr, nullptr, row_mask, row_map, M, N, K, dtype, as_stream(stream));
}

extern "C" int cgym_gemm(void* y, const void* x, const void* w, const uint8_t* row_mask, int M, int N, int K,
                         int dtype, int impl, void* workspace, int64_t workspace_bytes, int32_t* status,
                         cgym_stream_t stream) {
  return cgym_gemm_scatter(y, x, w, row_mask, nullptr, M, N, K, dtype, impl, workspace, workspace_bytes, status,
                           stream);
}

extern "C" int cgym_gemm_fp8_scatter(void* y, const uint8_t* xq, const float* x_scales, const uint8_t* wq,
                                     const float* w_scales, const uint8_t* row_mask, const int32_t* row_map, int M,
                                     int N, int K, int impl, void* workspace, int64_t workspace_bytes,
                                     int32_t* status, cgym_stream_t stream) {
  CGYM_REQUIRE(M >= 0 && N > 0 && K > 0, "gemm_fp8: bad shape (%d, %d, %d)", M, N, K);
  CGYM_REQUIRE(y && xq && wq && x_scales && w_scales, "gemm_fp8: null operand");
  CGYM_REQUIRE(impl >= 0 && impl <= 5, "gemm_fp8: impl must be 0..5");
  if (M == 0) return 0;
  if (impl == 0) impl = gemm_tcgen05_supports(M, N, K, true, xq, wq) ? 2 : 1;
  if (impl >= 2)
    return launch_gemm_tcgen05(y, xq, wq, x_scales, w_scales, row_mask, row_map, M, N, K, true, workspace,
                               workspace_bytes, status, impl == 3 ? 4 : (impl == 4 ? -2 : (impl == 5 ? -3 : 0)), as_stream(stream));
  return launch_gemm_simt(y, xq, wq, x_scales, w_scales, row_mask, row_map, M, N, K, CGYM_E4M3, as_stream(stream));
}

extern "C" int cgym_gemm_fp8(void* y, const uint8_t* xq, const float* x_scales, const uint8_t* wq,
                             const float* w_scales, const uint8_t* row_mask, int M, int N, int K, int impl,
                             void* workspace, int64_t workspace_bytes, int32_t* status, cgym_stream_t stream) {
  return cgym_gemm_fp8_scatter(y, xq, x_scales, wq, w_scales, row_mask, nullptr, M, N, K, impl, workspace,
                               workspace_bytes, status, stream);
}
