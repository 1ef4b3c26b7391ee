// Lossless 12-bit stream of bf16 weights for single-request decode (B = 1 is pure weight streaming).
//
// A bf16 value is sign (1) | exponent (8) | mantissa (7). Trained weights use a narrow band of
// exponents, so the stream stores sign + mantissa as one byte and the exponent as a 4-bit code:
// code c in 1..15 stands for exponent base + c - 1; code 0 says "read the original bf16 value"
// (zeros, denormals, large magnitudes, infinities, NaN payloads stay exact that way). A GEMV over the
// stream reads 1.5 bytes per weight instead of 2. This is the format of the reference's
// PackedBF16Weight (src/climbing_gym/inference/lfm25_bf16.py:1-58), decoded by a kernel written for
// 16-byte accesses: a lane takes 16 consecutive weights of a row per step (one 16-byte load of sign /
// mantissa bytes, one 8-byte load of exponent codes, two 16-byte loads of x from shared memory), a warp
// owns an output row, and the weights are never staged in shared memory (each is used once).
#include "common.cuh"

namespace cgym {

constexpr int STREAM_THREADS = 256;

__global__ void bf16_pack_kernel(uint8_t* __restrict__ mantissa, uint8_t* __restrict__ exponent,
                                 const uint16_t* __restrict__ w, int64_t pairs, int base) {
  const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= pairs) return;
  const uint32_t both = reinterpret_cast<const uint32_t*>(w)[i];
  const uint32_t w0 = both & 0xFFFFu, w1 = both >> 16;
  const int e0 = (w0 >> 7) & 255, e1 = (w1 >> 7) & 255;
  const int c0 = (e0 >= base && e0 < base + 15) ? e0 - base + 1 : 0;
  const int c1 = (e1 >= base && e1 < base + 15) ? e1 - base + 1 : 0;
  const uint16_t bytes = static_cast<uint16_t>(((w0 & 127u) | ((w0 >> 8) & 128u)) |
                                               (((w1 & 127u) | ((w1 >> 8) & 128u)) << 8));
  reinterpret_cast<uint16_t*>(mantissa)[i] = bytes;
  exponent[i] = static_cast<uint8_t>(c0 | (c1 << 4));
}

__device__ __forceinline__ uint16_t stream_decode(uint32_t m, uint32_t code, uint16_t original, int base) {
  if (code == 0) return original;
  return static_cast<uint16_t>((m & 127u) | ((m & 128u) << 8) | (static_cast<uint32_t>(code + base - 1) << 7));
}

__global__ void bf16_unpack_kernel(uint16_t* __restrict__ out, const uint16_t* __restrict__ w,
                                   const uint8_t* __restrict__ mantissa, const uint8_t* __restrict__ exponent,
                                   int64_t numel, int base) {
  const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= numel) return;
  const uint32_t code = (exponent[i >> 1] >> ((i & 1) * 4)) & 15u;
  out[i] = stream_decode(mantissa[i], code, code == 0 ? w[i] : 0, base);
}

// y[n] = sum_k w[n][k] * x[k], one warp per output row, fp32 accumulation, bf16 result.
__global__ void __launch_bounds__(STREAM_THREADS)
bf16_stream_gemv_kernel(__nv_bfloat16* __restrict__ y, const __nv_bfloat16* __restrict__ x,
                        const uint16_t* __restrict__ w, const uint8_t* __restrict__ mantissa,
                        const uint8_t* __restrict__ exponent, const uint8_t* __restrict__ row_mask, int N, int K,
                        int base) {
  extern __shared__ __align__(16) uint8_t stream_smem[];
  __nv_bfloat16* xs = reinterpret_cast<__nv_bfloat16*>(stream_smem);
  pdl_trigger();
  pdl_wait();
  if (row_mask != nullptr && !row_mask[0]) return;  // the (single) row is masked: y keeps its contents
  for (int i = threadIdx.x; i < K; i += STREAM_THREADS) xs[i] = x[i];
  __syncthreads();
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int row = blockIdx.x * (STREAM_THREADS / 32) + warp;
  if (row >= N) return;
  const uint8_t* m_row = mantissa + static_cast<int64_t>(row) * K;
  const uint8_t* e_row = exponent + static_cast<int64_t>(row) * (K / 2);
  const uint16_t* w_row = w + static_cast<int64_t>(row) * K;
  float acc = 0.0f;
  // 16 weights per lane and step; rows of the byte streams start on 16-byte boundaries only when K is a
  // multiple of 16, other widths go through the scalar loop below
  const int groups = (K % 16 == 0) ? K / 16 : 0;
  for (int g = lane; g < groups; g += 32) {
    const uint4 mm = *reinterpret_cast<const uint4*>(m_row + g * 16);
    const uint2 ee = *reinterpret_cast<const uint2*>(e_row + g * 8);
    const uint32_t m_words[4] = {mm.x, mm.y, mm.z, mm.w};
    const uint32_t e_words[2] = {ee.x, ee.y};
    const __nv_bfloat16* xg = xs + g * 16;
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      const uint32_t m = (m_words[j >> 2] >> ((j & 3) * 8)) & 255u;
      const uint32_t code = (e_words[j >> 3] >> ((j & 7) * 4)) & 15u;
      const uint16_t bits = stream_decode(m, code, code == 0 ? w_row[g * 16 + j] : 0, base);
      acc = fmaf(__bfloat162float(__ushort_as_bfloat16(bits)), __bfloat162float(xg[j]), acc);
    }
  }
  for (int k = groups * 16 + lane; k < K; k += 32) {
    const uint32_t code = (e_row[k >> 1] >> ((k & 1) * 4)) & 15u;
    const uint16_t bits = stream_decode(m_row[k], code, code == 0 ? w_row[k] : 0, base);
    acc = fmaf(__bfloat162float(__ushort_as_bfloat16(bits)), __bfloat162float(xs[k]), acc);
  }
  acc = warp_sum(acc);
  if (lane == 0) y[row] = __float2bfloat16_rn(acc);
}

}  // namespace cgym

using namespace cgym;

extern "C" int cgym_bf16_stream_pack(uint8_t* mantissa, uint8_t* exponent, const void* w, int64_t numel, int base,
                                     cgym_stream_t stream) {
  CGYM_REQUIRE(mantissa && exponent && w && numel >= 0 && numel % 2 == 0, "bf16_stream_pack: an even number of weights");
  CGYM_REQUIRE(base >= 0 && base <= 240, "bf16_stream_pack: exponent base out of range");
  if (numel == 0) return 0;
  const int64_t pairs = numel / 2;
  bf16_pack_kernel<<<static_cast<unsigned>((pairs + 255) / 256), 256, 0, as_stream(stream)>>>(
      mantissa, exponent, static_cast<const uint16_t*>(w), pairs, base);
  return check_launch("bf16_stream_pack");
}

extern "C" int cgym_bf16_stream_unpack(void* out, const void* w, const uint8_t* mantissa, const uint8_t* exponent,
                                       int64_t numel, int base, cgym_stream_t stream) {
  CGYM_REQUIRE(out && w && mantissa && exponent && numel >= 0, "bf16_stream_unpack: bad arguments");
  if (numel == 0) return 0;
  bf16_unpack_kernel<<<static_cast<unsigned>((numel + 255) / 256), 256, 0, as_stream(stream)>>>(
      static_cast<uint16_t*>(out), static_cast<const uint16_t*>(w), mantissa, exponent, numel, base);
  return check_launch("bf16_stream_unpack");
}

extern "C" int cgym_bf16_stream_gemv(void* y, const void* x, const void* w, const uint8_t* mantissa,
                                     const uint8_t* exponent, const uint8_t* row_mask, int N, int K, int base,
                                     cgym_stream_t stream) {
  CGYM_REQUIRE(y && x && w && mantissa && exponent && N > 0 && K > 0, "bf16_stream_gemv: bad arguments");
  CGYM_REQUIRE(K % 2 == 0 && K <= 16384, "bf16_stream_gemv: even input width up to 16384");
  CGYM_REQUIRE((reinterpret_cast<uintptr_t>(mantissa) & 15u) == 0 && (reinterpret_cast<uintptr_t>(exponent) & 7u) == 0,
               "bf16_stream_gemv: the streams must be 16-byte aligned");
  const int smem = K * static_cast<int>(sizeof(__nv_bfloat16));
  const dim3 grid((N + STREAM_THREADS / 32 - 1) / (STREAM_THREADS / 32));
  const cudaError_t rc = launch_dependent(bf16_stream_gemv_kernel, grid, dim3(STREAM_THREADS), smem, as_stream(stream),
                                          static_cast<__nv_bfloat16*>(y), static_cast<const __nv_bfloat16*>(x),
                                          static_cast<const uint16_t*>(w), mantissa, exponent, row_mask, N, K, base);
  CGYM_REQUIRE(rc == cudaSuccess, "bf16_stream_gemv: launch failed: %s", cudaGetErrorString(rc));
  return check_launch("bf16_stream_gemv");
}
