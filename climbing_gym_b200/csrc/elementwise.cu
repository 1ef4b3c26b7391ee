// HBM-bound row kernels of the LFM2.5 decode / prefill step: embedding gather, RMSNorm
// (+residual, +e4m3 quantisation), SwiGLU (+quantisation), row quantisation, gated
// short-convolution state update (decode) and packed causal conv (prefill), QK-norm + RoPE +
// paged KV append, and target log-prob gathering for completion scoring.
//
// Every kernel is one pass over its rows: reads each input once with 16-byte-friendly
// coalesced accesses, keeps the row in registers/shared memory, and applies the model-dtype
// rounding at the points listed in include/cgym_b200.h.
#include "common.cuh"

namespace cgym {

// ------------------------------------------------------------------------------------------
// embedding
// ------------------------------------------------------------------------------------------
template <typename T>
__global__ void embedding_kernel(T* __restrict__ out, const T* __restrict__ table,
                                 const int64_t* __restrict__ tokens, int hidden, int vocab) {
  pdl_trigger();
  pdl_wait();
  const int row = blockIdx.x;
  int64_t tok = tokens[row];
  if (tok < 0 || tok >= vocab) tok = 0;  // padding rows carry arbitrary ids; never index outside the table
  const T* src = table + tok * hidden;
  T* dst = out + static_cast<int64_t>(row) * hidden;
  const size_t row_bytes = static_cast<size_t>(hidden) * sizeof(T);
  if (row_bytes % 16 == 0 && ((reinterpret_cast<uintptr_t>(table) | reinterpret_cast<uintptr_t>(out)) & 15u) == 0) {
    // 16-byte copies: a 4 KB row is one load per thread, i.e. one memory round trip
    const uint4* src16 = reinterpret_cast<const uint4*>(src);
    uint4* dst16 = reinterpret_cast<uint4*>(dst);
    for (int i = threadIdx.x; i < static_cast<int>(row_bytes / 16); i += blockDim.x) dst16[i] = __ldg(src16 + i);
    return;
  }
  for (int i = threadIdx.x; i < hidden; i += blockDim.x) dst[i] = src[i];
}

// ------------------------------------------------------------------------------------------
// RMSNorm (+ residual) (+ e4m3 row quantisation)
// ------------------------------------------------------------------------------------------
template <typename T, bool QUANT>
__global__ void rmsnorm_kernel(T* __restrict__ y, uint8_t* __restrict__ q, float* __restrict__ scales,
                               T* __restrict__ sum_out, const T* __restrict__ x,
                               const T* __restrict__ residual, const T* __restrict__ w, int hidden,
                               float eps) {
  extern __shared__ float row_buf[];  // hidden floats
  __shared__ float scratch[32];
  pdl_trigger();
  pdl_wait();
  const int64_t base = static_cast<int64_t>(blockIdx.x) * hidden;
  float ss = 0.0f;
  for (int i = threadIdx.x; i < hidden; i += blockDim.x) {
    float v = Elem<T>::load(x + base + i);
    if (residual != nullptr) {
      v = Elem<T>::round(__fadd_rn(v, Elem<T>::load(residual + base + i)));
      Elem<T>::store(sum_out + base + i, v);
    }
    row_buf[i] = v;
    ss = fmaf(v, v, ss);
  }
  const float total = block_sum(ss, scratch);
  const float inv = rsqrtf(total / static_cast<float>(hidden) + eps);
  float amax = 0.0f;
  for (int i = threadIdx.x; i < hidden; i += blockDim.x) {
    const float n = Elem<T>::round(__fmul_rn(row_buf[i], inv));
    const float v = Elem<T>::round(__fmul_rn(n, Elem<T>::load(w + i)));
    if (QUANT) {
      row_buf[i] = v;
      amax = fmaxf(amax, fabsf(v));
    } else {
      Elem<T>::store(y + base + i, v);
    }
  }
  if (QUANT) {
    amax = block_max(amax, scratch);
    const float scale = fmaxf(amax / 448.0f, 1.0e-12f);
    for (int i = threadIdx.x; i < hidden; i += blockDim.x) {
      const float s = fminf(fmaxf(__fdiv_rn(row_buf[i], scale), -448.0f), 448.0f);
      q[base + i] = to_e4m3(s);
    }
    if (threadIdx.x == 0) scales[blockIdx.x] = scale;
  }
}

// bf16 fast path: a row lives in registers. Thread t owns the 16-byte chunks t, t + 256, ... (CHUNKS of
// them), all of whose loads are issued back to back, so a row costs one L2 round trip instead of one
// per element; the norm weights do not depend on the previous kernel and are fetched before the
// dependent-launch wait. Same rounding points as rmsnorm_kernel.
constexpr int RMS_THREADS = 256;

__device__ __forceinline__ void unpack8(const uint4& raw, float* out) {
  const __nv_bfloat162* p = reinterpret_cast<const __nv_bfloat162*>(&raw);
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const float2 f = __bfloat1622float2(p[j]);
    out[2 * j] = f.x;
    out[2 * j + 1] = f.y;
  }
}

__device__ __forceinline__ uint4 pack8(const float* v) {
  uint4 raw;
  __nv_bfloat162* p = reinterpret_cast<__nv_bfloat162*>(&raw);
#pragma unroll
  for (int j = 0; j < 4; ++j) p[j] = __floats2bfloat162_rn(v[2 * j], v[2 * j + 1]);
  return raw;
}

template <int CHUNKS, bool QUANT>
__global__ void __launch_bounds__(RMS_THREADS)
rmsnorm_rows_bf16_kernel(__nv_bfloat16* __restrict__ y, uint8_t* __restrict__ q, float* __restrict__ scales,
                         __nv_bfloat16* __restrict__ sum_out, const __nv_bfloat16* __restrict__ x,
                         const __nv_bfloat16* __restrict__ residual, const __nv_bfloat16* __restrict__ w,
                         int hidden, float eps) {
  __shared__ float scratch[32];
  const int n_chunks = hidden >> 3;
  uint4 w_raw[CHUNKS];
#pragma unroll
  for (int c = 0; c < CHUNKS; ++c) {
    const int chunk = threadIdx.x + c * RMS_THREADS;
    w_raw[c] = chunk < n_chunks ? __ldg(reinterpret_cast<const uint4*>(w) + chunk) : make_uint4(0, 0, 0, 0);
  }
  pdl_trigger();
  pdl_wait();
  x = pdl_fresh(x);
  residual = pdl_fresh(residual);
  const int64_t base = static_cast<int64_t>(blockIdx.x) * n_chunks;  // in 16-byte chunks
  uint4 x_raw[CHUNKS], r_raw[CHUNKS];
#pragma unroll
  for (int c = 0; c < CHUNKS; ++c) {
    const int chunk = threadIdx.x + c * RMS_THREADS;
    x_raw[c] = r_raw[c] = make_uint4(0, 0, 0, 0);
    if (chunk < n_chunks) {
      x_raw[c] = *(reinterpret_cast<const uint4*>(x) + base + chunk);
      if (residual != nullptr) r_raw[c] = *(reinterpret_cast<const uint4*>(residual) + base + chunk);
    }
  }
  float v[CHUNKS][8];
  float ss = 0.0f;
#pragma unroll
  for (int c = 0; c < CHUNKS; ++c) {
    const int chunk = threadIdx.x + c * RMS_THREADS;
    unpack8(x_raw[c], v[c]);
    if (residual != nullptr) {
      float r[8];
      unpack8(r_raw[c], r);
#pragma unroll
      for (int j = 0; j < 8; ++j) v[c][j] = Elem<__nv_bfloat16>::round(__fadd_rn(v[c][j], r[j]));
      if (chunk < n_chunks) *(reinterpret_cast<uint4*>(sum_out) + base + chunk) = pack8(v[c]);
    }
#pragma unroll
    for (int j = 0; j < 8; ++j) ss = fmaf(v[c][j], v[c][j], ss);
  }
  const float total = block_sum(ss, scratch);
  const float inv = rsqrtf(total / static_cast<float>(hidden) + eps);
  float amax = 0.0f;
#pragma unroll
  for (int c = 0; c < CHUNKS; ++c) {
    const int chunk = threadIdx.x + c * RMS_THREADS;
    float wv[8];
    unpack8(w_raw[c], wv);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const float n = Elem<__nv_bfloat16>::round(__fmul_rn(v[c][j], inv));
      v[c][j] = Elem<__nv_bfloat16>::round(__fmul_rn(n, wv[j]));
      amax = fmaxf(amax, fabsf(v[c][j]));
    }
    if (!QUANT && chunk < n_chunks) *(reinterpret_cast<uint4*>(y) + base + chunk) = pack8(v[c]);
  }
  if (QUANT) {
    amax = block_max(amax, scratch);
    const float scale = fmaxf(amax / 448.0f, 1.0e-12f);
#pragma unroll
    for (int c = 0; c < CHUNKS; ++c) {
      const int chunk = threadIdx.x + c * RMS_THREADS;
      if (chunk >= n_chunks) continue;
      uint2 codes;
      uint8_t* bytes = reinterpret_cast<uint8_t*>(&codes);
#pragma unroll
      for (int j = 0; j < 8; ++j) bytes[j] = to_e4m3(fminf(fmaxf(__fdiv_rn(v[c][j], scale), -448.0f), 448.0f));
      *(reinterpret_cast<uint2*>(q) + base + chunk) = codes;
    }
    if (threadIdx.x == 0) scales[blockIdx.x] = scale;
  }
}

// true when the register-resident kernel applies: bf16, rows of whole 16-byte chunks, 16-byte aligned
static bool rms_fast_path(int hidden, const void* a, const void* b, const void* c, const void* d, const void* e) {
  const uintptr_t bits = reinterpret_cast<uintptr_t>(a) | reinterpret_cast<uintptr_t>(b) | reinterpret_cast<uintptr_t>(c) |
                         reinterpret_cast<uintptr_t>(d) | reinterpret_cast<uintptr_t>(e);
  return hidden % 8 == 0 && hidden <= 8 * RMS_THREADS * 4 && (bits & 15u) == 0;
}

template <bool QUANT>
static void launch_rms_fast(__nv_bfloat16* y, uint8_t* q, float* scales, __nv_bfloat16* sum_out, const __nv_bfloat16* x,
                            const __nv_bfloat16* residual, const __nv_bfloat16* w, int rows, int hidden, float eps,
                            cudaStream_t stream) {
  const int chunks = (hidden / 8 + RMS_THREADS - 1) / RMS_THREADS;
  if (chunks <= 1)
    launch_dependent(rmsnorm_rows_bf16_kernel<1, QUANT>, dim3(rows), dim3(RMS_THREADS), 0, stream, y, q, scales, sum_out,
                     x, residual, w, hidden, eps);
  else if (chunks == 2)
    launch_dependent(rmsnorm_rows_bf16_kernel<2, QUANT>, dim3(rows), dim3(RMS_THREADS), 0, stream, y, q, scales, sum_out,
                     x, residual, w, hidden, eps);
  else
    launch_dependent(rmsnorm_rows_bf16_kernel<4, QUANT>, dim3(rows), dim3(RMS_THREADS), 0, stream, y, q, scales, sum_out,
                     x, residual, w, hidden, eps);
}

// ------------------------------------------------------------------------------------------
// SwiGLU (+ quantisation)
// ------------------------------------------------------------------------------------------
template <typename T>
__device__ __forceinline__ float swiglu_value(float gate, float up) {
  const float act = Elem<T>::round(__fdiv_rn(gate, __fadd_rn(1.0f, expf(-gate))));
  return Elem<T>::round(__fmul_rn(act, up));
}

template <typename T>
__global__ void swiglu_kernel(T* __restrict__ y, const T* __restrict__ gate_up, int ffn) {
  pdl_trigger();
  pdl_wait();
  const int64_t row = blockIdx.y;
  const int col = blockIdx.x * blockDim.x + threadIdx.x;
  if (col >= ffn) return;
  const float gate = Elem<T>::load(gate_up + row * 2 * ffn + col);
  const float up = Elem<T>::load(gate_up + row * 2 * ffn + ffn + col);
  Elem<T>::store(y + row * ffn + col, swiglu_value<T>(gate, up));
}

// bf16 fast path: eight columns per thread, 16-byte loads and stores (ffn a multiple of 8, 16-byte
// aligned rows)
__global__ void __launch_bounds__(256)
swiglu_rows_bf16_kernel(__nv_bfloat16* __restrict__ y, const __nv_bfloat16* __restrict__ gate_up, int ffn) {
  pdl_trigger();
  pdl_wait();
  const int64_t row = blockIdx.y;
  const int chunk = blockIdx.x * blockDim.x + threadIdx.x;  // 8 columns
  if (chunk * 8 >= ffn) return;
  const uint4 g_raw = *(reinterpret_cast<const uint4*>(gate_up + row * 2 * ffn) + chunk);
  const uint4 u_raw = *(reinterpret_cast<const uint4*>(gate_up + row * 2 * ffn + ffn) + chunk);
  float g[8], u[8];
  unpack8(g_raw, g);
  unpack8(u_raw, u);
#pragma unroll
  for (int j = 0; j < 8; ++j) g[j] = swiglu_value<__nv_bfloat16>(g[j], u[j]);
  *(reinterpret_cast<uint4*>(y + row * ffn) + chunk) = pack8(g);
}

// bf16 fast path of the fused SwiGLU + row quantisation: the row's activations stay in registers
// (CHUNKS groups of eight per thread, 16-byte loads of gate and up, 8-byte stores of the codes)
constexpr int SWIGLU_Q_THREADS = 512;

template <int CHUNKS>
__global__ void __launch_bounds__(SWIGLU_Q_THREADS)
swiglu_quant_rows_bf16_kernel(uint8_t* __restrict__ q, float* __restrict__ scales,
                              const __nv_bfloat16* __restrict__ gate_up, int ffn) {
  __shared__ float scratch[32];
  pdl_trigger();
  pdl_wait();
  const int64_t row = blockIdx.x;
  const int n_chunks = ffn >> 3;
  const uint4* gate = reinterpret_cast<const uint4*>(gate_up + row * 2 * ffn);
  const uint4* up = reinterpret_cast<const uint4*>(gate_up + row * 2 * ffn + ffn);
  uint4 g_raw[CHUNKS], u_raw[CHUNKS];
#pragma unroll
  for (int c = 0; c < CHUNKS; ++c) {
    const int chunk = threadIdx.x + c * SWIGLU_Q_THREADS;
    g_raw[c] = u_raw[c] = make_uint4(0, 0, 0, 0);
    if (chunk < n_chunks) {
      g_raw[c] = gate[chunk];
      u_raw[c] = up[chunk];
    }
  }
  float v[CHUNKS][8];
  float amax = 0.0f;
#pragma unroll
  for (int c = 0; c < CHUNKS; ++c) {
    float u[8];
    unpack8(g_raw[c], v[c]);
    unpack8(u_raw[c], u);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      v[c][j] = swiglu_value<__nv_bfloat16>(v[c][j], u[j]);  // swiglu(0, 0) = 0 for the padding chunks
      amax = fmaxf(amax, fabsf(v[c][j]));
    }
  }
  amax = block_max(amax, scratch);
  const float scale = fmaxf(amax / 448.0f, 1.0e-12f);
#pragma unroll
  for (int c = 0; c < CHUNKS; ++c) {
    const int chunk = threadIdx.x + c * SWIGLU_Q_THREADS;
    if (chunk >= n_chunks) continue;
    uint2 codes;
    uint8_t* bytes = reinterpret_cast<uint8_t*>(&codes);
#pragma unroll
    for (int j = 0; j < 8; ++j) bytes[j] = to_e4m3(fminf(fmaxf(__fdiv_rn(v[c][j], scale), -448.0f), 448.0f));
    *(reinterpret_cast<uint2*>(q + row * ffn) + chunk) = codes;
  }
  if (threadIdx.x == 0) scales[row] = scale;
}

template <typename T>
__global__ void swiglu_quant_kernel(uint8_t* __restrict__ q, float* __restrict__ scales,
                                    const T* __restrict__ gate_up, int ffn) {
  extern __shared__ float row_buf[];
  __shared__ float scratch[32];
  pdl_trigger();
  pdl_wait();
  const int64_t row = blockIdx.x;
  float amax = 0.0f;
  for (int i = threadIdx.x; i < ffn; i += blockDim.x) {
    const float v = swiglu_value<T>(Elem<T>::load(gate_up + row * 2 * ffn + i),
                                    Elem<T>::load(gate_up + row * 2 * ffn + ffn + i));
    row_buf[i] = v;
    amax = fmaxf(amax, fabsf(v));
  }
  amax = block_max(amax, scratch);
  const float scale = fmaxf(amax / 448.0f, 1.0e-12f);
  for (int i = threadIdx.x; i < ffn; i += blockDim.x)
    q[row * ffn + i] = to_e4m3(fminf(fmaxf(__fdiv_rn(row_buf[i], scale), -448.0f), 448.0f));
  if (threadIdx.x == 0) scales[row] = scale;
}

template <typename T>
__global__ void quantize_rows_kernel(uint8_t* __restrict__ q, float* __restrict__ scales,
                                     const T* __restrict__ x, int width) {
  __shared__ float scratch[32];
  const int64_t row = blockIdx.x;
  float amax = 0.0f;
  for (int i = threadIdx.x; i < width; i += blockDim.x) amax = fmaxf(amax, fabsf(Elem<T>::load(x + row * width + i)));
  amax = block_max(amax, scratch);
  const float scale = fmaxf(amax / 448.0f, 1.0e-12f);
  for (int i = threadIdx.x; i < width; i += blockDim.x)
    q[row * width + i] = to_e4m3(fminf(fmaxf(__fdiv_rn(Elem<T>::load(x + row * width + i), scale), -448.0f), 448.0f));
  if (threadIdx.x == 0) scales[row] = scale;
}

// ------------------------------------------------------------------------------------------
// gated short convolution, kernel size 3
// ------------------------------------------------------------------------------------------
// decode: state [n_slots][3][hidden], tap 2 is the newest
template <typename T>
__global__ void conv_update_kernel(T* __restrict__ y, T* __restrict__ state, const T* __restrict__ bcx,
                                   const T* __restrict__ conv_w, const uint8_t* __restrict__ active,
                                   const int32_t* __restrict__ slots, int hidden) {
  pdl_trigger();
  const int row = blockIdx.y;
  const int col = blockIdx.x * blockDim.x + threadIdx.x;
  // the taps, the filter and the row's slot do not depend on the kernel ahead: fetch them before the wait
  int slot = slots != nullptr ? slots[row] : row;
  if (slot < 0) slot = 0;
  T* st = state + static_cast<int64_t>(slot) * 3 * hidden;
  float s0 = 0.f, s1 = 0.f, w0 = 0.f, w1 = 0.f, w2 = 0.f;
  if (col < hidden) {
    s0 = Elem<T>::load(st + hidden + col), s1 = Elem<T>::load(st + 2 * hidden + col);
    w0 = Elem<T>::load(conv_w + col * 3), w1 = Elem<T>::load(conv_w + col * 3 + 1), w2 = Elem<T>::load(conv_w + col * 3 + 2);
  }
  pdl_wait();
  if (col >= hidden) return;
  const T* in = pdl_fresh(bcx) + static_cast<int64_t>(row) * 3 * hidden;
  const float b = Elem<T>::load(in + col), c = Elem<T>::load(in + hidden + col), x = Elem<T>::load(in + 2 * hidden + col);
  const float bx = Elem<T>::round(__fmul_rn(b, x));
  const float p0 = Elem<T>::round(__fmul_rn(s0, w0)), p1 = Elem<T>::round(__fmul_rn(s1, w1)), p2 = Elem<T>::round(__fmul_rn(bx, w2));
  const float conv = Elem<T>::round(__fadd_rn(__fadd_rn(p0, p1), p2));
  if (active == nullptr || active[row]) {
    Elem<T>::store(st + col, s0);
    Elem<T>::store(st + hidden + col, s1);
    Elem<T>::store(st + 2 * hidden + col, bx);
  }
  Elem<T>::store(y + static_cast<int64_t>(row) * hidden + col, Elem<T>::round(__fmul_rn(c, conv)));
}

__device__ __forceinline__ int find_sequence(const int32_t* cu, int n_seqs, int row) {
  int lo = 0, hi = n_seqs - 1;  // largest s with cu[s] <= row
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (cu[mid] <= row) lo = mid; else hi = mid - 1;
  }
  return lo;
}

// prefill: history value b*x at chunk-local time t (t < 0 reads the slot's carried taps)
template <typename T>
__device__ __forceinline__ float conv_history(const T* __restrict__ bcx, const T* __restrict__ st, int seq_begin,
                                              int t, bool carried, int hidden, int col) {
  if (t >= 0) {
    const T* in = bcx + static_cast<int64_t>(seq_begin + t) * 3 * hidden;
    return Elem<T>::round(__fmul_rn(Elem<T>::load(in + col), Elem<T>::load(in + 2 * hidden + col)));
  }
  return carried ? Elem<T>::load(st + (3 + t) * hidden + col) : 0.0f;  // t in [-3, -1] -> tap 3+t
}

template <typename T>
__global__ void conv_prefill_kernel(T* __restrict__ y, const T* __restrict__ state, const T* __restrict__ bcx,
                                    const T* __restrict__ conv_w, const int32_t* __restrict__ cu,
                                    const int32_t* __restrict__ seq_slots, const int32_t* __restrict__ seq_starts,
                                    int n_seqs, int hidden) {
  const int row = blockIdx.y;
  const int col = blockIdx.x * blockDim.x + threadIdx.x;
  if (col >= hidden) return;
  const int seq = find_sequence(cu, n_seqs, row);
  const int begin = cu[seq], t = row - begin;
  const bool carried = seq_starts[seq] > 0;
  const T* st = state + static_cast<int64_t>(seq_slots[seq]) * 3 * hidden;
  const float h0 = conv_history<T>(bcx, st, begin, t - 2, carried, hidden, col);
  const float h1 = conv_history<T>(bcx, st, begin, t - 1, carried, hidden, col);
  const float h2 = conv_history<T>(bcx, st, begin, t, carried, hidden, col);
  const float w0 = Elem<T>::load(conv_w + col * 3), w1 = Elem<T>::load(conv_w + col * 3 + 1), w2 = Elem<T>::load(conv_w + col * 3 + 2);
  // exact products, fp32 sum in tap order, one rounding
  const float conv = Elem<T>::round(__fadd_rn(__fadd_rn(__fmul_rn(h0, w0), __fmul_rn(h1, w1)), __fmul_rn(h2, w2)));
  const float c = Elem<T>::load(bcx + static_cast<int64_t>(row) * 3 * hidden + hidden + col);
  Elem<T>::store(y + static_cast<int64_t>(row) * hidden + col, Elem<T>::round(__fmul_rn(c, conv)));
}

// runs after conv_prefill_kernel on the same stream: the slot's taps become the last three
// history values of its chunk
template <typename T>
__global__ void conv_prefill_state_kernel(T* __restrict__ state, const T* __restrict__ bcx,
                                          const int32_t* __restrict__ cu, const int32_t* __restrict__ seq_slots,
                                          const int32_t* __restrict__ seq_starts, int hidden) {
  const int seq = blockIdx.y;
  const int col = blockIdx.x * blockDim.x + threadIdx.x;
  if (col >= hidden) return;
  const int begin = cu[seq], len = cu[seq + 1] - begin;
  const bool carried = seq_starts[seq] > 0;
  T* st = state + static_cast<int64_t>(seq_slots[seq]) * 3 * hidden;
  float taps[3];
#pragma unroll
  for (int j = 0; j < 3; ++j) taps[j] = conv_history<T>(bcx, st, begin, len - 3 + j, carried, hidden, col);
#pragma unroll
  for (int j = 0; j < 3; ++j) Elem<T>::store(st + j * hidden + col, taps[j]);
}

// ------------------------------------------------------------------------------------------
// QK-norm + RoPE + paged KV append
// ------------------------------------------------------------------------------------------
// grid (rows, Hq + Hkv), block = head_dim threads. K-head blocks also move the V head.
template <typename T, typename KV>
__global__ void qk_rope_append_kernel(T* __restrict__ q_out, T* __restrict__ k_new, T* __restrict__ v_new,
                                      const T* __restrict__ qkv, const T* __restrict__ q_w,
                                      const T* __restrict__ k_w, const float* __restrict__ rope_cos,
                                      const float* __restrict__ rope_sin, const int32_t* __restrict__ positions,
                                      const int32_t* __restrict__ slots, const uint8_t* __restrict__ active,
                                      cgym_kv_layout kv, int layer, int n_q_heads, float eps, int32_t* status) {
  __shared__ float buf[256];
  __shared__ float scratch[32];
  pdl_trigger();
  const int row = blockIdx.x, head = blockIdx.y, d = threadIdx.x, D = kv.head_dim, half = D >> 1;
  const int n_kv = kv.n_kv_heads;
  const int width = (n_q_heads + 2 * n_kv) * D;
  const bool is_q = head < n_q_heads;
  // Everything but qkv is settled before the kernel ahead of this one starts (positions, slots, active
  // and the block table date from the start of the step, the tables and weights are constants), so
  // the dependent position -> RoPE row -> page chain is walked before the dependent-launch wait.
  const int pos = positions[row];
  const float c = Elem<T>::round(rope_cos[static_cast<int64_t>(pos) * half + (d % half)]);
  const float s = Elem<T>::round(rope_sin[static_cast<int64_t>(pos) * half + (d % half)]);
  const float norm_w = Elem<T>::load((is_q ? q_w : k_w) + d);
  const bool writes_cache = !is_q && (active == nullptr || active[row]);
  const int slot = slots != nullptr ? slots[row] : row;
  int page = -1;
  if (writes_cache && slot >= 0) {
    const int block = pos / kv.page_size;
    page = block < kv.max_blocks ? kv.block_table[static_cast<int64_t>(slot) * kv.max_blocks + block] : -1;
  }
  pdl_wait();
  qkv = pdl_fresh(qkv);
  const float x = Elem<T>::load(qkv + static_cast<int64_t>(row) * width + head * D + d);
  const float ms = block_sum(x * x, scratch) / static_cast<float>(D);
  float n = Elem<T>::round(__fmul_rn(x, rsqrtf(ms + eps)));
  n = Elem<T>::round(__fmul_rn(n, norm_w));
  buf[d] = n;
  __syncthreads();
  const float other = buf[d < half ? d + half : d - half];
  const float left = Elem<T>::round(__fmul_rn(n, c)), right = Elem<T>::round(__fmul_rn(other, s));
  const float rot = Elem<T>::round(d < half ? __fsub_rn(left, right) : __fadd_rn(left, right));
  if (is_q) {
    Elem<T>::store(q_out + (static_cast<int64_t>(row) * n_q_heads + head) * D + d, rot);
    return;
  }
  const int kh = head - n_q_heads;
  const float v = Elem<T>::load(qkv + static_cast<int64_t>(row) * width + (n_q_heads + n_kv + kh) * D + d);
  if (k_new != nullptr) {
    Elem<T>::store(k_new + (static_cast<int64_t>(row) * n_kv + kh) * D + d, rot);
    Elem<T>::store(v_new + (static_cast<int64_t>(row) * n_kv + kh) * D + d, v);
  }
  if (!writes_cache || slot < 0) return;
  const int tok = pos % kv.page_size;
  if (page < 0 || page >= kv.n_pages) {  // uniform across the block
    if (d == 0) atomicOr(status, CGYM_STATUS_BAD_PAGE);
    return;
  }
  KV* pool = static_cast<KV*>(kv.kv_pool);
  const int64_t ko = kv_k_offset(kv, layer, page, kh, tok, d, static_cast<int>(sizeof(KV)));
  const int64_t vo = kv_v_offset(kv, layer, page, kh, tok, d, static_cast<int>(sizeof(KV)));
  if constexpr (sizeof(KV) == 1) {
    const float ak = block_max(fabsf(rot), scratch);
    const float av = block_max(fabsf(v), scratch);
    const float sk = fmaxf(ak / 448.0f, 1.0e-12f), sv = fmaxf(av / 448.0f, 1.0e-12f);
    reinterpret_cast<uint8_t*>(pool)[ko] = to_e4m3(__fdiv_rn(rot, sk));
    reinterpret_cast<uint8_t*>(pool)[vo] = to_e4m3(__fdiv_rn(v, sv));
    if (d == 0) {
      kv.kv_scales[kv_scale_offset(kv, layer, page, 0, kh, tok)] = sk;
      kv.kv_scales[kv_scale_offset(kv, layer, page, 1, kh, tok)] = sv;
    }
  } else {
    Elem<KV>::store(pool + ko, rot);
    Elem<KV>::store(pool + vo, v);
  }
}

// head_dim 64: one WARP per head (lane l holds dims l and l + 32, i.e. a RoPE pair), eight heads per
// CTA, reductions by shuffle only. Same arithmetic, in the same order, as the kernel above (the mean
// square is the sum of the two 32-dim halves, each reduced by the same butterfly).
template <typename T, typename KV>
__global__ void __launch_bounds__(256)
qk_rope_append_d64_kernel(T* __restrict__ q_out, T* __restrict__ k_new, T* __restrict__ v_new,
                          const T* __restrict__ qkv, const T* __restrict__ q_w, const T* __restrict__ k_w,
                          const float* __restrict__ rope_cos, const float* __restrict__ rope_sin,
                          const int32_t* __restrict__ positions, const int32_t* __restrict__ slots,
                          const uint8_t* __restrict__ active, cgym_kv_layout kv, int layer, int n_q_heads, float eps,
                          int32_t* status) {
  constexpr int D = 64, HALF = 32;
  pdl_trigger();
  const int row = blockIdx.x, lane = threadIdx.x & 31;
  const int head = blockIdx.y * 8 + (threadIdx.x >> 5);
  const int n_kv = kv.n_kv_heads;
  const bool valid = head < n_q_heads + n_kv, is_q = head < n_q_heads;
  // settled before the chain of dependent launches starts: position, RoPE row, norm weights
  const int pos = positions[row];
  const float c = Elem<T>::round(rope_cos[static_cast<int64_t>(pos) * HALF + lane]);
  const float s = Elem<T>::round(rope_sin[static_cast<int64_t>(pos) * HALF + lane]);
  const T* norm_w = is_q ? q_w : k_w;
  const float w_lo = Elem<T>::load(norm_w + lane), w_hi = Elem<T>::load(norm_w + lane + HALF);
  pdl_wait();
  if (!valid) return;
  qkv = pdl_fresh(qkv);
  const int width = (n_q_heads + 2 * n_kv) * D;
  const T* src = qkv + static_cast<int64_t>(row) * width + head * D;
  const float x_lo = Elem<T>::load(src + lane), x_hi = Elem<T>::load(src + lane + HALF);
  const float ms = __fadd_rn(warp_sum(x_lo * x_lo), warp_sum(x_hi * x_hi)) / static_cast<float>(D);
  const float inv = rsqrtf(ms + eps);
  const float n_lo = Elem<T>::round(__fmul_rn(Elem<T>::round(__fmul_rn(x_lo, inv)), w_lo));
  const float n_hi = Elem<T>::round(__fmul_rn(Elem<T>::round(__fmul_rn(x_hi, inv)), w_hi));
  const float rot_lo = Elem<T>::round(__fsub_rn(Elem<T>::round(__fmul_rn(n_lo, c)), Elem<T>::round(__fmul_rn(n_hi, s))));
  const float rot_hi = Elem<T>::round(__fadd_rn(Elem<T>::round(__fmul_rn(n_hi, c)), Elem<T>::round(__fmul_rn(n_lo, s))));
  if (is_q) {
    T* dst = q_out + (static_cast<int64_t>(row) * n_q_heads + head) * D;
    Elem<T>::store(dst + lane, rot_lo);
    Elem<T>::store(dst + lane + HALF, rot_hi);
    return;
  }
  const int kh = head - n_q_heads;
  const T* v_src = qkv + static_cast<int64_t>(row) * width + (n_q_heads + n_kv + kh) * D;
  const float v_lo = Elem<T>::load(v_src + lane), v_hi = Elem<T>::load(v_src + lane + HALF);
  if (k_new != nullptr) {
    const int64_t o = (static_cast<int64_t>(row) * n_kv + kh) * D;
    Elem<T>::store(k_new + o + lane, rot_lo);
    Elem<T>::store(k_new + o + lane + HALF, rot_hi);
    Elem<T>::store(v_new + o + lane, v_lo);
    Elem<T>::store(v_new + o + lane + HALF, v_hi);
  }
  if (active != nullptr && !active[row]) return;
  const int slot = slots != nullptr ? slots[row] : row;
  if (slot < 0) return;
  const int block = pos / kv.page_size, tok = pos % kv.page_size;
  const int page = block < kv.max_blocks ? kv.block_table[static_cast<int64_t>(slot) * kv.max_blocks + block] : -1;
  if (page < 0 || page >= kv.n_pages) {  // uniform across the warp
    if (lane == 0) atomicOr(status, CGYM_STATUS_BAD_PAGE);
    return;
  }
  KV* pool = static_cast<KV*>(kv.kv_pool);
  constexpr int EB = static_cast<int>(sizeof(KV));
  const int64_t k_lo = kv_k_offset(kv, layer, page, kh, tok, lane, EB), k_hi = kv_k_offset(kv, layer, page, kh, tok, lane + HALF, EB);
  const int64_t o_lo = kv_v_offset(kv, layer, page, kh, tok, lane, EB), o_hi = kv_v_offset(kv, layer, page, kh, tok, lane + HALF, EB);
  if constexpr (sizeof(KV) == 1) {
    const float ak = warp_max(fmaxf(fabsf(rot_lo), fabsf(rot_hi)));
    const float av = warp_max(fmaxf(fabsf(v_lo), fabsf(v_hi)));
    const float sk = fmaxf(ak / 448.0f, 1.0e-12f), sv = fmaxf(av / 448.0f, 1.0e-12f);
    uint8_t* bytes = reinterpret_cast<uint8_t*>(pool);
    bytes[k_lo] = to_e4m3(__fdiv_rn(rot_lo, sk));
    bytes[k_hi] = to_e4m3(__fdiv_rn(rot_hi, sk));
    bytes[o_lo] = to_e4m3(__fdiv_rn(v_lo, sv));
    bytes[o_hi] = to_e4m3(__fdiv_rn(v_hi, sv));
    if (lane == 0) {
      kv.kv_scales[kv_scale_offset(kv, layer, page, 0, kh, tok)] = sk;
      kv.kv_scales[kv_scale_offset(kv, layer, page, 1, kh, tok)] = sv;
    }
  } else {
    Elem<KV>::store(pool + k_lo, rot_lo);
    Elem<KV>::store(pool + k_hi, rot_hi);
    Elem<KV>::store(pool + o_lo, v_lo);
    Elem<KV>::store(pool + o_hi, v_hi);
  }
}

// ------------------------------------------------------------------------------------------
// logit[target] - logsumexp(logits) per row
// ------------------------------------------------------------------------------------------
template <typename T>
__global__ void target_logprob_kernel(float* __restrict__ out, const T* __restrict__ logits,
                                      const int64_t* __restrict__ targets, int vocab) {
  __shared__ float scratch[32];
  const T* row = logits + static_cast<int64_t>(blockIdx.x) * vocab;
  float m = -INFINITY;
  for (int i = threadIdx.x; i < vocab; i += blockDim.x) m = fmaxf(m, Elem<T>::load(row + i));
  m = block_max(m, scratch);
  float s = 0.0f;
  for (int i = threadIdx.x; i < vocab; i += blockDim.x) s += expf(Elem<T>::load(row + i) - m);
  s = block_sum(s, scratch);
  if (threadIdx.x == 0) out[blockIdx.x] = Elem<T>::load(row + targets[blockIdx.x]) - (m + logf(s));
}

}  // namespace cgym

using namespace cgym;

#define DISPATCH_DTYPE(dtype, ...)                                   \
  if ((dtype) == CGYM_F32) { using T = float; __VA_ARGS__; }         \
  else if ((dtype) == CGYM_BF16) { using T = __nv_bfloat16; __VA_ARGS__; } \
  else return fail("unsupported activation dtype %d", (dtype));

extern "C" int cgym_embedding(void* out, const void* table, const int64_t* tokens, int rows, int hidden,
                              int vocab, int dtype, cgym_stream_t stream) {
  CGYM_REQUIRE(rows >= 0 && hidden > 0 && vocab > 0, "embedding: bad shape");
  if (rows == 0) return 0;
  DISPATCH_DTYPE(dtype, launch_dependent(embedding_kernel<T>, dim3(rows), dim3(256), 0, as_stream(stream),
                                         static_cast<T*>(out), static_cast<const T*>(table), tokens, hidden, vocab));
  return check_launch("embedding");
}

extern "C" int cgym_rmsnorm(void* y, void* sum_out, const void* x, const void* residual, const void* w,
                            int rows, int hidden, float eps, int dtype, cgym_stream_t stream) {
  CGYM_REQUIRE(rows >= 0 && hidden > 0 && hidden <= 12288, "rmsnorm: hidden must be in [1, 12288]");
  CGYM_REQUIRE(residual == nullptr || sum_out != nullptr, "rmsnorm: residual needs sum_out");
  if (rows == 0) return 0;
  if (dtype == CGYM_BF16 && rms_fast_path(hidden, y, sum_out, x, residual, w)) {
    using B = __nv_bfloat16;
    launch_rms_fast<false>(static_cast<B*>(y), nullptr, nullptr, static_cast<B*>(sum_out), static_cast<const B*>(x),
                           static_cast<const B*>(residual), static_cast<const B*>(w), rows, hidden, eps,
                           as_stream(stream));
    return check_launch("rmsnorm");
  }
  DISPATCH_DTYPE(dtype, (launch_dependent(rmsnorm_kernel<T, false>, dim3(rows), dim3(256), hidden * sizeof(float),
                                          as_stream(stream), static_cast<T*>(y), nullptr, nullptr,
                                          static_cast<T*>(sum_out), static_cast<const T*>(x),
                                          static_cast<const T*>(residual), static_cast<const T*>(w), hidden, eps)));
  return check_launch("rmsnorm");
}

extern "C" int cgym_rmsnorm_quant(uint8_t* q, float* scales, void* sum_out, const void* x, const void* residual,
                                  const void* w, int rows, int hidden, float eps, cgym_stream_t stream) {
  CGYM_REQUIRE(rows >= 0 && hidden > 0 && hidden <= 12288, "rmsnorm_quant: hidden must be in [1, 12288]");
  CGYM_REQUIRE(residual == nullptr || sum_out != nullptr, "rmsnorm_quant: residual needs sum_out");
  if (rows == 0) return 0;
  using T = __nv_bfloat16;
  if (rms_fast_path(hidden, q, sum_out, x, residual, w) && (reinterpret_cast<uintptr_t>(q) & 7u) == 0) {
    launch_rms_fast<true>(nullptr, q, scales, static_cast<T*>(sum_out), static_cast<const T*>(x),
                          static_cast<const T*>(residual), static_cast<const T*>(w), rows, hidden, eps,
                          as_stream(stream));
    return check_launch("rmsnorm_quant");
  }
  launch_dependent(rmsnorm_kernel<T, true>, dim3(rows), dim3(256), hidden * sizeof(float), as_stream(stream), nullptr,
                   q, scales, static_cast<T*>(sum_out), static_cast<const T*>(x), static_cast<const T*>(residual),
                   static_cast<const T*>(w), hidden, eps);
  return check_launch("rmsnorm_quant");
}

extern "C" int cgym_swiglu(void* y, const void* gate_up, int rows, int ffn, int dtype, cgym_stream_t stream) {
  CGYM_REQUIRE(rows >= 0 && ffn > 0, "swiglu: bad shape");
  if (rows == 0) return 0;
  if (dtype == CGYM_BF16 && ffn % 8 == 0 && rows <= 65535 &&
      ((reinterpret_cast<uintptr_t>(y) | reinterpret_cast<uintptr_t>(gate_up)) & 15u) == 0) {
    using B = __nv_bfloat16;
    launch_dependent(swiglu_rows_bf16_kernel, dim3((ffn / 8 + 255) / 256, rows), dim3(256), 0, as_stream(stream),
                     static_cast<B*>(y), static_cast<const B*>(gate_up), ffn);
    return check_launch("swiglu");
  }
  dim3 grid((ffn + 255) / 256, rows);
  DISPATCH_DTYPE(dtype, launch_dependent(swiglu_kernel<T>, grid, dim3(256), 0, as_stream(stream), static_cast<T*>(y),
                                         static_cast<const T*>(gate_up), ffn));
  return check_launch("swiglu");
}

extern "C" int cgym_swiglu_quant(uint8_t* q, float* scales, const void* gate_up, int rows, int ffn,
                                 cgym_stream_t stream) {
  CGYM_REQUIRE(rows >= 0 && ffn > 0 && ffn <= 12288, "swiglu_quant: ffn must be in [1, 12288]");
  if (rows == 0) return 0;
  using T = __nv_bfloat16;
  const int chunks = (ffn / 8 + SWIGLU_Q_THREADS - 1) / SWIGLU_Q_THREADS;
  if (ffn % 8 == 0 && chunks <= 3 && (reinterpret_cast<uintptr_t>(gate_up) & 15u) == 0 &&
      (reinterpret_cast<uintptr_t>(q) & 7u) == 0) {
    const T* in = static_cast<const T*>(gate_up);
    const dim3 grid(rows), block(SWIGLU_Q_THREADS);
    if (chunks <= 1) launch_dependent(swiglu_quant_rows_bf16_kernel<1>, grid, block, 0, as_stream(stream), q, scales, in, ffn);
    else if (chunks == 2) launch_dependent(swiglu_quant_rows_bf16_kernel<2>, grid, block, 0, as_stream(stream), q, scales, in, ffn);
    else launch_dependent(swiglu_quant_rows_bf16_kernel<3>, grid, block, 0, as_stream(stream), q, scales, in, ffn);
    return check_launch("swiglu_quant");
  }
  launch_dependent(swiglu_quant_kernel<T>, dim3(rows), dim3(512), ffn * sizeof(float), as_stream(stream), q, scales,
                   static_cast<const T*>(gate_up), ffn);
  return check_launch("swiglu_quant");
}

extern "C" int cgym_quantize_rows(uint8_t* q, float* scales, const void* x, int rows, int width, int dtype,
                                  cgym_stream_t stream) {
  CGYM_REQUIRE(rows >= 0 && width > 0 && width <= 32768, "quantize_rows: FP8 row width must be in [1, 32768]");
  if (rows == 0) return 0;
  DISPATCH_DTYPE(dtype, quantize_rows_kernel<T><<<rows, 256, 0, as_stream(stream)>>>(
      q, scales, static_cast<const T*>(x), width));
  return check_launch("quantize_rows");
}

extern "C" int cgym_conv_update(void* y, void* state, const void* bcx, const void* conv_w, const uint8_t* active,
                                const int32_t* slots, int rows, int hidden, int dtype, cgym_stream_t stream) {
  CGYM_REQUIRE(rows >= 0 && hidden > 0, "conv_update: bad shape");
  if (rows == 0) return 0;
  dim3 grid((hidden + 255) / 256, rows);
  DISPATCH_DTYPE(dtype, launch_dependent(conv_update_kernel<T>, grid, dim3(256), 0, as_stream(stream),
                                         static_cast<T*>(y), static_cast<T*>(state), static_cast<const T*>(bcx),
                                         static_cast<const T*>(conv_w), active, slots, hidden));
  return check_launch("conv_update");
}

extern "C" int cgym_conv_prefill(void* y, void* state, const void* bcx, const void* conv_w,
                                 const int32_t* cu_seqlens, const int32_t* seq_slots, const int32_t* seq_starts,
                                 int n_seqs, int total_rows, int hidden, int dtype, cgym_stream_t stream) {
  CGYM_REQUIRE(n_seqs >= 0 && total_rows >= 0 && hidden > 0, "conv_prefill: bad shape");
  if (n_seqs == 0 || total_rows == 0) return 0;
  CGYM_REQUIRE(total_rows <= 65535 * 64, "conv_prefill: too many rows");
  dim3 grid((hidden + 255) / 256, total_rows);
  dim3 sgrid((hidden + 255) / 256, n_seqs);
  DISPATCH_DTYPE(dtype, {
    conv_prefill_kernel<T><<<grid, 256, 0, as_stream(stream)>>>(
        static_cast<T*>(y), static_cast<const T*>(state), static_cast<const T*>(bcx),
        static_cast<const T*>(conv_w), cu_seqlens, seq_slots, seq_starts, n_seqs, hidden);
    conv_prefill_state_kernel<T><<<sgrid, 256, 0, as_stream(stream)>>>(
        static_cast<T*>(state), static_cast<const T*>(bcx), cu_seqlens, seq_slots, seq_starts, hidden);
  });
  return check_launch("conv_prefill", 2);
}

extern "C" int cgym_qk_norm_rope_append(void* q_out, void* k_new, void* v_new, const void* qkv,
                                        const void* q_norm_w, const void* k_norm_w, const float* rope_cos,
                                        const float* rope_sin, const int32_t* positions, const int32_t* slots,
                                        const uint8_t* active, const cgym_kv_layout* kv, int layer, int rows,
                                        int n_q_heads, float eps, int dtype, int32_t* status,
                                        cgym_stream_t stream) {
  CGYM_REQUIRE(kv != nullptr && status != nullptr, "qk_norm_rope_append: kv layout and status are required");
  const int D = kv->head_dim;
  CGYM_REQUIRE(D == 32 || D == 64 || D == 128 || D == 256, "qk_norm_rope_append: head_dim must be 32, 64, 128 or 256");
  CGYM_REQUIRE((kv->page_size & (kv->page_size - 1)) == 0 && kv->page_size > 0, "page_size must be a power of two");
  CGYM_REQUIRE((k_new == nullptr) == (v_new == nullptr), "k_new and v_new go together");
  CGYM_REQUIRE(kv->kv_dtype != CGYM_E4M3 || kv->kv_scales != nullptr, "e4m3 KV needs a scale pool");
  if (rows == 0) return 0;
  CGYM_REQUIRE(n_q_heads + kv->n_kv_heads <= 65535, "too many heads");
  const bool per_warp = D == 64;  // one warp per head, eight heads per CTA
  dim3 grid(rows, per_warp ? (n_q_heads + kv->n_kv_heads + 7) / 8 : n_q_heads + kv->n_kv_heads);
#define LAUNCH_QK(T, KV)                                                                                   \
  if (per_warp)                                                                                            \
    launch_dependent(qk_rope_append_d64_kernel<T, KV>, grid, dim3(256), 0, as_stream(stream),              \
                     static_cast<T*>(q_out), static_cast<T*>(k_new), static_cast<T*>(v_new),               \
                     static_cast<const T*>(qkv), static_cast<const T*>(q_norm_w),                          \
                     static_cast<const T*>(k_norm_w), rope_cos, rope_sin, positions, slots, active, *kv,   \
                     layer, n_q_heads, eps, status);                                                       \
  else                                                                                                     \
  launch_dependent(qk_rope_append_kernel<T, KV>, grid, dim3(D), 0, as_stream(stream), static_cast<T*>(q_out),     \
                   static_cast<T*>(k_new), static_cast<T*>(v_new), static_cast<const T*>(qkv),                   \
                   static_cast<const T*>(q_norm_w), static_cast<const T*>(k_norm_w), rope_cos, rope_sin,         \
                   positions, slots, active, *kv, layer, n_q_heads, eps, status)
  if (dtype == CGYM_F32 && kv->kv_dtype == CGYM_F32) LAUNCH_QK(float, float);
  else if (dtype == CGYM_BF16 && kv->kv_dtype == CGYM_BF16) LAUNCH_QK(__nv_bfloat16, __nv_bfloat16);
  else if (dtype == CGYM_BF16 && kv->kv_dtype == CGYM_E4M3) LAUNCH_QK(__nv_bfloat16, uint8_t);
  else return fail("qk_norm_rope_append: unsupported dtype pair (%d, kv %d)", dtype, kv->kv_dtype);
#undef LAUNCH_QK
  return check_launch("qk_norm_rope_append");
}

extern "C" int cgym_target_logprobs(float* out, const void* logits, const int64_t* targets, int rows, int vocab,
                                    int dtype, cgym_stream_t stream) {
  CGYM_REQUIRE(rows >= 0 && vocab > 0, "target_logprobs: bad shape");
  if (rows == 0) return 0;
  DISPATCH_DTYPE(dtype, target_logprob_kernel<T><<<rows, 512, 0, as_stream(stream)>>>(
      out, static_cast<const T*>(logits), targets, vocab));
  return check_launch("target_logprobs");
}
