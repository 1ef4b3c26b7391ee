/*
 * cgym_b200 - C ABI of the B200-native LFM2.5 rollout-engine kernels (sm_100a).
 *
 * The reference (lms21a/climbing-gym) has no FFI: its hot path is Python calling Triton
 * kernels, FlashAttention and cuBLAS. Each entry point below replaces one of those call
 * sites; the comment on each cites the reference file:line it stands in for (paths are
 * relative to src/climbing_gym/inference/ in the reference project).
 *
 * Conventions
 *  - every pointer is a DEVICE pointer unless its name ends in _host;
 *  - all device memory is owned by the caller (PyTorch tensors on the Python side);
 *    the library allocates nothing unless an entry point says otherwise;
 *  - every launch goes on the caller's stream and is CUDA-graph capturable;
 *  - return value 0 = launched; non-zero = rejected before launch, message in
 *    cgym_last_error(); device-detected conditions are reported through an int32 status
 *    word the caller passes in (never a trap);
 *  - dtype: CGYM_F32 (0) or CGYM_BF16 (1) for activations/weights; KV caches may also be
 *    CGYM_E4M3 (2) with fp32 per-(token, head) scales.
 *  - "rows" are batch rows of one step; a row maps to a physical cache slot through
 *    `slots` (int32, may be NULL meaning row == slot; negative = padding row);
 *    `active` (uint8, may be NULL meaning all active) masks state writes.
 */
#ifndef CGYM_B200_H
#define CGYM_B200_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef void* cgym_stream_t; /* a cudaStream_t */

enum { CGYM_F32 = 0, CGYM_BF16 = 1, CGYM_E4M3 = 2 };

/* status-word bits written by device code */
enum {
  CGYM_STATUS_OK = 0,
  CGYM_STATUS_PAGE_POOL_EXHAUSTED = 1,
  CGYM_STATUS_BAD_PAGE = 2,
  CGYM_STATUS_WAIT_TIMEOUT = 4,
  CGYM_STATUS_CAPACITY = 8
};

/* Geometry of the paged hybrid cache (replaces the dense LFM25HybridCache,
 * lfm25_engine.py:370-431,1165-1221). One page holds `page_size` tokens of every KV head of one attention
 * layer. kv_pool is [layer][n_pages][kv_head][2 * page_size * head_dim] elements; one (page, head) block is
 *     K   as [token][dim]   (page_size rows of head_dim elements), followed by
 *     V^T as [dim][token]   (head_dim rows of page_size elements),
 * i.e. both are stored contraction-contiguous for the tensor-core attention kernels, and a block moves to
 * shared memory with one linear bulk copy. Inside every row the 16-byte chunks are permuted, in global
 * memory: chunk c of row r (c = byte offset / 16 within the row, n = chunks per row) is stored at chunk
 *     c ^ (r & 7)                      when n >= 8,
 *     c ^ ((r / (8 / n)) & (n - 1))    when n < 8 (8 / n consecutive rows share a 128-byte line),
 * so that 8 consecutive rows read at one logical column hit 8 different 16-byte bank groups. For K the row is
 * the token and the column the dim; for V^T the row is the dim and the column the token. Element (token t,
 * dim d) of K therefore lives at block + t * head_dim + swz(t, d / e, head_dim / e) * e + d % e with e = 16 /
 * element size, and of V at block + page_size * head_dim + d * page_size + swz(d, t / e, page_size / e) * e +
 * t % e. cgym_scatter_kv_dense / cgym_gather_kv_dense write and read the cache through this mapping. */
typedef struct {
  void* kv_pool;          /* element type kv_dtype */
  float* kv_scales;       /* [layer][n_pages][kv_head][k|v][token] fp32, only for CGYM_E4M3, else NULL */
  const int32_t* block_table; /* [n_slots][max_blocks] page ids, -1 = none */
  int32_t n_pages;
  int32_t page_size;      /* tokens per page, power of two */
  int32_t max_blocks;     /* block_table row length */
  int32_t n_kv_heads;
  int32_t head_dim;
  int32_t kv_dtype;
} cgym_kv_layout;

const char* cgym_last_error(void);
int cgym_version(void);
/* kernels this library has enqueued so far in this process (launches recorded into a CUDA graph
 * count once, at capture) */
long long cgym_launch_count(void);
/* Programmatic dependent launch for the kernels of the decode step (embedding, norms, GEMMs,
 * QK/RoPE/append, decode attention, conv update, SwiGLU, sampler): while enabled they are launched
 * with programmatic stream serialization, so a kernel is scheduled - and the GEMMs prefetch their
 * first weight tiles - while its predecessor is still draining; each of them waits for the
 * predecessor grid before touching dependent memory. What a kernel reads BEFORE that wait is, by
 * contract, settled before the chain of dependent launches begins: weights and tables, positions /
 * kv_lens / slots / active, block tables, conv taps and every cache position the step does not
 * write (in the decode step these come from cgym_step_begin - launched without the attribute, so it
 * completes before the chain starts - or from earlier steps). A caller that chains entry points
 * itself while this is enabled must keep to the same rule. Off by default; returns the previous setting.
 * The flag belongs to the calling host thread and is read at launch time by launches from that thread (set
 * it around a graph capture; other threads' launches, e.g. a second engine's, are unaffected). No reference
 * counterpart (the reference relies on CUDA graphs alone, lfm25_cuda.py:246-262). */
int cgym_set_pdl(int enabled);
/* 1 when the device of the current context is compute capability 10.x */
int cgym_device_supported(void);

/* F.embedding (lfm25_cuda.py:134). tokens int64 [rows]. */
int cgym_embedding(void* out, const void* table, const int64_t* tokens, int rows, int hidden,
                   int vocab, int dtype, cgym_stream_t stream);

/* _rms_kernel / rms_norm (lfm25_cuda_kernels.py:32-55): optional residual add, rounded and
 * emitted to sum_out; y = round(round(x*rsqrt(mean(x^2)+eps)) * w). */
int cgym_rmsnorm(void* y, void* sum_out, const void* x, const void* residual, const void* w,
                 int rows, int hidden, float eps, int dtype, cgym_stream_t stream);

/* _rms_quantize / rms_norm_fp8 (lfm25_fp8.py:26-64): as above, then per-row e4m3. */
int cgym_rmsnorm_quant(uint8_t* q, float* scales, void* sum_out, const void* x,
                       const void* residual, const void* w, int rows, int hidden, float eps,
                       cgym_stream_t stream);

/* _swiglu_kernel (lfm25_cuda_kernels.py:58-72): [rows, 2F] -> [rows, F]. */
int cgym_swiglu(void* y, const void* gate_up, int rows, int ffn, int dtype, cgym_stream_t stream);

/* _swiglu_quantize / swiglu_fp8 (lfm25_fp8.py:44-73). */
int cgym_swiglu_quant(uint8_t* q, float* scales, const void* gate_up, int rows, int ffn,
                      cgym_stream_t stream);

/* _quantize_rows (lfm25_fp8.py:16-23,108-116): per-row scale max(absmax/448, 1e-12). */
int cgym_quantize_rows(uint8_t* q, float* scales, const void* x, int rows, int width, int dtype,
                       cgym_stream_t stream);

/* _conv_kernel / conv_update (lfm25_cuda_kernels.py:75-110): gated short-conv (k=3) decode
 * step. state is [n_slots][3][hidden] (tap-major; newest tap last). */
int cgym_conv_update(void* y, void* state, const void* bcx, const void* conv_w,
                     const uint8_t* active, const int32_t* slots, int rows, int hidden, int dtype,
                     cgym_stream_t stream);

/* Prefill-side gated short-conv over packed sequences (lfm25_engine.py:1451-1511):
 * sequence s covers packed rows [cu_seqlens[s], cu_seqlens[s+1]) and cache slot seq_slots[s];
 * seq_starts[s] > 0 continues from the slot's stored taps (chunked prefill), 0 starts from
 * zeros. Writes the slot's final taps. */
int cgym_conv_prefill(void* y, void* state, const void* bcx, const void* conv_w,
                      const int32_t* cu_seqlens, const int32_t* seq_slots,
                      const int32_t* seq_starts, int n_seqs, int total_rows, int hidden,
                      int dtype, cgym_stream_t stream);

/* _qkv_kernel / prepare_qkv + KV append (lfm25_cuda_kernels.py:113-151, lfm25_batching.py:49-69,
 * lfm25_fp8_kv.py:27-70): per-head RMSNorm of q and k, RoPE with model-dtype coefficients,
 * q written to q_out [rows, Hq, D]; k and v of row r written into the paged cache of its slot at
 * positions[r] (e4m3 caches quantise per (token, head)). k_new/v_new (optional) also receive the
 * un-quantised rows [rows, Hkv, D]. */
int cgym_qk_norm_rope_append(void* q_out, void* k_new, void* v_new, const void* qkv,
                             const void* q_norm_w, const void* k_norm_w, const float* rope_cos,
                             const float* rope_sin, const int32_t* positions,
                             const int32_t* slots, const uint8_t* active,
                             const cgym_kv_layout* kv, int layer, int rows, int n_q_heads,
                             float eps, int dtype, int32_t* status, cgym_stream_t stream);

/* flash_attn_with_kvcache / fp8 decode+combine (lfm25_cuda.py:146-165,
 * lfm25_fp8_kv.py:72-172) and, for prefill rows, causal attention (lfm25_engine.py:1387-1394):
 * row r attends to cache positions [0, kv_lens[r]) of its slot. out [rows, Hq, D].
 * workspace: fp32, >= rows * Hq * n_splits * (D + 2) elements when n_splits > 1.
 * impl: 0 = auto, 1 = CUDA-core kernel (any dtype / head_dim / page size), 2 = tensor-core kernel
 * with bulk-copy page staging (bf16 activations, bf16 or e4m3 cache, head_dim 64, 64-token pages);
 * status is required for impl 2 (bounded waits report there).
 * While cgym_set_pdl(1) is in force, impl 2 starts fetching every page but a row's last one before
 * the kernel launched just ahead of it has finished: kv_lens, slots, active, the block table and
 * all cache positions below kv_lens[r] - 1 must then be final before that kernel starts (in the
 * decode step they come from cgym_step_begin and from earlier steps). */
int cgym_paged_attention(void* out, const void* q, const int32_t* kv_lens, const int32_t* slots,
                         const uint8_t* active, const cgym_kv_layout* kv, int layer, int rows,
                         int n_q_heads, float scale, int n_splits, float* workspace, int dtype,
                         int impl, int32_t* status, cgym_stream_t stream);

/* flash_attn_func on padded prompts (lfm25_engine.py:1387-1389,1415-1417), here on packed rows
 * against the paged cache: tile i is tile_ntok[i] (<= 128 / group) consecutive query tokens of one
 * sequence starting at packed row tile_row0[i] and cache position tile_pos0[i] in slot
 * tile_slot[i]; each token attends causally to cache positions [0, its position]. The tile's K/V
 * must already be in the cache (cgym_qk_norm_rope_append), which also makes a chunked prompt see
 * its earlier chunks. Tensor-core kernel: bf16 activations, bf16 or e4m3 cache, head_dim 64,
 * 64-token pages. q, out: [rows, Hq, D]. */
int cgym_prefill_attention(void* out, const void* q, const int32_t* tile_row0,
                           const int32_t* tile_ntok, const int32_t* tile_slot,
                           const int32_t* tile_pos0, const cgym_kv_layout* kv, int layer,
                           int n_tiles, int n_q_heads, float scale, int dtype, int32_t* status,
                           cgym_stream_t stream);

/* F.linear / cuBLAS GEMM and _gemv_kernel (lfm25_cuda_kernels.py:10-29; call sites
 * lfm25_cuda.py:124-126,141,166,170-172,180,192): y[M,N] = x[M,K] . w[N,K]^T, fp32 accumulate.
 * row_mask (uint8[M], optional): rows with 0 are not written (replaces the saved-logits
 * where-merge, lfm25_cuda.py:237-245). impl: 0 = auto, 1 = SIMT tile kernel, 2 = tcgen05/TMEM.
 * impl 3 = tcgen05 with split-K forced, 4 = CTA pairs (tcgen05.mma.cta_group::2, one 256 x 256 tile per
 * pair; N must be a multiple of 256), 5 = persistent CTA pairs (test hooks: auto picks among them by
 * shape). Split-K runs inside a thread-block cluster and is deterministic. workspace/workspace_bytes (optional, 16-byte aligned, contents irrelevant): when
 * it holds tiles * splits * token_tile * 128 fp32 (2 * 148 * token_tile * 512 bytes always suffice;
 * token_tile = 32 / 64 / 128 / 256 >= M) the partial tiles are exchanged through it (L2), which is
 * faster; without it they go through distributed shared memory, same bits. Launches that share a
 * workspace must be stream-ordered. status receives CGYM_STATUS_WAIT_TIMEOUT if a bounded barrier
 * wait gave up. */
int cgym_gemm(void* y, const void* x, const void* w, const uint8_t* row_mask, int M, int N, int K,
              int dtype, int impl, void* workspace, int64_t workspace_bytes, int32_t* status,
              cgym_stream_t stream);

/* Which kernel and grid cgym_gemm / cgym_gemm_fp8 take for a shape, without launching anything
 * (no reference counterpart; callable without a device). impl as in cgym_gemm (0 = auto, 2..5 = the tcgen05 forms);
 * in_dependent_chain != 0 plans as inside a captured decode step (cgym_set_pdl(1)). plan6 receives
 * {kind, token tile, feature sub-tiles per CTA, K splits, grid x, grid y}; kind 0 = single-CTA tiles,
 * 1 = CTA pairs with one tile per pair, 2 = persistent CTA pairs. */
int cgym_gemm_plan(int M, int N, int K, int fp8, int impl, int in_dependent_chain, int* plan6);

/* cgym_gemm whose output rows are scattered: token row m is written to y row row_map[m] (int32[M]; negative =
 * not written; NULL = cgym_gemm). Replaces the compact decode graphs' _scatter_logits copy
 * (lfm25_batching.py:25-33, 96-101): the LM head of a step over a compacted set of rows writes each row's
 * logits straight into its slot's row of the session-wide logits buffer. */
int cgym_gemm_scatter(void* y, const void* x, const void* w, const uint8_t* row_mask, const int32_t* row_map,
                      int M, int N, int K, int dtype, int impl, void* workspace, int64_t workspace_bytes,
                      int32_t* status, cgym_stream_t stream);

/* _matmul (+_reduce_split) / PackedFP8Weight.linear_quantized (lfm25_fp8.py:76-168):
 * y = bf16((xq . wq^T) * x_scales[m] * w_scales[n]). */
int cgym_gemm_fp8(void* y, const uint8_t* xq, const float* x_scales, const uint8_t* wq,
                  const float* w_scales, const uint8_t* row_mask, int M, int N, int K, int impl,
                  void* workspace, int64_t workspace_bytes, int32_t* status, cgym_stream_t stream);

/* cgym_gemm_fp8 with scattered output rows, for an FP8 LM head in a compact decode graph (see
 * cgym_gemm_scatter; lfm25_batching.py:25-33, lfm25_cuda.py:190-191). */
int cgym_gemm_fp8_scatter(void* y, const uint8_t* xq, const float* x_scales, const uint8_t* wq,
                          const float* w_scales, const uint8_t* row_mask, const int32_t* row_map, int M, int N,
                          int K, int impl, void* workspace, int64_t workspace_bytes, int32_t* status,
                          cgym_stream_t stream);

/* PackedBF16Weight (lfm25_bf16.py:17-102): a lossless 12-bit stream of a bf16 matrix for single-request
 * decode. Per weight: one byte of sign + mantissa, and a 4-bit exponent code (two per byte): code c in 1..15
 * stands for exponent base + c - 1, code 0 for "read the original value" (every bit pattern stays exact).
 * pack fills mantissa [numel] and exponent [numel / 2] from w (bf16, numel even); unpack rebuilds the bf16
 * matrix bit for bit; gemv computes y[N] = w[N, K] . x[K] from the stream (x, y bf16, fp32 accumulation, K
 * even and <= 16384, the original w still needed for code 0; row_mask (uint8[1], optional): 0 leaves y
 * untouched, like cgym_gemm's row mask). The reference's base is 110. */
int cgym_bf16_stream_pack(uint8_t* mantissa, uint8_t* exponent, const void* w, int64_t numel, int base,
                          cgym_stream_t stream);
int cgym_bf16_stream_unpack(void* out, const void* w, const uint8_t* mantissa, const uint8_t* exponent,
                            int64_t numel, int base, cgym_stream_t stream);
int cgym_bf16_stream_gemv(void* y, const void* x, const void* w, const uint8_t* mantissa, const uint8_t* exponent,
                          const uint8_t* row_mask, int N, int K, int base, cgym_stream_t stream);

/* Per-slot request state of the slot scheduler (LFM25GenerationSession's row tensors,
 * lfm25_session.py:147-167). All arrays are indexed by slot. */
typedef struct {
  int64_t* tokens;        /* [n_slots][capacity] generated ids */
  float* logprobs;        /* [n_slots][capacity] */
  int32_t* lengths;       /* generated so far */
  int32_t* limits;        /* per-request max_new_tokens */
  int8_t* reasons;        /* 0 running, 1 EOS, 2 stop, 3 length */
  uint8_t* alive;
  uint8_t* pending;       /* last sampled token not yet in the cache */
  int64_t* input_tokens;  /* next decode input */
  int64_t* stop_states;
  int64_t* stop_offsets;
  const int32_t* stop_table; /* flat [states*vocab] tables, next_state + 65536*matched */
  uint8_t* ignore_eos;
  int64_t* rng_positions;
  const int64_t* seeds;
  const float* temperatures;
  const int64_t* rng_offsets; /* Philox counter base per slot: row*vocab (batch keying) or 0 */
  const int32_t* force_eos_at; /* TEST HOOK, NULL in production: generated position whose token is replaced by
                                  EOS (-1 none); stands in for the sampler wrap the reference's tests use to
                                  force an EOS (tests/test_text_stops.py:122-126) */
  int32_t* seq_lens;      /* cache length per slot; advanced here for rows in `advance` */
  const float* min_logits; /* optional: per slot, logits below this value cannot be drawn (top-k / top-p
                              support from cgym_filter_thresholds); they still count in the log-prob */
  const float* gumbel_noise; /* optional, [n_slots][vocab] fp32: log(-log(u)) of this step's draw for every alive,
                                tempered slot, filled by cgym_gumbel_noise earlier in the step; NULL = the sampler
                                evaluates the Philox stream itself (same values either way) */
  const int32_t* out_rows; /* optional: slot s writes its tokens / log-probs to row out_rows[s] of `tokens` /
                              `logprobs` (which then hold more rows than slots) instead of row s: with
                              device-side slot turnover a request keeps its row after its slot is reused */
  int32_t capacity;
  int32_t eos_token_id;
} cgym_slot_state;

/* _partial_sample + _finish_sample + _record_sample fused (lfm25_sampling.py:10-58,
 * lfm25_session.py:34-56): Gumbel-max / greedy over logits [n_slots, vocab], sampled-token
 * log-prob from the untempered logits, then the per-slot bookkeeping. `advance` (uint8[n_slots],
 * optional) marks rows whose decode input was consumed this step: their seq_lens += 1
 * (lfm25_cuda.py:185-189). sampled_out/logp_out (optional) receive the raw draw per slot.
 * workspace (optional, cgym_sample_workspace_bytes(n_slots) bytes, zero before the first call and
 * re-armed by the kernel): lets a row's vocabulary be sliced over several CTAs, the reference's
 * 4096-wide tiles (lfm25_sampling.py:76-91); without it one CTA reduces a whole row. */
int cgym_sample_record(const void* logits, const cgym_slot_state* state, const uint8_t* advance,
                       int64_t* sampled_out, float* logp_out, int n_slots, int vocab, int dtype,
                       float* workspace, cgym_stream_t stream);

/* The noise half of the Gumbel-max draw, ahead of the logits: noise[slot][col] = log(-log(u)) with u the
 * reference sampler's uniform for (seed, rng position, offset + col) (tl.rand in _partial_sample,
 * lfm25_sampling.py:17-26), for every slot that is alive with temperature > 0 (other rows are left alone).
 * It depends on the slot state only, so a decode step launches it on a side stream at the start of the step,
 * beside the layers, and passes the buffer to cgym_sample_record through cgym_slot_state.gumbel_noise; the
 * draw is bit-identical to the sampler evaluating the stream itself. */
int cgym_gumbel_noise(float* noise, const cgym_slot_state* state, int n_slots, int vocab, cgym_stream_t stream);

/* Stand-alone sampler (sample_logits / RowSampler.sample, lfm25_sampling.py:61-123). */
int cgym_sample(int64_t* tokens, float* logprobs, const void* logits, const int64_t* seeds,
                const int64_t* steps, const float* temperatures, const int64_t* rng_offsets,
                int rows, int vocab, int dtype, float* workspace, cgym_stream_t stream);

/* Bytes of sampler workspace for `rows` rows (the scores / indices / maxima / totals scratch of
 * lfm25_sampling.py:77-80 plus one arrival counter per row). */
int64_t cgym_sample_workspace_bytes(int rows);

/* _apply_top_k_top_p (lfm25_engine.py:1759-1775) as a per-row value threshold for the fused sampler:
 * min_logits[r] = the smallest raw logit that stays drawable after top-k (keep logits >= the k-th
 * largest; top_k[r] <= 0 or >= vocab disables) and then top-p over the tempered softmax of what is
 * left (keep the values whose inclusive cumulative probability, in descending order, is <= top_p[r];
 * the most probable value always stays; top_p[r] >= 1 disables). A group of equal logits at the top-p
 * boundary is kept or dropped as a whole (torch.sort splits it arbitrarily). Rows with temperature 0
 * or no filter get -inf. One CTA per row, order-preserving bit-wise search with deterministic block
 * reductions (no float atomics), vocab <= 65536 per 1024 threads * 64. alive (uint8, optional) skips
 * dead rows. Feed the result to cgym_sample_record through cgym_slot_state.min_logits. */
int cgym_filter_thresholds(float* min_logits, const void* logits, const float* temperatures,
                           const int32_t* top_k, const float* top_p, const uint8_t* alive, int rows,
                           int vocab, int dtype, cgym_stream_t stream);

/* cgym_sample for callers that cannot hand over a workspace and must not cause a device
 * allocation: it has no counterpart in the reference, whose sampler allocates its slice scratch
 * with torch on every call. Same draws, slicing and results as cgym_sample with a workspace; the
 * slice scratch is a fixed 130 KiB array inside the library image, one copy per device.
 *  - At most CGYM_SAMPLE_STATIC_MAX_ROWS rows per call; more is rejected with an error that says
 *    so (split the batch, or use cgym_sample with your own workspace).
 *  - The first call on each device, made with that device current, resolves the address of the
 *    device's copy of the array (this may load the library's device code). Make that call before
 *    any stream capture begins on the device; rows = 0 does only this set-up and launches nothing.
 *  - EVERY call picks the array of the CURRENT device: make each call with the device that owns
 *    `stream` (and the tensors) current, or the kernel is handed another device's copy of the array.
 *  - Each call clears the row counters it needs with a memset on `stream` ahead of the kernel; it
 *    calls no allocating or freeing routine of the CUDA runtime.
 *  - Calls on one device share the one array: two calls whose execution can overlap (different
 *    streams, or different host threads without ordering) race on it and give undefined draws.
 *    Serialise them on one stream. The array keeps the last call's slices until the next call. */
#define CGYM_SAMPLE_STATIC_MAX_ROWS 512
int cgym_sample_static(int64_t* tokens, float* logprobs, const void* logits, const int64_t* seeds,
                       const int64_t* steps, const float* temperatures, const int64_t* rng_offsets,
                       int rows, int vocab, int dtype, cgym_stream_t stream);

/* behavior_topk + _record_head (lfm25_sampling.py:127-149, lfm25_session.py:22-31): for every live
 * slot, the k <= 128 most probable tokens of the UNFILTERED distribution, as ids (int32) and
 * log-probs (logit - logsumexp), sorted by descending logit (equal logits by ascending id), written
 * at out[slot][lengths[slot]][0..k) of buffers shaped [n_slots][capacity][k]. Run it before
 * cgym_sample_record of the same step (which advances lengths). alive / lengths optional (all live /
 * position 0). The head is metadata: it never changes the draw. */
int cgym_topk_head(int32_t* out_ids, float* out_logprobs, const void* logits, const uint8_t* alive,
                   const int32_t* lengths, int n_slots, int vocab, int capacity, int k, int dtype,
                   cgym_stream_t stream);

/* _apply_repetition_penalty + the seen-token mask of generate (lfm25_engine.py:1777-1791, :933-958,
 * lfm25_cuda.py:336-337): out[row][i] (fp32, [rows][vocab]) = logits[row][i], and for every token the
 * row has seen, logit * penalty when negative, logit / penalty otherwise. seen is one byte per
 * (row, token), set by the caller for the prompt's tokens; the row's latest generated token
 * (tokens[row][lengths[row] - 1], rows of `capacity` tokens; tokens may be NULL) counts as seen and its
 * byte is set here, so calling this once per step before the sampler keeps the mask current. Dead
 * rows (alive[row] == 0; alive optional) are left untouched. Feed `out` to cgym_filter_thresholds /
 * cgym_sample_record as CGYM_F32 logits: the recorded log-prob is then that of the penalised
 * distribution, as in the reference. */
int cgym_repetition_penalty(float* out, const void* logits, uint8_t* seen, const int64_t* tokens,
                            const int32_t* lengths, const uint8_t* alive, const float* penalties, int rows,
                            int vocab, int capacity, int dtype, cgym_stream_t stream);

/* Chunked-head completion scoring (lfm25_engine.py:1150-1154): logit[target] - logsumexp. */
int cgym_target_logprobs(float* out, const void* logits, const int64_t* targets, int rows,
                         int vocab, int dtype, cgym_stream_t stream);

/* GPU-resident page allocator (no reference counterpart: the reference cache is dense per
 * slot). free_bitmap bit=1 means free; pages are handed out lowest id first. */
typedef struct {
  uint32_t* free_bitmap;  /* [ceil(n_pages/32)] */
  int32_t* refcount;      /* [n_pages] */
  int32_t* block_table;   /* [n_slots][max_blocks] */
  int32_t* n_blocks;      /* [n_slots] pages held */
  int32_t n_pages;
  int32_t page_size;
  int32_t max_blocks;
  int32_t n_slots;
} cgym_page_pool;

/* Start of a decode step, inside the graph: snapshots pending -> active_out (the rows whose input
 * token is consumed this step, lfm25_session.py:467) when `pending` is given, else uses `active`;
 * then every active row whose next position (seq_lens[slot]) needs a page it does not hold yet
 * gets the lowest free page, rows served in row order. kv_lens_out (int32[rows], optional) receives
 * each row's attention length for this step, seq_lens[slot] + 1 (the cache_seqlens + new token of
 * flash_attn_with_kvcache, lfm25_cuda.py:156-165). At most 1024 rows. */
int cgym_step_begin(const cgym_page_pool* pool, const int32_t* seq_lens, const uint8_t* pending,
                    uint8_t* active_out, const uint8_t* active, const int32_t* slots,
                    int32_t* kv_lens_out, int rows, int32_t* status, cgym_stream_t stream);

/* Start of a decode step over a COMPACT set of rows (adaptive batching: _gather_inputs and the slot
 * indirection of capture_compact, lfm25_batching.py:11-23, 88-101). Row e stands for slot slots[e] (-1 =
 * padding row). Per row: row_active_out[e] = pending[slot] (pending is indexed by SLOT here),
 * row_tokens_out[e] = input_tokens[slot], row_positions_out[e] = seq_lens[slot], kv_lens_out[e] =
 * seq_lens[slot] + 1; padding rows get 0. slot_active_out (uint8[n_state_slots]) is cleared and then set for
 * the slots whose input is consumed this step: it is the `advance` mask cgym_sample_record wants, which stays
 * indexed by slot. Pages are allocated for active rows as in cgym_step_begin. At most 1024 rows. */
int cgym_step_begin_rows(const cgym_page_pool* pool, const int32_t* seq_lens, const uint8_t* pending,
                         const int64_t* input_tokens, const int32_t* slots, uint8_t* row_active_out,
                         uint8_t* slot_active_out, int64_t* row_tokens_out, int32_t* row_positions_out,
                         int32_t* kv_lens_out, int rows, int n_state_slots, int32_t* status, cgym_stream_t stream);

/* Reserve pages so slot s can hold need_tokens[s] tokens (admission / prefill chunk).
 * No reference counterpart (the reference allocates slots x capacity up front). */
int cgym_pages_reserve(const cgym_page_pool* pool, const int32_t* slot_ids,
                       const int32_t* need_tokens, int n, int32_t* status, cgym_stream_t stream);

/* Drop every page of the slots with release_mask != 0 (refcount-aware) and zero their
 * seq_lens (eviction of finished sequences; the reference only zeroes seq_lens on release,
 * lfm25_session.py:511-518). */
int cgym_pages_release(const cgym_page_pool* pool, const uint8_t* release_mask,
                       int32_t* seq_lens, cgym_stream_t stream);

/* Device-resident admission queue and result index of the slot scheduler. No reference counterpart: the
 * reference scans its slots on the host at every poll, releases finished requests from Python and admits
 * with a host-driven prefill (lfm25_session.py:259-292, 456-518). Here the host only parks prefilled prompts
 * (a spare row of the paged cache + the prompt's next-token logits) in this queue and later drains results;
 * finished requests leave their slots and parked ones enter them inside the decode graph.
 * Entry i lives at index i % capacity; entries [head, tail) are pending (the host publishes by advancing
 * tail, stream-ordered; the device consumes by advancing head). Results are indexed by request id %
 * result_capacity: the host must keep fewer than result_capacity requests between enqueue and delivery. */
typedef struct {
  const int32_t* rows;         /* [capacity] parked cache row that holds the entry's prefilled prompt */
  const int32_t* requests;     /* [capacity] request id (>= 0) */
  const int32_t* limits;       /* [capacity] max_new_tokens */
  const int64_t* seeds;        /* [capacity] */
  const float* temperatures;   /* [capacity] */
  const uint8_t* ignore_eos;   /* [capacity] */
  const int64_t* stop_offsets; /* [capacity] offset of the request's stop table in cgym_slot_state.stop_table */
  const void* logits;          /* [capacity][vocab] next-token logits after the prompt (model dtype) */
  int32_t* head;               /* [1] */
  const int32_t* tail;         /* [1] */
  int32_t capacity;
  int32_t result_capacity;
  int32_t* result_lengths;     /* [result_capacity] tokens generated, written when the request finishes */
  int8_t* result_reasons;      /* [result_capacity] finish reason (1 EOS, 2 stop, 3 length), 0 = not finished */
  int32_t* slot_requests;      /* [n_slots] request id in each slot, -1 = free */
  int32_t* out_rows;           /* [n_slots] = request id % result_capacity: pass as cgym_slot_state.out_rows */
  int32_t* adopt_rows;         /* [n_slots] scratch */
  int32_t* adopt_entries;      /* [n_slots] scratch */
  uint8_t* release_mask;       /* [n_rows] scratch; bytes beyond n_slots must stay 0 */
} cgym_admit_queue;

/* Slot turnover at the start of a decode step, on the device (capturable): every finished request's length
 * and reason are published under its request id and its pages returned to the pool; the queue's pending
 * entries are dealt first-in first-out to the free slots in ascending slot order; an adopting slot takes
 * over the parked row's block table (a move: no KV is copied, no reference count changes), length, conv taps
 * and logits row, and its request state is re-armed from the entry (length 0, alive, not pending), so the
 * step's sampler draws its first token from the prompt's logits. pool_rows spans all n_rows cache rows
 * (slots first); row_lens is [n_rows] (its first n_slots entries are the slots' seq_lens); conv_state is
 * [n_conv_layers][n_rows][3][hidden]; logits is [n_slots][vocab]. At most 1024 slots.
 * No reference counterpart (see cgym_admit_queue; host-side equivalent: lfm25_session.py:456-518). */
int cgym_slot_turnover(const cgym_page_pool* pool_rows, int n_slots, const cgym_slot_state* state,
                       const cgym_admit_queue* queue, void* logits, void* conv_state, int32_t* row_lens,
                       int n_conv_layers, int hidden, int vocab, int dtype, cgym_stream_t stream);

/* Share a prefix: dst slots get src's full pages by reference (refcount++) and a private copy of
 * the partially filled last page (replaces copy_prefix_from, lfm25_engine.py:400-423). */
int cgym_pages_fork(const cgym_page_pool* pool, const cgym_kv_layout* kv, int n_layers,
                    const int32_t* src_slots, const int32_t* dst_slots, const int32_t* prefix_lens,
                    int n, int32_t* status, cgym_stream_t stream);

/* ---- TEST HOOKS ----------------------------------------------------------------------------------------
 * The first two entry points below exist for tests: they read and write the paged cache through dense fp32 arrays,
 * standing in for the dense k_cache / v_cache views the reference's tests index directly. Nothing on the
 * generate path calls them. (cgym_slot_state.force_eos_at above and cgym_test_gemm_wait below are the other
 * test hooks of this ABI.) */

/* Test/debug helper: gather one slot's K or V history into a dense [len][Hkv][D] fp32 array
 * (dequantised), standing in for the dense k_cache/v_cache views the reference tests read
 * (tests/test_lfm25_adaptive.py:12-60). No reference counterpart as a kernel. */
int cgym_gather_kv_dense(float* out, const cgym_kv_layout* kv, int layer, int which, int slot,
                         int length, cgym_stream_t stream);

/* Test/debug helper, inverse of the gather: writes dense fp32 k, v [length][Hkv][D] into cache
 * positions [start, start + length) of one slot (pages must be reserved), quantising e4m3 caches
 * per (token, head) like the append kernel. No reference counterpart as a kernel (the reference
 * tests assign into k_cache / v_cache views, tests/test_lfm25_fp8_kv.py:24-90). */
int cgym_scatter_kv_dense(const float* k, const float* v, const cgym_kv_layout* kv, int layer,
                          int slot, int start, int length, cgym_stream_t stream);

/* Test hook for the bounded waits of the tcgen05 GEMM (no reference counterpart): limit_ns replaces the limit
 * (about two seconds) after which a wait that decides to give up does so (0 = restore it), and drop_loads != 0
 * makes the producer arm its barriers without issuing the tile copies, so the consumer's wait is one that
 * nothing satisfies. A GEMM launched in that state returns normally with CGYM_STATUS_WAIT_TIMEOUT in its status
 * word and an undefined y; nothing faults and nothing is left in flight. Call it with the device current and no
 * GEMM running; call it again with (0, 0) before any real work. */
int cgym_test_gemm_wait(unsigned long long limit_ns, int drop_loads);

#ifdef __cplusplus
}
#endif
#endif /* CGYM_B200_H */
