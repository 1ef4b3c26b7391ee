// GPU-resident page allocator and block tables of the paged hybrid cache.
//
// State lives in device memory: a free bitmap (bit = 1: page free), a per-page reference count
// (prefix sharing), block_table[slot][block] and n_blocks[slot]. Pages are always handed out
// lowest id first and entries are served in entry order, so the tables are a pure function of
// the admit / step / release trace (restated on the CPU in oracle/pages.py). Everything runs on
// the caller's stream inside the decode graph; no host round-trip is involved.
#include "common.cuh"

namespace cgym {

constexpr int POOL_THREADS = 1024;

// exclusive scan of one int per thread over the block; returns the exclusive prefix and the total
__device__ __forceinline__ int block_exclusive_scan(int v, int* total, int* scratch /*33 ints*/) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  int inc = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int n = __shfl_up_sync(0xffffffffu, inc, o);
    if (lane >= o) inc += n;
  }
  __syncthreads();
  if (lane == 31) scratch[warp] = inc;
  __syncthreads();
  if (warp == 0) {
    int w = scratch[lane];
    int winc = w;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int n = __shfl_up_sync(0xffffffffu, winc, o);
      if (lane >= o) winc += n;
    }
    scratch[lane] = winc - w;
    if (lane == 31) scratch[32] = winc;
  }
  __syncthreads();
  *total = scratch[32];
  return scratch[warp] + inc - v;
}

// What a step over a compact set of rows (row e = slot slot_ids[e], -1 = padding) gathers per row from the
// per-slot request state, next to the per-slot copy of the row mask that the sampler's bookkeeping reads.
struct CompactRows {
  const int64_t* input_tokens;  // [n_slots] next decode input per slot
  int64_t* row_tokens;          // [rows]
  int32_t* row_positions;       // [rows] seq_lens[slot]
  uint8_t* slot_active;         // [n_state_slots] cleared, then 1 for the slots whose input is consumed this step
  int n_state_slots;
};

// Entries e < n ask that slot_e can hold need_e tokens. One CTA.
//   step mode   (need_tokens == nullptr): entry = batch row, need = seq_lens[slot] + 1 for active rows;
//                also snapshots pending -> active_out when given (pending is indexed by row, or by slot
//                when `compact` is given).
//   reserve mode: entry e = (slot_ids[e], need_tokens[e]).
__global__ void __launch_bounds__(POOL_THREADS)
pages_reserve_kernel(cgym_page_pool pool, const int32_t* __restrict__ slot_ids,
                     const int32_t* __restrict__ need_tokens, const int32_t* __restrict__ seq_lens,
                     const uint8_t* __restrict__ active, const uint8_t* __restrict__ pending_in,
                     uint8_t* __restrict__ active_out, int32_t* __restrict__ kv_lens_out, int n,
                     int32_t* __restrict__ status, CompactRows compact = CompactRows{}) {
  __shared__ int s_excl[POOL_THREADS + 1];
  __shared__ int s_old[POOL_THREADS];
  __shared__ int s_slot[POOL_THREADS];
  __shared__ int scratch[33];
  const int e = threadIdx.x;
  int cnt = 0, slot = -1, old = 0;
  if (compact.slot_active != nullptr) {
    for (int i = e; i < compact.n_state_slots; i += POOL_THREADS) compact.slot_active[i] = 0;
    __syncthreads();
  }
  if (e < n) {
    bool act = true;
    slot = slot_ids != nullptr ? slot_ids[e] : e;
    const bool valid = slot >= 0 && slot < pool.n_slots;
    if (compact.slot_active != nullptr) {
      act = valid && pending_in[slot] != 0;
      active_out[e] = act ? 1 : 0;
      if (act) compact.slot_active[slot] = 1;
      compact.row_tokens[e] = valid ? compact.input_tokens[slot] : 0;
      compact.row_positions[e] = valid ? seq_lens[slot] : 0;
    } else if (pending_in != nullptr) {
      act = pending_in[e] != 0;
      if (active_out != nullptr) active_out[e] = act ? 1 : 0;
    } else if (active != nullptr) {
      act = active[e] != 0;
    }
    // attention length of the row this step: its cached tokens plus the one being appended
    if (kv_lens_out != nullptr) kv_lens_out[e] = (slot >= 0 && slot < pool.n_slots) ? seq_lens[slot] + 1 : 0;
    if (act && slot >= 0 && slot < pool.n_slots) {
      const int need = need_tokens != nullptr ? need_tokens[e] : seq_lens[slot] + 1;
      int target = (need + pool.page_size - 1) / pool.page_size;
      if (target > pool.max_blocks) {
        atomicOr(status, CGYM_STATUS_CAPACITY);
        target = pool.max_blocks;
      }
      old = pool.n_blocks[slot];
      cnt = max(0, target - old);
    } else {
      slot = -1;
    }
  }
  int total = 0;
  const int excl = block_exclusive_scan(cnt, &total, scratch);
  s_excl[e] = excl;
  s_old[e] = old;
  s_slot[e] = slot;
  if (e == 0) s_excl[POOL_THREADS] = total;
  __syncthreads();
  if (total == 0) return;

  const int n_words = (pool.n_pages + 31) >> 5;
  int found = 0;  // free pages consumed so far (block-uniform)
  for (int base = 0; base < n_words && found < total; base += POOL_THREADS) {
    const int wi = base + threadIdx.x;
    uint32_t word = wi < n_words ? pool.free_bitmap[wi] : 0u;
    int chunk_total = 0;
    const int before = block_exclusive_scan(__popc(word), &chunk_total, scratch) + found;
    int r = before;
    uint32_t taken = 0u;
    while (word != 0u && r < total) {
      const int bit = __ffs(word) - 1;
      word &= word - 1u;
      taken |= 1u << bit;
      const int page = wi * 32 + bit;
      // entry owning rank r: last e with s_excl[e] <= r (entries with cnt 0 share a prefix value
      // with their successor, so search for the first prefix that exceeds r)
      int lo = 0, hi = POOL_THREADS;  // find smallest idx with s_excl[idx] > r; owner = idx - 1
      while (lo < hi) {
        const int mid = (lo + hi) >> 1;
        if (s_excl[mid] > r) hi = mid; else lo = mid + 1;
      }
      const int owner = lo - 1;
      const int block = s_old[owner] + (r - s_excl[owner]);
      pool.block_table[static_cast<int64_t>(s_slot[owner]) * pool.max_blocks + block] = page;
      pool.refcount[page] = 1;
      ++r;
    }
    if (taken != 0u) pool.free_bitmap[wi] &= ~taken;
    found += chunk_total;
  }
  const int granted = min(found, total);
  if (granted < total && threadIdx.x == 0) atomicOr(status, CGYM_STATUS_PAGE_POOL_EXHAUSTED);
  if (e < n && cnt > 0) {
    const int got = max(0, min(cnt, granted - excl));
    pool.n_blocks[slot] = old + got;
  }
}

__global__ void pages_release_kernel(cgym_page_pool pool, const uint8_t* __restrict__ release_mask,
                                     int32_t* __restrict__ seq_lens) {
  const int slot = blockIdx.x;
  if (!release_mask[slot]) return;
  const int held = pool.n_blocks[slot];
  __syncthreads();
  for (int b = threadIdx.x; b < held; b += blockDim.x) {
    int32_t* entry = pool.block_table + static_cast<int64_t>(slot) * pool.max_blocks + b;
    const int page = *entry;
    *entry = -1;
    if (page >= 0 && page < pool.n_pages && atomicSub(&pool.refcount[page], 1) == 1)
      atomicOr(&pool.free_bitmap[page >> 5], 1u << (page & 31));
  }
  if (threadIdx.x == 0) {
    pool.n_blocks[slot] = 0;
    if (seq_lens != nullptr) seq_lens[slot] = 0;
  }
}

// dst slots (empty) take src's full prefix pages by reference
__global__ void pages_share_kernel(cgym_page_pool pool, const int32_t* __restrict__ src_slots,
                                   const int32_t* __restrict__ dst_slots, const int32_t* __restrict__ prefix_lens) {
  const int i = blockIdx.x;
  const int src = src_slots[i], dst = dst_slots[i];
  const int full = prefix_lens[i] / pool.page_size;
  for (int b = threadIdx.x; b < full; b += blockDim.x) {
    const int page = pool.block_table[static_cast<int64_t>(src) * pool.max_blocks + b];
    pool.block_table[static_cast<int64_t>(dst) * pool.max_blocks + b] = page;
    if (page >= 0) atomicAdd(&pool.refcount[page], 1);
  }
  if (threadIdx.x == 0) pool.n_blocks[dst] = full;
}

// private copy of the partially filled last prefix page, all layers / K and V / heads
template <typename KV>
__global__ void pages_copy_tail_kernel(cgym_page_pool pool, cgym_kv_layout kv, const int32_t* __restrict__ src_slots,
                                       const int32_t* __restrict__ dst_slots, const int32_t* __restrict__ prefix_lens) {
  const int i = blockIdx.x;
  const int rem = prefix_lens[i] % pool.page_size;
  if (rem == 0) return;
  const int block = prefix_lens[i] / pool.page_size;
  const int sp = pool.block_table[static_cast<int64_t>(src_slots[i]) * pool.max_blocks + block];
  const int dp = pool.block_table[static_cast<int64_t>(dst_slots[i]) * pool.max_blocks + block];
  if (sp < 0 || dp < 0 || sp == dp) return;
  const int plane = blockIdx.y;  // layer * n_kv_heads + head
  const int head = plane % kv.n_kv_heads, layer = plane / kv.n_kv_heads;
  // the whole (page, head) block is copied: tokens past `rem` are don't-care in both copies
  KV* pool_data = static_cast<KV*>(kv.kv_pool);
  const int64_t so = kv_block_offset(kv, layer, sp, head), doff = kv_block_offset(kv, layer, dp, head);
  const int block_elems = 2 * kv.page_size * kv.head_dim;
  for (int j = threadIdx.x; j < block_elems; j += blockDim.x) pool_data[doff + j] = pool_data[so + j];
  if (kv.kv_scales != nullptr) {
    const int64_t ss = kv_scale_offset(kv, layer, sp, 0, head, 0), ds = kv_scale_offset(kv, layer, dp, 0, head, 0);
    for (int j = threadIdx.x; j < 2 * kv.page_size; j += blockDim.x) kv.kv_scales[ds + j] = kv.kv_scales[ss + j];
  }
}

template <typename KV>
__global__ void gather_kv_dense_kernel(float* __restrict__ out, cgym_kv_layout kv, int layer, int which, int slot) {
  const int tok = blockIdx.x;
  const int page = kv.block_table[static_cast<int64_t>(slot) * kv.max_blocks + tok / kv.page_size];
  const int width = kv.n_kv_heads * kv.head_dim;
  for (int j = threadIdx.x; j < width; j += blockDim.x) {
    const int head = j / kv.head_dim, d = j % kv.head_dim;
    float v = 0.0f;
    if (page >= 0) {
      const int eb = static_cast<int>(sizeof(KV));
      const int64_t off = which == 0 ? kv_k_offset(kv, layer, page, head, tok % kv.page_size, d, eb)
                                     : kv_v_offset(kv, layer, page, head, tok % kv.page_size, d, eb);
      if constexpr (sizeof(KV) == 1) {
        v = from_e4m3(static_cast<const uint8_t*>(kv.kv_pool)[off]) *
            kv.kv_scales[kv_scale_offset(kv, layer, page, which, head, tok % kv.page_size)];
      } else {
        v = Elem<KV>::load(static_cast<const KV*>(kv.kv_pool) + off);
      }
    }
    out[static_cast<int64_t>(tok) * width + j] = v;
  }
}

// inverse of the gather: rows [start, start + gridDim.x) of one slot from dense fp32 [len][Hkv][D];
// e4m3 caches quantise per (token, head) exactly like the append kernel. grid (len, Hkv), block D.
template <typename KV>
__global__ void scatter_kv_dense_kernel(const float* __restrict__ k, const float* __restrict__ v, cgym_kv_layout kv,
                                        int layer, int slot, int start) {
  __shared__ float scratch[32];
  const int tok = start + blockIdx.x, head = blockIdx.y, d = threadIdx.x;
  const int page = kv.block_table[static_cast<int64_t>(slot) * kv.max_blocks + tok / kv.page_size];
  if (page < 0) return;
  const int64_t src = (static_cast<int64_t>(blockIdx.x) * kv.n_kv_heads + head) * kv.head_dim + d;
  const float kval = k[src], vval = v[src];
  const int eb = static_cast<int>(sizeof(KV));
  const int64_t ko = kv_k_offset(kv, layer, page, head, tok % kv.page_size, d, eb);
  const int64_t vo = kv_v_offset(kv, layer, page, head, tok % kv.page_size, d, eb);
  if constexpr (sizeof(KV) == 1) {
    const float sk = fmaxf(block_max(fabsf(kval), scratch) / 448.0f, 1.0e-12f);
    const float sv = fmaxf(block_max(fabsf(vval), scratch) / 448.0f, 1.0e-12f);
    static_cast<uint8_t*>(kv.kv_pool)[ko] = to_e4m3(__fdiv_rn(kval, sk));
    static_cast<uint8_t*>(kv.kv_pool)[vo] = to_e4m3(__fdiv_rn(vval, sv));
    if (d == 0) {
      kv.kv_scales[kv_scale_offset(kv, layer, page, 0, head, tok % kv.page_size)] = sk;
      kv.kv_scales[kv_scale_offset(kv, layer, page, 1, head, tok % kv.page_size)] = sv;
    }
  } else {
    Elem<KV>::store(static_cast<KV*>(kv.kv_pool) + ko, kval);
    Elem<KV>::store(static_cast<KV*>(kv.kv_pool) + vo, vval);
  }
}

// ---- slot turnover: eviction of finished requests and admission from a device-resident queue -------------
// Runs at the start of a decode step, inside the captured graph. Three kernels:
//   1. slot_turnover_kernel (one CTA): publishes the length / finish reason of every finished request under
//      its request id, marks its slot for eviction, and deals the queue's pending entries to the free slots
//      (free now or just finished) in ascending slot order, entry order first-in first-out. An adopted
//      slot's request state is re-armed from the entry. Everything is a pure function of the state it
//      reads, so the schedule is reproducible.
//   2. pages_release_kernel: the evicted slots' pages go back to the pool.
//   3. slot_adopt_kernel: an adopting slot takes over the parked row's block table (a move: no reference
//      count changes, no KV copy), its length, conv taps and next-token logits; the parked row is left empty.
__global__ void __launch_bounds__(POOL_THREADS)
slot_turnover_kernel(cgym_slot_state st, cgym_admit_queue q, int n_slots) {
  __shared__ int scratch[33];
  const int s = threadIdx.x;
  int is_free = 0, finished = 0;
  if (s < n_slots) {
    const int rid = q.slot_requests[s];
    finished = rid >= 0 && st.reasons[s] != 0;
    if (finished) {
      const int slot_of_result = rid % q.result_capacity;
      q.result_lengths[slot_of_result] = st.lengths[s];
      q.result_reasons[slot_of_result] = st.reasons[s];
    }
    is_free = rid < 0 || finished;
  }
  int total_free = 0;
  const int rank = block_exclusive_scan(is_free, &total_free, scratch);
  const int head = *q.head, available = *q.tail - head;
  if (s < n_slots) {
    int adopt_row = -1, adopt_entry = -1;
    if (is_free && rank < available) {
      adopt_entry = (head + rank) % q.capacity;
      adopt_row = q.rows[adopt_entry];
      const int rid = q.requests[adopt_entry];
      q.slot_requests[s] = rid;
      q.out_rows[s] = rid % q.result_capacity;
      st.lengths[s] = 0;
      st.reasons[s] = 0;
      st.alive[s] = 1;
      st.pending[s] = 0;
      st.stop_states[s] = 0;
      st.rng_positions[s] = 0;
      st.limits[s] = q.limits[adopt_entry];
      st.ignore_eos[s] = q.ignore_eos[adopt_entry];
      st.stop_offsets[s] = q.stop_offsets[adopt_entry];
      // armed by the scheduler, read-only for the sampler: the same device arrays, written here
      const_cast<int64_t*>(st.seeds)[s] = q.seeds[adopt_entry];
      const_cast<float*>(st.temperatures)[s] = q.temperatures[adopt_entry];
      const_cast<int64_t*>(st.rng_offsets)[s] = 0;
    } else if (finished) {
      q.slot_requests[s] = -1;
      st.reasons[s] = 0;  // published above; the slot is free and must not be published again
      st.alive[s] = 0;
      st.pending[s] = 0;
    }
    q.adopt_rows[s] = adopt_row;
    q.adopt_entries[s] = adopt_entry;
    q.release_mask[s] = finished ? 1 : 0;
  }
  __syncthreads();
  if (threadIdx.x == 0) *q.head = head + min(total_free, max(available, 0));
}

template <typename T>
__global__ void slot_adopt_kernel(cgym_page_pool pool, cgym_admit_queue q, int32_t* __restrict__ row_lens,
                                  T* __restrict__ logits, T* __restrict__ conv_state, int n_conv_layers, int n_rows,
                                  int hidden, int vocab) {
  const int s = blockIdx.x;
  const int row = q.adopt_rows[s];
  if (row < 0) return;
  const int entry = q.adopt_entries[s];
  for (int b = threadIdx.x; b < pool.max_blocks; b += blockDim.x) {
    int32_t* from = pool.block_table + static_cast<int64_t>(row) * pool.max_blocks + b;
    pool.block_table[static_cast<int64_t>(s) * pool.max_blocks + b] = *from;
    *from = -1;
  }
  const T* src_logits = static_cast<const T*>(q.logits) + static_cast<int64_t>(entry) * vocab;
  for (int i = threadIdx.x; i < vocab; i += blockDim.x) logits[static_cast<int64_t>(s) * vocab + i] = src_logits[i];
  const int taps = 3 * hidden;
  for (int layer = 0; layer < n_conv_layers; ++layer) {
    const T* from = conv_state + (static_cast<int64_t>(layer) * n_rows + row) * taps;
    T* to = conv_state + (static_cast<int64_t>(layer) * n_rows + s) * taps;
    for (int i = threadIdx.x; i < taps; i += blockDim.x) to[i] = from[i];
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    pool.n_blocks[s] = pool.n_blocks[row];
    pool.n_blocks[row] = 0;
    row_lens[s] = row_lens[row];
    row_lens[row] = 0;
  }
}

static int check_pool(const cgym_page_pool* pool) {
  CGYM_REQUIRE(pool != nullptr && pool->free_bitmap && pool->refcount && pool->block_table && pool->n_blocks,
               "page pool is incomplete");
  CGYM_REQUIRE(pool->n_pages > 0 && pool->max_blocks > 0 && pool->n_slots > 0, "page pool has an empty dimension");
  CGYM_REQUIRE(pool->page_size > 0 && (pool->page_size & (pool->page_size - 1)) == 0,
               "page_size must be a power of two");
  return 0;
}

}  // namespace cgym

using namespace cgym;

extern "C" int cgym_step_begin(const cgym_page_pool* pool, const int32_t* seq_lens, const uint8_t* pending,
                               uint8_t* active_out, const uint8_t* active, const int32_t* slots,
                               int32_t* kv_lens_out, int rows, int32_t* status, cgym_stream_t stream) {
  if (int rc = check_pool(pool)) return rc;
  CGYM_REQUIRE(seq_lens != nullptr && status != nullptr, "step_begin: seq_lens and status are required");
  CGYM_REQUIRE(rows >= 0 && rows <= POOL_THREADS, "step_begin: at most 1024 rows per step");
  if (rows == 0) return 0;
  pages_reserve_kernel<<<1, POOL_THREADS, 0, as_stream(stream)>>>(*pool, slots, nullptr, seq_lens, active, pending,
                                                                  active_out, kv_lens_out, rows, status);
  return check_launch("step_begin");
}

extern "C" int cgym_step_begin_rows(const cgym_page_pool* pool, const int32_t* seq_lens, const uint8_t* pending,
                                    const int64_t* input_tokens, const int32_t* slots, uint8_t* row_active_out,
                                    uint8_t* slot_active_out, int64_t* row_tokens_out, int32_t* row_positions_out,
                                    int32_t* kv_lens_out, int rows, int n_state_slots, int32_t* status,
                                    cgym_stream_t stream) {
  if (int rc = check_pool(pool)) return rc;
  CGYM_REQUIRE(seq_lens && pending && input_tokens && slots && row_active_out && slot_active_out && row_tokens_out &&
                   row_positions_out && kv_lens_out && status,
               "step_begin_rows: every array is required");
  CGYM_REQUIRE(rows >= 0 && rows <= POOL_THREADS, "step_begin_rows: at most 1024 rows per step");
  CGYM_REQUIRE(n_state_slots >= 0 && n_state_slots <= pool->n_slots, "step_begin_rows: n_state_slots out of range");
  if (rows == 0) return 0;
  const CompactRows compact{input_tokens, row_tokens_out, row_positions_out, slot_active_out, n_state_slots};
  pages_reserve_kernel<<<1, POOL_THREADS, 0, as_stream(stream)>>>(*pool, slots, nullptr, seq_lens, nullptr, pending,
                                                                  row_active_out, kv_lens_out, rows, status, compact);
  return check_launch("step_begin_rows");
}

extern "C" int cgym_pages_reserve(const cgym_page_pool* pool, const int32_t* slot_ids, const int32_t* need_tokens,
                                  int n, int32_t* status, cgym_stream_t stream) {
  if (int rc = check_pool(pool)) return rc;
  CGYM_REQUIRE(slot_ids && need_tokens && status, "pages_reserve: slot_ids, need_tokens and status are required");
  CGYM_REQUIRE(n >= 0, "pages_reserve: negative count");
  for (int done = 0; done < n; done += POOL_THREADS) {
    const int m = n - done < POOL_THREADS ? n - done : POOL_THREADS;
    pages_reserve_kernel<<<1, POOL_THREADS, 0, as_stream(stream)>>>(*pool, slot_ids + done, need_tokens + done,
                                                                    nullptr, nullptr, nullptr, nullptr, nullptr, m,
                                                                    status);
  }
  return check_launch("pages_reserve", (n + POOL_THREADS - 1) / POOL_THREADS);
}

extern "C" int cgym_pages_release(const cgym_page_pool* pool, const uint8_t* release_mask, int32_t* seq_lens,
                                  cgym_stream_t stream) {
  if (int rc = check_pool(pool)) return rc;
  CGYM_REQUIRE(release_mask != nullptr, "pages_release: mask is required");
  pages_release_kernel<<<pool->n_slots, 128, 0, as_stream(stream)>>>(*pool, release_mask, seq_lens);
  return check_launch("pages_release");
}

extern "C" int cgym_slot_turnover(const cgym_page_pool* pool_rows, int n_slots, const cgym_slot_state* state,
                                  const cgym_admit_queue* queue, void* logits, void* conv_state, int32_t* row_lens,
                                  int n_conv_layers, int hidden, int vocab, int dtype, cgym_stream_t stream) {
  if (int rc = check_pool(pool_rows)) return rc;
  CGYM_REQUIRE(state && queue && logits && conv_state && row_lens, "slot_turnover: missing argument");
  CGYM_REQUIRE(n_slots > 0 && n_slots <= POOL_THREADS && n_slots <= pool_rows->n_slots,
               "slot_turnover: n_slots must be in [1, 1024] and within the pool's rows");
  CGYM_REQUIRE(queue->capacity > 0 && queue->result_capacity > 0 && queue->rows && queue->requests && queue->head &&
                   queue->tail && queue->slot_requests && queue->out_rows && queue->adopt_rows &&
                   queue->adopt_entries && queue->release_mask && queue->result_lengths && queue->result_reasons,
               "slot_turnover: the admission queue is incomplete");
  const cudaStream_t cs = as_stream(stream);
  slot_turnover_kernel<<<1, POOL_THREADS, 0, cs>>>(*state, *queue, n_slots);
  cgym_page_pool slots_view = *pool_rows;  // eviction walks the decode slots only
  slots_view.n_slots = n_slots;
  pages_release_kernel<<<n_slots, 128, 0, cs>>>(slots_view, queue->release_mask, row_lens);
  const int n_rows = pool_rows->n_slots;
  if (dtype == CGYM_F32)
    slot_adopt_kernel<float><<<n_slots, 256, 0, cs>>>(*pool_rows, *queue, row_lens, static_cast<float*>(logits),
                                                      static_cast<float*>(conv_state), n_conv_layers, n_rows, hidden,
                                                      vocab);
  else if (dtype == CGYM_BF16)
    slot_adopt_kernel<__nv_bfloat16><<<n_slots, 256, 0, cs>>>(
        *pool_rows, *queue, row_lens, static_cast<__nv_bfloat16*>(logits), static_cast<__nv_bfloat16*>(conv_state),
        n_conv_layers, n_rows, hidden, vocab);
  else
    return fail("slot_turnover: unsupported dtype %d", dtype);
  return check_launch("slot_turnover", 3);
}

extern "C" int cgym_pages_fork(const cgym_page_pool* pool, const cgym_kv_layout* kv, int n_layers,
                               const int32_t* src_slots, const int32_t* dst_slots, const int32_t* prefix_lens, int n,
                               int32_t* status, cgym_stream_t stream) {
  if (int rc = check_pool(pool)) return rc;
  CGYM_REQUIRE(kv && src_slots && dst_slots && prefix_lens && status, "pages_fork: missing argument");
  CGYM_REQUIRE(n >= 0 && n <= POOL_THREADS, "pages_fork: at most 1024 children per call");
  if (n == 0) return 0;
  pages_share_kernel<<<n, 128, 0, as_stream(stream)>>>(*pool, src_slots, dst_slots, prefix_lens);
  pages_reserve_kernel<<<1, POOL_THREADS, 0, as_stream(stream)>>>(*pool, dst_slots, prefix_lens, nullptr, nullptr,
                                                                  nullptr, nullptr, nullptr, n, status);
  dim3 grid(n, n_layers * kv->n_kv_heads);
  if (kv->kv_dtype == CGYM_F32) pages_copy_tail_kernel<float><<<grid, 256, 0, as_stream(stream)>>>(*pool, *kv, src_slots, dst_slots, prefix_lens);
  else if (kv->kv_dtype == CGYM_BF16) pages_copy_tail_kernel<__nv_bfloat16><<<grid, 256, 0, as_stream(stream)>>>(*pool, *kv, src_slots, dst_slots, prefix_lens);
  else if (kv->kv_dtype == CGYM_E4M3) pages_copy_tail_kernel<uint8_t><<<grid, 256, 0, as_stream(stream)>>>(*pool, *kv, src_slots, dst_slots, prefix_lens);
  else return fail("pages_fork: unsupported kv dtype %d", kv->kv_dtype);
  return check_launch("pages_fork", 3);
}

extern "C" int cgym_gather_kv_dense(float* out, const cgym_kv_layout* kv, int layer, int which, int slot, int length,
                                    cgym_stream_t stream) {
  CGYM_REQUIRE(kv != nullptr && out != nullptr && length >= 0, "gather_kv_dense: bad arguments");
  if (length == 0) return 0;
  if (kv->kv_dtype == CGYM_F32) gather_kv_dense_kernel<float><<<length, 128, 0, as_stream(stream)>>>(out, *kv, layer, which, slot);
  else if (kv->kv_dtype == CGYM_BF16) gather_kv_dense_kernel<__nv_bfloat16><<<length, 128, 0, as_stream(stream)>>>(out, *kv, layer, which, slot);
  else if (kv->kv_dtype == CGYM_E4M3) gather_kv_dense_kernel<uint8_t><<<length, 128, 0, as_stream(stream)>>>(out, *kv, layer, which, slot);
  else return fail("gather_kv_dense: unsupported kv dtype %d", kv->kv_dtype);
  return check_launch("gather_kv_dense");
}

extern "C" int cgym_scatter_kv_dense(const float* k, const float* v, const cgym_kv_layout* kv, int layer, int slot,
                                     int start, int length, cgym_stream_t stream) {
  CGYM_REQUIRE(kv != nullptr && k != nullptr && v != nullptr && length >= 0 && start >= 0,
               "scatter_kv_dense: bad arguments");
  if (length == 0) return 0;
  dim3 grid(length, kv->n_kv_heads);
  if (kv->kv_dtype == CGYM_F32) scatter_kv_dense_kernel<float><<<grid, kv->head_dim, 0, as_stream(stream)>>>(k, v, *kv, layer, slot, start);
  else if (kv->kv_dtype == CGYM_BF16) scatter_kv_dense_kernel<__nv_bfloat16><<<grid, kv->head_dim, 0, as_stream(stream)>>>(k, v, *kv, layer, slot, start);
  else if (kv->kv_dtype == CGYM_E4M3) scatter_kv_dense_kernel<uint8_t><<<grid, kv->head_dim, 0, as_stream(stream)>>>(k, v, *kv, layer, slot, start);
  else return fail("scatter_kv_dense: unsupported kv dtype %d", kv->kv_dtype);
  return check_launch("scatter_kv_dense");
}
