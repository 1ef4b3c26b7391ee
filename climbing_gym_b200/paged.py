"""Paged hybrid cache: block-table KV pages + per-slot short-conv taps, all resident in HBM.

This replaces the reference's dense per-slot cache (``LFM25HybridCache``,
src/climbing_gym/inference/lfm25_engine.py:370-431, allocation :1165-1221), whose footprint is
``slots x capacity`` whether or not a row uses it. Here a sequence holds
``ceil(len / page_size)`` pages, prefix pages are shared by reference between the samples of a
group, and the allocator state (free bitmap, refcounts, block tables) lives on the device so the
decode graph grows and evicts sequences without a host round-trip.

HBM layout
  kv_pool     [attn_layers, n_pages, kv_heads, 2 * page_size * head_dim]  model dtype or e4m3; one
              (page, head) block is K as [token][dim] followed by V^T as [dim][token], with the
              16-byte chunks of every row XOR-swizzled by the row index (the layout the attention
              kernels' shared-memory fragment loads want, so a block moves with one linear copy)
  kv_scales   [attn_layers, n_pages, kv_heads, 2 (k|v), page_size] fp32   (e4m3 only)
  conv_state  [conv_layers, n_slots, 3, hidden]   tap-major, newest tap last
  block_table [n_rows, max_blocks] int32, n_blocks [n_rows], seq_lens [n_rows]
  free_bitmap [ceil(n_pages/32)] (bit = 1: free), refcount [n_pages], status [1]

One page of one head is ``page_size * head_dim`` contiguous elements (8 KB for bf16 at 64 x 64),
i.e. one bulk copy per (page, head) for the attention kernels.

Rows: the first ``n_slots`` rows are the slots a decode step runs over; ``spare_rows`` more rows hold
sequences that are parked rather than decoded (a session's prefix snapshots). A spare row owns pages,
conv taps and a length like any slot, can be prefilled, and is the source of ``fork``; the step,
``release`` and everything sized by ``n_slots`` never see it.
"""
from __future__ import annotations

import ctypes as C

import torch

from . import _native as nv


class PagedHybridCache:
    def __init__(self, *, n_attn_layers: int, n_conv_layers: int, n_slots: int, max_seq_len: int,
                 n_kv_heads: int, head_dim: int, hidden_size: int, dtype: torch.dtype, device,
                 page_size: int = 64, n_pages: int | None = None, fp8_kv: bool = False, spare_rows: int = 0):
        if n_slots <= 0:
            raise ValueError("max_slots must be > 0")
        if max_seq_len <= 0:
            raise ValueError("max_seq_len must be > 0")
        if page_size <= 0 or page_size & (page_size - 1):
            raise ValueError("page_size must be a power of two")
        self.device = torch.device(device)
        self.dtype = dtype
        self.page_size = page_size
        self.n_slots = n_slots
        self.n_rows = n_rows = n_slots + max(0, int(spare_rows))
        self.max_blocks = -(-max_seq_len // page_size)
        self.capacity = max_seq_len
        self.n_pages = int(n_pages) if n_pages is not None else n_slots * self.max_blocks
        self.n_attn_layers, self.n_conv_layers = n_attn_layers, n_conv_layers
        self.n_kv_heads, self.head_dim, self.hidden_size = n_kv_heads, head_dim, hidden_size
        self.fp8_kv = bool(fp8_kv)
        dev = self.device
        if page_size < 16:
            raise ValueError("page_size must be at least 16 tokens")
        # one (page, head) block = K [token][dim] then V^T [dim][token], 16-byte chunks swizzled by row
        pool_shape = (max(n_attn_layers, 1), self.n_pages, n_kv_heads, 2 * page_size * head_dim)
        if fp8_kv:
            self.kv_pool = torch.zeros(pool_shape, device=dev, dtype=torch.uint8)
            self.kv_scales = torch.zeros((*pool_shape[:-1], 2, page_size), device=dev, dtype=torch.float32)
            self.kv_dtype = nv.E4M3
        else:
            self.kv_pool = torch.zeros(pool_shape, device=dev, dtype=dtype)
            self.kv_scales = None
            self.kv_dtype = nv.dtype_code(dtype)
        self.conv_state = torch.zeros((max(n_conv_layers, 1), n_rows, 3, hidden_size), device=dev, dtype=dtype)
        self.row_lens = torch.zeros(n_rows, device=dev, dtype=torch.int32)
        self.seq_lens = self.row_lens[:n_slots]  # the decode slots' lengths (same storage)
        self.block_table = torch.full((n_rows, self.max_blocks), -1, device=dev, dtype=torch.int32)
        self.n_blocks = torch.zeros(n_rows, device=dev, dtype=torch.int32)
        words = -(-self.n_pages // 32)
        bitmap = torch.full((words,), -1, dtype=torch.int32)
        if self.n_pages % 32:
            bitmap[-1] = (1 << (self.n_pages % 32)) - 1
        self.free_bitmap = bitmap.to(dev)
        self.refcount = torch.zeros(self.n_pages, device=dev, dtype=torch.int32)
        self.status = torch.zeros(1, device=dev, dtype=torch.int32)
        self._kv_struct = nv.KVLayout(nv.ptr(self.kv_pool), nv.ptr(self.kv_scales), nv.ptr(self.block_table),
                                      self.n_pages, page_size, self.max_blocks, n_kv_heads, head_dim, self.kv_dtype)
        self._pool_struct = nv.PagePool(nv.ptr(self.free_bitmap), nv.ptr(self.refcount), nv.ptr(self.block_table),
                                        nv.ptr(self.n_blocks), self.n_pages, page_size, self.max_blocks, n_slots)
        self._rows_struct = nv.PagePool(nv.ptr(self.free_bitmap), nv.ptr(self.refcount), nv.ptr(self.block_table),
                                        nv.ptr(self.n_blocks), self.n_pages, page_size, self.max_blocks, n_rows)

    # ---- views for the kernels -------------------------------------------------------------
    @property
    def kv(self):
        return C.byref(self._kv_struct)

    @property
    def pool(self):
        return C.byref(self._pool_struct)

    @property
    def pool_rows(self):
        """The same pool seen over every row, spare rows included (reserve / fork / release_rows)."""
        return C.byref(self._rows_struct)

    @property
    def max_slots(self) -> int:
        return self.n_slots

    @property
    def max_seq_len(self) -> int:
        return self.capacity

    def conv_layer(self, index: int) -> torch.Tensor:
        return self.conv_state[index]

    # ---- allocator calls (device-side; these only enqueue kernels) ---------------------------
    def reserve(self, slot_ids: torch.Tensor, need_tokens: torch.Tensor) -> None:
        """Make sure slot_ids[i] holds pages for need_tokens[i] tokens (int32 device tensors)."""
        nv.call("cgym_pages_reserve", self.pool_rows, nv.ptr(slot_ids), nv.ptr(need_tokens), slot_ids.numel(),
                nv.ptr(self.status), nv.stream_ptr(self.device))

    def release(self, mask: torch.Tensor) -> None:
        """Evict every slot whose mask byte is non-zero: pages back to the pool, seq_len = 0."""
        nv.call("cgym_pages_release", self.pool, nv.ptr(mask), nv.ptr(self.seq_lens), nv.stream_ptr(self.device))

    def release_rows(self, mask: torch.Tensor) -> None:
        """``release`` over all ``n_rows`` rows (one mask byte per row, spare rows included)."""
        nv.call("cgym_pages_release", self.pool_rows, nv.ptr(mask), nv.ptr(self.row_lens), nv.stream_ptr(self.device))

    def fork(self, src_slots: torch.Tensor, dst_slots: torch.Tensor, prefix_lens: torch.Tensor) -> None:
        """dst slots (empty) share src's full prefix pages and get a private copy of the partial
        last page, the conv taps and the sequence length."""
        nv.call("cgym_pages_fork", self.pool_rows, self.kv, self.n_attn_layers, nv.ptr(src_slots), nv.ptr(dst_slots),
                nv.ptr(prefix_lens), src_slots.numel(), nv.ptr(self.status), nv.stream_ptr(self.device))
        src, dst = src_slots.long(), dst_slots.long()
        self.conv_state[:, dst] = self.conv_state[:, src]
        self.row_lens[dst] = prefix_lens

    def check_status(self) -> None:
        """Host read of the device status word (call at poll boundaries, never per step)."""
        code = int(self.status.item())
        if code:
            self.status.zero_()
            problems = [name for bit, name in ((1, "page pool exhausted"), (2, "write to an unmapped page"),
                                               (4, "kernel wait timed out"), (8, "cache capacity exceeded")) if code & bit]
            raise RuntimeError("cache capacity exceeded: " + ", ".join(problems))

    # ---- dense views for tests / debugging ----------------------------------------------------
    def dense_kv(self, layer: int, slot: int, length: int | None = None) -> tuple[torch.Tensor, torch.Tensor]:
        """(k, v) of one slot as fp32 [length, kv_heads, head_dim] (dequantised for e4m3)."""
        length = int(self.seq_lens[slot]) if length is None else int(length)
        out = []
        for which in (0, 1):
            dense = torch.empty((length, self.n_kv_heads, self.head_dim), device=self.device, dtype=torch.float32)
            nv.call("cgym_gather_kv_dense", nv.ptr(dense), self.kv, layer, which, slot, length,
                    nv.stream_ptr(self.device))
            out.append(dense)
        return out[0], out[1]

    def write_dense_kv(self, layer: int, slot: int, start: int, k: torch.Tensor, v: torch.Tensor) -> None:
        """Test helper: store fp32 k, v [length, kv_heads, head_dim] at positions [start, start+length)."""
        k, v = k.contiguous().float(), v.contiguous().float()
        nv.call("cgym_scatter_kv_dense", nv.ptr(k), nv.ptr(v), self.kv, layer, slot, start, k.size(0),
                nv.stream_ptr(self.device))
        torch.cuda.current_stream(self.device).synchronize()  # k, v may be temporaries of the caller

    def dense_conv(self, layer: int, slot: int) -> torch.Tensor:
        """Conv taps of one slot in the reference's [hidden, 3] orientation."""
        return self.conv_state[layer, slot].transpose(0, 1)

    def free_pages(self) -> int:
        words = self.free_bitmap.cpu().numpy().view("uint32")
        return int(sum(bin(int(w)).count("1") for w in words))

    def bytes_allocated(self) -> int:
        tensors = [self.kv_pool, self.conv_state, self.block_table, self.free_bitmap, self.refcount]
        if self.kv_scales is not None:
            tensors.append(self.kv_scales)
        return sum(t.numel() * t.element_size() for t in tensors)
