"""ctypes binding of libcgym_b200.so (the C ABI declared in include/cgym_b200.h).

The library is the only compute path: importing this module never falls back to PyTorch
or CPU code. ``load()`` raises ``NativeLibraryError`` when the shared object is missing
(build it with ``python -m climbing_gym_b200.build``) and every wrapper raises
``NativeKernelError`` with the library's own message when a call is rejected.
"""
from __future__ import annotations

import ctypes as C
from pathlib import Path

import torch

LIB_PATH = Path(__file__).resolve().parent / "libcgym_b200.so"

F32, BF16, E4M3 = 0, 1, 2
STATUS_PAGE_POOL_EXHAUSTED, STATUS_BAD_PAGE, STATUS_WAIT_TIMEOUT, STATUS_CAPACITY = 1, 2, 4, 8

_DTYPE_CODES = {torch.float32: F32, torch.bfloat16: BF16, torch.float8_e4m3fn: E4M3, torch.uint8: E4M3}


class NativeLibraryError(RuntimeError):
    pass


class NativeKernelError(RuntimeError):
    pass


class KVLayout(C.Structure):
    _fields_ = [("kv_pool", C.c_void_p), ("kv_scales", C.c_void_p), ("block_table", C.c_void_p),
                ("n_pages", C.c_int32), ("page_size", C.c_int32), ("max_blocks", C.c_int32),
                ("n_kv_heads", C.c_int32), ("head_dim", C.c_int32), ("kv_dtype", C.c_int32)]


class PagePool(C.Structure):
    _fields_ = [("free_bitmap", C.c_void_p), ("refcount", C.c_void_p), ("block_table", C.c_void_p),
                ("n_blocks", C.c_void_p), ("n_pages", C.c_int32), ("page_size", C.c_int32),
                ("max_blocks", C.c_int32), ("n_slots", C.c_int32)]


class SlotState(C.Structure):
    _fields_ = [("tokens", C.c_void_p), ("logprobs", C.c_void_p), ("lengths", C.c_void_p),
                ("limits", C.c_void_p), ("reasons", C.c_void_p), ("alive", C.c_void_p),
                ("pending", C.c_void_p), ("input_tokens", C.c_void_p), ("stop_states", C.c_void_p),
                ("stop_offsets", C.c_void_p), ("stop_table", C.c_void_p), ("ignore_eos", C.c_void_p),
                ("rng_positions", C.c_void_p), ("seeds", C.c_void_p), ("temperatures", C.c_void_p),
                ("rng_offsets", C.c_void_p), ("force_eos_at", C.c_void_p), ("seq_lens", C.c_void_p),
                ("min_logits", C.c_void_p), ("gumbel_noise", C.c_void_p), ("out_rows", C.c_void_p),
                ("capacity", C.c_int32),
                ("eos_token_id", C.c_int32)]


class AdmitQueue(C.Structure):
    _fields_ = [("rows", C.c_void_p), ("requests", C.c_void_p), ("limits", C.c_void_p), ("seeds", C.c_void_p),
                ("temperatures", C.c_void_p), ("ignore_eos", C.c_void_p), ("stop_offsets", C.c_void_p),
                ("logits", C.c_void_p), ("head", C.c_void_p), ("tail", C.c_void_p), ("capacity", C.c_int32),
                ("result_capacity", C.c_int32), ("result_lengths", C.c_void_p), ("result_reasons", C.c_void_p),
                ("slot_requests", C.c_void_p), ("out_rows", C.c_void_p), ("adopt_rows", C.c_void_p),
                ("adopt_entries", C.c_void_p), ("release_mask", C.c_void_p)]


_P, _I, _F, _L = C.c_void_p, C.c_int, C.c_float, C.c_int64

# name -> argument types (all return int); must mirror include/cgym_b200.h
SIGNATURES = {
    "cgym_embedding": [_P, _P, _P, _I, _I, _I, _I, _P],
    "cgym_rmsnorm": [_P, _P, _P, _P, _P, _I, _I, _F, _I, _P],
    "cgym_rmsnorm_quant": [_P, _P, _P, _P, _P, _P, _I, _I, _F, _P],
    "cgym_swiglu": [_P, _P, _I, _I, _I, _P],
    "cgym_swiglu_quant": [_P, _P, _P, _I, _I, _P],
    "cgym_quantize_rows": [_P, _P, _P, _I, _I, _I, _P],
    "cgym_conv_update": [_P, _P, _P, _P, _P, _P, _I, _I, _I, _P],
    "cgym_conv_prefill": [_P, _P, _P, _P, _P, _P, _P, _I, _I, _I, _I, _P],
    "cgym_qk_norm_rope_append": [_P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P, C.POINTER(KVLayout), _I, _I, _I,
                                 _F, _I, _P, _P],
    "cgym_paged_attention": [_P, _P, _P, _P, _P, C.POINTER(KVLayout), _I, _I, _I, _F, _I, _P, _I, _I, _P, _P],
    "cgym_prefill_attention": [_P, _P, _P, _P, _P, _P, C.POINTER(KVLayout), _I, _I, _I, _F, _I, _P, _P],
    "cgym_scatter_kv_dense": [_P, _P, C.POINTER(KVLayout), _I, _I, _I, _I, _P],
    "cgym_gemm": [_P, _P, _P, _P, _I, _I, _I, _I, _I, _P, _L, _P, _P],
    "cgym_gemm_fp8": [_P, _P, _P, _P, _P, _P, _I, _I, _I, _I, _P, _L, _P, _P],
    "cgym_gemm_scatter": [_P, _P, _P, _P, _P, _I, _I, _I, _I, _I, _P, _L, _P, _P],
    "cgym_gemm_plan": [_I, _I, _I, _I, _I, _I, _P],
    "cgym_gemm_fp8_scatter": [_P, _P, _P, _P, _P, _P, _P, _I, _I, _I, _I, _P, _L, _P, _P],
    "cgym_bf16_stream_pack": [_P, _P, _P, _L, _I, _P],
    "cgym_bf16_stream_unpack": [_P, _P, _P, _P, _L, _I, _P],
    "cgym_bf16_stream_gemv": [_P, _P, _P, _P, _P, _P, _I, _I, _I, _P],
    "cgym_slot_turnover": [C.POINTER(PagePool), _I, C.POINTER(SlotState), C.POINTER(AdmitQueue), _P, _P, _P, _I, _I, _I,
                           _I, _P],
    "cgym_step_begin_rows": [C.POINTER(PagePool), _P, _P, _P, _P, _P, _P, _P, _P, _P, _I, _I, _P, _P],
    "cgym_sample_record": [_P, C.POINTER(SlotState), _P, _P, _P, _I, _I, _I, _P, _P],
    "cgym_sample": [_P, _P, _P, _P, _P, _P, _P, _I, _I, _I, _P, _P],
    "cgym_gumbel_noise": [_P, C.POINTER(SlotState), _I, _I, _P],
    "cgym_sample_static": [_P, _P, _P, _P, _P, _P, _P, _I, _I, _I, _P],
    "cgym_filter_thresholds": [_P, _P, _P, _P, _P, _P, _I, _I, _I, _P],
    "cgym_topk_head": [_P, _P, _P, _P, _P, _I, _I, _I, _I, _I, _P],
    "cgym_repetition_penalty": [_P, _P, _P, _P, _P, _P, _P, _I, _I, _I, _I, _P],
    "cgym_target_logprobs": [_P, _P, _P, _I, _I, _I, _P],
    "cgym_step_begin": [C.POINTER(PagePool), _P, _P, _P, _P, _P, _P, _I, _P, _P],
    "cgym_pages_reserve": [C.POINTER(PagePool), _P, _P, _I, _P, _P],
    "cgym_pages_release": [C.POINTER(PagePool), _P, _P, _P],
    "cgym_pages_fork": [C.POINTER(PagePool), C.POINTER(KVLayout), _I, _P, _P, _P, _I, _P, _P],
    "cgym_gather_kv_dense": [_P, C.POINTER(KVLayout), _I, _I, _I, _I, _P],
}
PLAIN = {"cgym_last_error": ([], C.c_char_p), "cgym_version": ([], _I), "cgym_device_supported": ([], _I),
         "cgym_launch_count": ([], C.c_longlong), "cgym_sample_workspace_bytes": ([_I], C.c_int64),
         "cgym_set_pdl": ([_I], _I), "cgym_test_gemm_wait": ([C.c_ulonglong, _I], _I)}

_lib = None


def load() -> C.CDLL:
    global _lib
    if _lib is not None:
        return _lib
    if not LIB_PATH.exists():
        raise NativeLibraryError(
            f"{LIB_PATH} is missing: build the sm_100a kernels with `python -m climbing_gym_b200.build`; "
            "there is no fallback path")
    lib = C.CDLL(str(LIB_PATH))
    for name, args in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.argtypes, fn.restype = args, _I
    for name, (args, res) in PLAIN.items():
        fn = getattr(lib, name)
        fn.argtypes, fn.restype = args, res
    _lib = lib
    return lib


def exported_symbols() -> list[str]:
    return sorted([*SIGNATURES, *PLAIN])


def ptr(t):
    """Device pointer of a tensor (None -> NULL)."""
    return None if t is None else t.data_ptr()


def dtype_code(dtype: torch.dtype) -> int:
    try:
        return _DTYPE_CODES[dtype]
    except KeyError as exc:
        raise ValueError(f"unsupported dtype for the native kernels: {dtype}") from exc


def stream_ptr(device=None) -> int:
    return torch.cuda.current_stream(device).cuda_stream


_graph_kernels = 0


def note_graph_replay(kernels: int) -> None:
    """A captured graph with ``kernels`` of this library's kernels was replayed once."""
    global _graph_kernels
    _graph_kernels += kernels


def launch_count() -> int:
    """Kernels of this library launched so far: direct launches plus kernels inside graph replays."""
    return int(load().cgym_launch_count()) + _graph_kernels


def call(name: str, *args) -> None:
    lib = load()
    rc = getattr(lib, name)(*args)
    if rc != 0:
        raise NativeKernelError(f"{name}: {lib.cgym_last_error().decode()}")
