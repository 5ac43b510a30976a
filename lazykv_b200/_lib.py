"""ctypes binding of liblkv_sm100.so (the C ABI declared in include/lkv.h).

The library is loaded from this package directory and must have been built for sm_100a
(`python -m lazykv_b200.build`). There is no fallback: if it is missing or a call fails, the
caller gets an exception carrying the library's own message.
"""

from __future__ import annotations

import ctypes
from ctypes import c_char_p, c_float, c_int, c_int64, c_size_t, c_void_p
from pathlib import Path

import torch

LIB_PATH = Path(__file__).resolve().parent / "liblkv_sm100.so"

LKV_F32, LKV_BF16 = 0, 1
LKV_COLD_INT8, LKV_COLD_PAIRS = 0, 1
LKV_ORDER_BOUND, LKV_ORDER_BLOCK = 0, 1
LKV_DEBUG_SELECT_WAIT_ITERS, LKV_DEBUG_SELECT_STALL_NEXT, LKV_DEBUG_EXCHANGE_WAIT_ITERS = 1, 2, 3
LKV_DEV_WAIT_TIMEOUT, LKV_DEV_LIST_OVERFLOW = 1, 2

_lib: ctypes.CDLL | None = None

# name -> (restype, argtypes); every entry point of include/lkv.h.
SIGNATURES: dict[str, tuple[object, list[object]]] = {
    "lkv_version": (c_char_p, []),
    "lkv_last_error": (c_size_t, [c_char_p, c_size_t]),
    "lkv_packed_pair_bytes": (c_int64, [c_int, c_int]),
    "lkv_block_minmax": (c_int, [c_void_p, c_int, c_int, c_int, c_int, c_int, c_int64, c_int64, c_int64, c_void_p, c_void_p, c_int64, c_int, c_void_p]),
    "lkv_pack_int8": (c_int, [c_void_p, c_int, c_int, c_int, c_int, c_int, c_void_p, c_void_p, c_void_p, c_int64, c_int, c_void_p, c_void_p]),
    "lkv_unpack_int8": (c_int, [c_void_p, c_int64, c_int, c_int, c_void_p, c_int, c_void_p]),
    "lkv_fetch_pairs": (c_int, [c_void_p, c_int, c_void_p, c_void_p, c_void_p, c_int64, c_int, c_int, c_int, c_void_p]),
    "lkv_quest_topk_workspace": (c_size_t, [c_int, c_int]),
    "lkv_quest_topk": (c_int, [c_void_p, c_int, c_int, c_int, c_int, c_void_p, c_void_p, c_int, c_int64, c_int, c_int, c_int, c_int, c_int, c_void_p, c_int, c_void_p, c_void_p, c_int, c_void_p, c_size_t, c_void_p]),
    "lkv_quest_topk_noalloc": (c_int, [c_void_p, c_int, c_int, c_int, c_int, c_void_p, c_void_p, c_int, c_int64, c_int, c_int, c_int, c_int, c_int, c_void_p, c_int, c_void_p, c_void_p, c_int, c_void_p]),
    "lkv_attention_workspace": (c_size_t, [c_int, c_int, c_int, c_int]),
    "lkv_shard_plan": (c_int, [c_int, c_int, c_int, c_int, c_void_p]),
    "lkv_topk_merge_workspace": (c_size_t, [c_int, c_int]),
    "lkv_topk_merge": (c_int, [c_void_p, c_void_p, c_int, c_int, c_int64, c_int, c_int, c_int, c_void_p, c_int, c_void_p, c_int, c_void_p, c_size_t, c_void_p]),
    "lkv_exchange_region_bytes": (c_size_t, [c_int, c_int, c_int]),
    "lkv_exchange_alloc": (c_int, [c_int, c_int, c_int, c_void_p, c_void_p]),
    "lkv_exchange_open": (c_int, [c_void_p, c_void_p]),
    "lkv_exchange_close": (c_int, [c_void_p]),
    "lkv_exchange_free": (c_int, [c_void_p]),
    "lkv_exchange_merge": (c_int, [c_void_p, c_void_p, c_int, c_int, c_int, c_int, c_void_p, c_void_p, c_int, c_void_p, c_void_p]),
    "lkv_quest_topk_resident": (c_int, [c_void_p, c_int, c_int, c_int, c_int, c_void_p, c_void_p, c_int, c_int64, c_int, c_int, c_int, c_int, c_void_p, c_int,
                                        c_void_p, c_int, c_void_p, c_int64, c_void_p, c_int, c_void_p, c_size_t, c_void_p]),
    "lkv_quest_bounds": (c_int, [c_void_p, c_int, c_int, c_int, c_int, c_void_p, c_void_p, c_int, c_int64, c_int, c_int, c_int, c_void_p, c_int, c_int64, c_void_p]),
    "lkv_topk_gathered": (c_int, [c_void_p, c_int, c_int, c_int, c_int64, c_void_p, c_int, c_int, c_int, c_void_p, c_int, c_int, c_void_p, c_int, c_void_p]),
    "lkv_topk_gathered_resident": (c_int, [c_void_p, c_int, c_int, c_int, c_int64, c_void_p, c_int, c_int, c_int, c_void_p, c_int, c_int, c_void_p, c_int,
                                           c_void_p, c_int, c_void_p, c_int64, c_void_p]),
    "lkv_hot_attention": (c_int, [c_void_p, c_int, c_int, c_int, c_int, c_void_p, c_void_p, c_int, c_int64, c_int64, c_int64, c_int64, c_void_p, c_int, c_void_p, c_int64, c_int, c_float, c_void_p, c_void_p, c_void_p, c_size_t, c_void_p]),
    "lkv_cold_attention": (c_int, [c_void_p, c_int, c_int, c_int, c_int, c_void_p, c_int, c_int, c_int, c_int, c_void_p, c_int, c_float, c_void_p, c_void_p, c_void_p, c_size_t, c_void_p]),
    "lkv_lse_merge_packed": (c_int, [c_void_p, c_int, c_int64, c_int, c_void_p, c_int, c_void_p, c_void_p]),
    "lkv_lse_merge": (c_int, [c_void_p, c_void_p, c_int, c_int64, c_int, c_void_p, c_int, c_void_p, c_void_p]),
    "lkv_exact_attention_workspace": (c_size_t, [c_int, c_int, c_int, c_int, c_int]),
    "lkv_exact_attention": (c_int, [c_void_p, c_int, c_int, c_int, c_int, c_void_p, c_void_p, c_float, c_void_p, c_int, c_void_p, c_void_p, c_void_p, c_void_p, c_size_t, c_void_p]),
    "lkv_device_status": (c_int, [c_void_p, c_int]),
    "lkv_status_attach": (c_int, []),
    "lkv_status_poll": (c_int, [c_void_p, c_int]),
    "lkv_debug_set": (c_int, [c_int, c_int64]),
    "lkv_ragged_topk_workspace": (c_size_t, [c_int, c_int]),
    "lkv_ragged_quest_topk": (c_int, [c_void_p, c_int, c_int, c_int, c_int, c_int, c_void_p, c_void_p, c_int, c_int64, c_int64, c_void_p, c_int64,
                                      c_void_p, c_int, c_void_p, c_int, c_int, c_void_p, c_int64, c_void_p, c_int, c_void_p, c_size_t, c_void_p]),
    "lkv_ragged_schedule": (c_int, [c_void_p, c_int, c_int, c_void_p, c_int, c_void_p]),
    "lkv_ragged_attention_workspace": (c_size_t, [c_int, c_int]),
    "lkv_ragged_exact_attention": (c_int, [c_void_p, c_int, c_int, c_int, c_int, c_int, c_void_p, c_void_p, c_int64, c_void_p, c_int64, c_void_p, c_int,
                                           c_void_p, c_void_p, c_int, c_int, c_float, c_void_p, c_int, c_void_p, c_void_p, c_size_t, c_void_p]),
    "lkv_tier_admit": (c_int, [c_void_p, c_int, c_int, c_int64, c_void_p, c_int, c_void_p, c_void_p, c_int, c_void_p, c_int64, c_void_p, c_int,
                               c_void_p, c_int, c_int, c_int, c_void_p, c_void_p, c_void_p, c_void_p, c_int64, c_void_p, c_void_p]),
    "lkv_quest_topk_admit": (c_int, [c_void_p, c_int, c_int, c_int, c_int, c_void_p, c_void_p, c_int, c_int64, c_int, c_int, c_int, c_int, c_void_p, c_int,
                                     c_void_p, c_void_p, c_int, c_void_p, c_size_t, c_void_p, c_int, c_void_p, c_void_p, c_int, c_void_p, c_int64,
                                     c_void_p, c_int, c_void_p, c_int, c_int, c_void_p, c_void_p, c_void_p, c_void_p, c_int64, c_void_p, c_void_p]),
    "lkv_mark_blocks": (c_int, [c_void_p, c_int, c_int, c_int64, c_void_p, c_int, c_void_p]),
    "lkv_split_events_create": (c_int, [c_void_p]),
    "lkv_split_events_destroy": (c_int, [c_void_p]),
    "lkv_split_step": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p]),
    "lkv_split_join": (c_int, [c_void_p, c_void_p]),
    "lkv_split_wait": (c_int, [c_void_p]),
    "lkv_append_tokens": (c_int, [c_void_p, c_int64, c_int64, c_void_p, c_int64, c_int64, c_int, c_int, c_int, c_int, c_void_p, c_int, c_int, c_void_p]),
    "lkv_ragged_stage_records": (c_int, [c_void_p, c_int64, c_int, c_int, c_void_p, c_int64, c_void_p, c_int, c_void_p, c_void_p, c_int, c_void_p,
                                         c_int64, c_void_p, c_void_p, c_int64, c_void_p]),
}


class HotSet(ctypes.Structure):
    """lkv_hot_set of include/lkv.h."""

    _fields_ = [("k_base", c_void_p), ("v_base", c_void_p), ("dtype", c_int), ("s_row", c_int64), ("s_head", c_int64), ("s_tok", c_int64),
                ("blocks", c_void_p), ("n_list", c_int), ("slot_of", c_void_p), ("slot_stride", c_int64), ("last_fill", c_int),
                ("n_rows", c_int64)]


class ColdSet(ctypes.Structure):
    """lkv_cold_set of include/lkv.h."""

    _fields_ = [("store", c_void_p), ("kind", c_int), ("first_block", c_int), ("n_blocks", c_int), ("excluded", c_void_p), ("bitmap_words", c_int)]


class SplitStepArgs(ctypes.Structure):
    """lkv_split_step_args of include/lkv.h (same fields, same order)."""

    _fields_ = [("q", c_void_p), ("q_dtype", c_int), ("hq", c_int), ("h", c_int), ("d", c_int), ("kmin", c_void_p), ("kmax", c_void_p),
                ("meta_dtype", c_int), ("m_head", c_int64), ("first_block", c_int), ("n_cand", c_int), ("k", c_int), ("bound_mode", c_int),
                ("chosen", c_void_p), ("chosen_ld", c_int), ("block_slot", c_void_p), ("cap", c_int), ("hot", c_void_p), ("hot_ld", c_int64),
                ("bitmap", c_void_p), ("bitmap_words", c_int), ("sel_workspace", c_void_p), ("sel_workspace_bytes", c_size_t), ("bs", c_int),
                ("hot_set", c_void_p), ("cold_set", c_void_p), ("scale", ctypes.c_float), ("out", c_void_p), ("out_dtype", c_int),
                ("lse", c_void_p), ("att_workspace", c_void_p), ("att_workspace_bytes", c_size_t), ("slot_block", c_void_p),
                ("last_used", c_void_p), ("n_slots", c_int), ("evicted_at", c_void_p), ("step", c_int64), ("store", c_void_p),
                ("store_kind", c_int), ("pool", c_void_p), ("pool_dtype", c_int), ("miss_blk", c_void_p), ("miss_slot", c_void_p),
                ("n_miss", c_void_p), ("miss_total", c_void_p), ("selected", c_int)]


class LkvError(RuntimeError):
    """A non-zero status from liblkv_sm100.so, with the library's message."""


def lib() -> ctypes.CDLL:
    """The loaded library; raises if it has not been built."""
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise RuntimeError(f"{LIB_PATH.name} is not built; run `python -m lazykv_b200.build` (needs nvcc, targets sm_100a)")
        handle = ctypes.CDLL(str(LIB_PATH))
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(handle, name)
            fn.restype = res
            fn.argtypes = args
        _lib = handle
    return _lib


def last_error() -> str:
    buf = ctypes.create_string_buffer(512)
    lib().lkv_last_error(buf, 512)
    return buf.value.decode()


def call(name: str, *args: object) -> None:
    """Call an lkv_* entry point returning a status; raise LkvError on failure."""
    rc = getattr(lib(), name)(*args)
    if rc != 0:
        raise LkvError(f"{name} failed ({rc}): {last_error()}")


def ptr(t: torch.Tensor | None) -> int | None:
    """Raw address of a tensor's first element (None for None)."""
    return None if t is None else t.data_ptr()


_RAW_STREAM = getattr(torch._C, "_cuda_getCurrentRawStream", None)  # torch's own fast accessor, where it has one


def stream_handle(device: torch.device | None = None) -> int:
    """The raw handle of torch's current stream on `device` (the current device by default)."""
    if device is None or _RAW_STREAM is None:
        return torch.cuda.current_stream(device).cuda_stream
    idx = device.index if isinstance(device, torch.device) else int(device)
    return _RAW_STREAM(torch.cuda.current_device() if idx is None else idx)


def dtype_code(dt: torch.dtype) -> int:
    if dt == torch.bfloat16:
        return LKV_BF16
    if dt == torch.float32:
        return LKV_F32
    raise ValueError(f"unsupported dtype {dt}; the kernels take bfloat16 or float32")


def require_cuda(*tensors: torch.Tensor) -> torch.device:
    """The kernels run on CUDA tensors only: there is no CPU path."""
    for t in tensors:
        if t is not None and not t.is_cuda:
            raise ValueError("lazykv_b200 computes on CUDA tensors; got a CPU tensor (there is no CPU fallback)")
    return next(t.device for t in tensors if t is not None)
