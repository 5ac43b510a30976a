"""torch-facing wrappers of the C ABI: shape checks, output allocation and a per-device workspace.

Each function launches on the current CUDA stream and never synchronises. Inputs must be CUDA
tensors (or device views of pinned host memory); there is no CPU path.
"""

from __future__ import annotations

import ctypes
import math

import torch

from lazykv_b200 import _lib as L
from lazykv_b200._lib import call, dtype_code, ptr, require_cuda, stream_handle

_WS: dict[tuple[int, int], torch.Tensor] = {}


def workspace(device: torch.device, nbytes: int, slot: int = 0) -> torch.Tensor:
    """A reusable device buffer of at least `nbytes` (grown on demand), one per (device, slot).

    Calls on one stream run in order, so reusing the buffer between them is safe; work on another
    stream must use another slot.
    """
    key = (device.index if device.index is not None else torch.cuda.current_device(), slot)
    buf = _WS.get(key)
    if buf is None or buf.numel() < nbytes:
        # Zeroed once: the selection keeps counters at the start of its workspace that must read
        # zero on entry and that its kernels leave zero.
        buf = torch.zeros(max(nbytes, 1 << 20), dtype=torch.uint8, device=device)
        _WS[key] = buf
    return buf


def current_workspace(device: torch.device, slot: int = 0) -> torch.Tensor | None:
    """The buffer workspace() would hand out now for (device, slot), without growing it (None if
    there is none yet): a caller holding an earlier buffer compares identities to see a regrowth."""
    return _WS.get((device.index if device.index is not None else torch.cuda.current_device(), slot))


def packed_pair_bytes(block_size: int, head_dim: int) -> int:
    return int(L.lib().lkv_packed_pair_bytes(block_size, head_dim))


def block_minmax(keys: torch.Tensor, block_size: int, kmin: torch.Tensor, kmax: torch.Tensor, first_block: int = 0) -> None:
    """kmin/kmax[j, first_block + b] = channel min/max of block b of `keys`: [h, n*bs, d] or
    [h, n, bs, d] (any strides; the 4-D form reads blocks that are not evenly spaced tokens, such as
    the keys of a store in its [n, h, 2, bs, d] layout)."""
    require_cuda(keys, kmin, kmax)
    if keys.dim() == 4:
        h, n, bs, d = keys.shape
        if bs != block_size:
            raise ValueError(f"block_minmax: blocks of {bs} tokens, block_size {block_size}")
        s_head, s_blk, s_tok = keys.stride(0), keys.stride(1), keys.stride(2)
    else:
        h, t, d = keys.shape
        n = t // block_size
        s_head, s_tok = keys.stride(0), keys.stride(1)
        s_blk = block_size * s_tok
    if kmin.shape[-1] != d or kmin.dtype != keys.dtype or kmax.dtype != keys.dtype or kmin.stride(-1) != 1 or keys.stride(-1) != 1:
        raise ValueError("block_minmax: metadata must be [h, cap, d] in the keys' dtype, contiguous in d")
    call("lkv_block_minmax", ptr(keys), dtype_code(keys.dtype), h, n, block_size, d, s_head, s_blk, s_tok,
         ptr(kmin), ptr(kmax), kmin.stride(-3) if kmin.dim() >= 3 else kmin.shape[-2] * d, first_block, stream_handle(keys.device))


def pack_int8(pairs: torch.Tensor, records: torch.Tensor | None = None, kmin: torch.Tensor | None = None, kmax: torch.Tensor | None = None,
              first_block: int = 0, deq: torch.Tensor | None = None) -> torch.Tensor:
    """Records [n, h, W] for pairs [n, h, 2, bs, d]; optionally metadata and dequantised pairs.

    kmin/kmax, when given, are [h, cap, d] in the pairs' dtype (written at first_block + b).
    """
    require_cuda(pairs)
    n, h, two, bs, d = pairs.shape
    if two != 2:
        raise ValueError(f"expected a [..., 2, block_size, head_dim] KV pair, got {tuple(pairs.shape)}")
    pairs = pairs.contiguous()
    w = packed_pair_bytes(bs, d)
    if records is None:
        records = torch.empty((n, h, w), dtype=torch.uint8, device=pairs.device)
    m_head = 0 if kmin is None else kmin.stride(-3)
    call("lkv_pack_int8", ptr(pairs), dtype_code(pairs.dtype), n, h, bs, d, ptr(records), ptr(kmin), ptr(kmax), m_head, first_block,
         ptr(deq), stream_handle(pairs.device))
    return records


def unpack_int8(records: torch.Tensor, block_size: int, head_dim: int, dtype: torch.dtype) -> torch.Tensor:
    """[m, W] uint8 records -> [m, 2, bs, d] in `dtype`, bit-exact with the reference's unpack."""
    require_cuda(records)
    out = torch.empty((records.shape[0], 2, block_size, head_dim), dtype=dtype, device=records.device)
    if records.shape[0]:
        call("lkv_unpack_int8", ptr(records.contiguous()), records.shape[0], block_size, head_dim, ptr(out), dtype_code(dtype),
             stream_handle(records.device))
    return out


def fetch_pairs(src: torch.Tensor, src_rows: torch.Tensor, dst: torch.Tensor, dst_rows: torch.Tensor, block_size: int, head_dim: int) -> None:
    """dst row dst_rows[i] <- src row src_rows[i]; int8 records are dequantised into dst's dtype."""
    kind = L.LKV_COLD_INT8 if src.dtype == torch.uint8 else L.LKV_COLD_PAIRS
    n = src_rows.numel()
    if n == 0:
        return
    call("lkv_fetch_pairs", ptr(src), kind, ptr(src_rows), ptr(dst), ptr(dst_rows), n, block_size, head_dim, dtype_code(dst.dtype),
         stream_handle(dst.device))


def quest_topk(query: torch.Tensor, kmin: torch.Tensor, kmax: torch.Tensor, first_block: int, n_cand: int, k: int,
               bound_dtype: torch.dtype | None = None, out_blocks: torch.Tensor | None = None, want_bound: bool = False,
               bitmap: torch.Tensor | None = None, ws_slot: int = 1, by_block: bool = False) -> tuple[torch.Tensor, torch.Tensor | None]:
    """Top-k block ids [h, k] (int32) over candidates [first_block, first_block + n_cand) of
    metadata [h, cap, d]: descending bound with ties to the lower id, or ascending id when
    `by_block` (the same set, no sort); optionally the bounds [h, n_cand].

    Its workspace (slot 1 by default) keeps zeroed counters between calls, so it is never shared
    with the attention calls' workspace (slot 0)."""
    dev = require_cuda(query, kmin, kmax)
    hq, d = query.shape[-3] if query.dim() == 4 else query.shape[0], query.shape[-1]
    q = query.reshape(hq, d).contiguous()
    h = kmin.shape[-3]
    bound_dtype = bound_dtype or q.dtype
    if out_blocks is None:
        out_blocks = torch.empty((h, k), dtype=torch.int32, device=dev)
    if out_blocks.stride(-1) != 1 or out_blocks.shape[-1] < k:
        raise ValueError("quest_topk: out_blocks must be [h, >=k] int32 with unit column stride")
    bound = torch.empty((h, n_cand), dtype=torch.float32, device=dev) if want_bound else None
    nbytes = int(L.lib().lkv_quest_topk_workspace(h, n_cand))
    ws = workspace(dev, nbytes, ws_slot)
    words = 0 if bitmap is None else bitmap.shape[-1]
    call("lkv_quest_topk", ptr(q), dtype_code(q.dtype), hq, h, d, ptr(kmin), ptr(kmax), dtype_code(kmin.dtype), kmin.stride(-3),
         first_block, n_cand, k, dtype_code(bound_dtype), L.LKV_ORDER_BLOCK if by_block else L.LKV_ORDER_BOUND, ptr(out_blocks),
         out_blocks.stride(0), ptr(bound), ptr(bitmap), words, ptr(ws), ws.numel(),
         stream_handle(dev))
    return out_blocks, bound


def quest_topk_resident(query: torch.Tensor, kmin: torch.Tensor, kmax: torch.Tensor, first_block: int, n_cand: int, k: int,
                        out_blocks: torch.Tensor, block_slot: torch.Tensor, hot: torch.Tensor, bitmap: torch.Tensor,
                        bound_dtype: torch.dtype | None = None, ws_slot: int = 1) -> torch.Tensor:
    """The selection (block order) for an attention before the admit: out_blocks [h, k] the chosen
    ids, hot [h, >= k] (a view, unit column stride) each chosen block's current slot or -1, and the
    bitmap of the resident chosen blocks only (lkv_quest_topk_resident)."""
    dev = require_cuda(query, kmin, kmax, out_blocks, block_slot, hot, bitmap)
    hq, d = query.shape[-3] if query.dim() == 4 else query.shape[0], query.shape[-1]
    q = query.reshape(hq, d).contiguous()
    h = kmin.shape[-3]
    bound_dtype = bound_dtype or q.dtype
    if hot.stride(-1) != 1 or hot.shape[-1] < k or block_slot.stride(-1) != 1 or not block_slot.is_contiguous():
        raise ValueError("quest_topk_resident: hot must be [h, >=k] with unit column stride and block_slot contiguous [h, cap]")
    ws = workspace(dev, int(L.lib().lkv_quest_topk_workspace(h, n_cand)), ws_slot)
    call("lkv_quest_topk_resident", ptr(q), dtype_code(q.dtype), hq, h, d, ptr(kmin), ptr(kmax), dtype_code(kmin.dtype), kmin.stride(-3), first_block,
         n_cand, k, dtype_code(bound_dtype), ptr(out_blocks), out_blocks.stride(0), ptr(block_slot), block_slot.shape[-1], ptr(hot), hot.stride(0),
         ptr(bitmap), bitmap.shape[-1], ptr(ws), ws.numel(), stream_handle(dev))
    return out_blocks


def quest_bounds(query: torch.Tensor, kmin: torch.Tensor, kmax: torch.Tensor, first_block: int, n_cand: int, out: torch.Tensor,
                 bound_dtype: torch.dtype | None = None) -> torch.Tensor:
    """The Quest bound of candidates [first_block, first_block + n_cand) into out [h, >= n_cand]
    (bf16 or float32; bf16 only with bf16 bounds), ranked as quest_topk ranks them; nothing else."""
    dev = require_cuda(query, kmin, kmax, out)
    hq, d = query.shape[-3] if query.dim() == 4 else query.shape[0], query.shape[-1]
    q = query.reshape(hq, d).contiguous()
    h = kmin.shape[-3]
    bound_dtype = bound_dtype or q.dtype
    if out.dim() != 2 or out.shape[0] != h or out.shape[1] < n_cand or out.stride(-1) != 1:
        raise ValueError(f"quest_bounds: out must be [{h}, >={n_cand}] with unit column stride, got {tuple(out.shape)}")
    call("lkv_quest_bounds", ptr(q), dtype_code(q.dtype), hq, h, d, ptr(kmin), ptr(kmax), dtype_code(kmin.dtype), kmin.stride(-3), first_block,
         n_cand, dtype_code(bound_dtype), ptr(out), dtype_code(out.dtype), out.stride(0), stream_handle(dev))
    return out


def topk_gathered(gathered: torch.Tensor, seg_n: list[int], k: int, rank: int, out_base: int, out: torch.Tensor,
                  bitmap: torch.Tensor | None = None, out_cols: int | None = None, block_slot: torch.Tensor | None = None,
                  hot: torch.Tensor | None = None) -> torch.Tensor:
    """Rank `rank`'s part of the global top-k over every rank's bounds gathered as [world, h, ld]
    (rank r holding seg_n[r] candidates after rank r-1's): out [h, >= out_cols] gets the chosen local
    ids (out_base + index in the rank), ascending, then -1; the bitmap those ids. With `block_slot`
    [h, cap] and `hot` [h, >= out_cols] (the resident split, lkv_topk_gathered_resident): hot gets
    each chosen block's current slot or -1, and the bitmap marks only the resident ones."""
    import ctypes

    dev = require_cuda(gathered, out)
    world, h, ld = gathered.shape
    if len(seg_n) != world or gathered.stride(-1) != 1 or not gathered.is_contiguous():
        raise ValueError("topk_gathered: gathered must be a contiguous [world, h, ld] with one count per rank")
    out_cols = out.shape[-1] if out_cols is None else out_cols
    counts = (ctypes.c_int32 * world)(*seg_n)
    words = 0 if bitmap is None else bitmap.shape[-1]
    if block_slot is None:
        call("lkv_topk_gathered", ptr(gathered), dtype_code(gathered.dtype), world, h, ld, ctypes.cast(counts, ctypes.c_void_p), k, rank, out_base,
             ptr(out), out.stride(0), out_cols, ptr(bitmap), words, stream_handle(dev))
    else:
        if hot is None or hot.stride(-1) != 1 or not block_slot.is_contiguous():
            raise ValueError("topk_gathered: the resident split needs hot [h, >=out_cols] (unit column stride) and a contiguous block_slot")
        call("lkv_topk_gathered_resident", ptr(gathered), dtype_code(gathered.dtype), world, h, ld, ctypes.cast(counts, ctypes.c_void_p), k, rank,
             out_base, ptr(out), out.stride(0), out_cols, ptr(bitmap), words, ptr(block_slot), block_slot.shape[-1], ptr(hot), hot.stride(0),
             stream_handle(dev))
    return out


def attention_workspace_bytes(h: int, hq: int, d: int, n_items: int) -> int:
    return int(L.lib().lkv_attention_workspace(h, hq, d, n_items))


def storage_rows(k_base: torch.Tensor, v_base: torch.Tensor, strides: tuple[int, int, int], h: int, block_size: int, d: int) -> int:
    """Storage rows addressable through (s_row, s_head, s_tok) for KV heads 0..h-1 inside both
    tensors' storage: the bound of the tensor-map loads (0 when not even one row fits)."""
    s_row, s_head, s_tok = strides
    reach = (h - 1) * s_head + (block_size - 1) * s_tok + d  # elements one row spans past its start
    rows = []
    for t in (k_base, v_base):
        avail = t.untyped_storage().nbytes() // t.element_size() - t.storage_offset()
        rows.append(0 if avail < reach else (avail - reach) // s_row + 1)
    return max(0, min(rows))


def hot_attention(query: torch.Tensor, k_base: torch.Tensor, v_base: torch.Tensor, strides: tuple[int, int, int], blocks: torch.Tensor,
                  last_fill: int, scale: float, block_size: int, slot_of: torch.Tensor | None = None, out: torch.Tensor | None = None,
                  lse: torch.Tensor | None = None, ws_slot: int = 0) -> tuple[torch.Tensor, torch.Tensor]:
    """Attention of query [hq, d] over, per KV head j, the blocks listed in blocks[j] (int32 [h, n]).

    Block b of head j is storage row slot_of[j, b] (or b), its key (t, c) at
    k_base[row*s_row + j*s_head + t*s_tok + c]; the last listed block has `last_fill` live tokens.
    Returns float32 (out [hq, d], lse [hq]).
    """
    dev = require_cuda(query, k_base, v_base, blocks)
    hq, d = query.shape[-3] if query.dim() == 4 else query.shape[0], query.shape[-1]
    q = query.reshape(hq, d).contiguous()
    h, n = blocks.shape
    out = torch.empty((hq, d), dtype=torch.float32, device=dev) if out is None else out
    lse = torch.empty((hq,), dtype=torch.float32, device=dev) if lse is None else lse
    ws = workspace(dev, attention_workspace_bytes(h, hq, d, n), ws_slot)
    s_row, s_head, s_tok = strides
    n_rows = storage_rows(k_base, v_base, strides, h, block_size, d)
    call("lkv_hot_attention", ptr(q), hq, h, d, block_size, ptr(k_base), ptr(v_base), dtype_code(k_base.dtype), s_row, s_head, s_tok, n_rows,
         ptr(blocks), n, ptr(slot_of), 0 if slot_of is None else slot_of.stride(0), last_fill, scale, ptr(out), ptr(lse), ptr(ws), ws.numel(),
         stream_handle(dev))
    return out, lse


def cold_attention(query: torch.Tensor, cold: torch.Tensor, block_size: int, first_block: int, n_blocks: int, scale: float,
                   excluded: torch.Tensor | None = None, dtype: torch.dtype | None = None, out: torch.Tensor | None = None,
                   lse: torch.Tensor | None = None, ws_slot: int = 0) -> tuple[torch.Tensor, torch.Tensor]:
    """Exact attention of query [hq, d] over blocks [first_block, first_block + n_blocks) of the
    cold store, minus the blocks set in excluded [h, words] (uint32 bitmap, viewed as int32).

    cold: int8 records [blocks, h, W] (uint8) or pairs [blocks, h, 2, bs, d]. Returns float32
    (out [hq, d], lse [hq]); a head with nothing left gets lse = -inf and out = 0.
    """
    dev = require_cuda(query, cold)
    hq, d = query.shape[-3] if query.dim() == 4 else query.shape[0], query.shape[-1]
    q = query.reshape(hq, d).contiguous()
    h = cold.shape[1]
    kind = L.LKV_COLD_INT8 if cold.dtype == torch.uint8 else L.LKV_COLD_PAIRS
    dt = q.dtype if dtype is None else dtype
    if kind == L.LKV_COLD_PAIRS and cold.dtype != dt:
        raise ValueError(f"cold pairs are {cold.dtype} but the query is {dt}")
    out = torch.empty((hq, d), dtype=torch.float32, device=dev) if out is None else out
    lse = torch.empty((hq,), dtype=torch.float32, device=dev) if lse is None else lse
    ws = workspace(dev, attention_workspace_bytes(h, hq, d, n_blocks), ws_slot)
    words = 0 if excluded is None else excluded.shape[-1]
    call("lkv_cold_attention", ptr(q), hq, h, d, block_size, ptr(cold), kind, dtype_code(dt), first_block, n_blocks, ptr(excluded), words,
         scale, ptr(out), ptr(lse), ptr(ws), ws.numel(), stream_handle(dev))
    return out, lse


def lse_merge(outs: torch.Tensor, lses: torch.Tensor, out_dtype: torch.dtype = torch.float32, out: torch.Tensor | None = None,
              lse_out: torch.Tensor | None = None) -> tuple[torch.Tensor, torch.Tensor]:
    """Merge partials outs [p, rows, d] / lses [p, rows] (float32) into (out [rows, d], lse [rows])."""
    dev = require_cuda(outs, lses)
    p, rows, d = outs.shape
    out = torch.empty((rows, d), dtype=out_dtype, device=dev) if out is None else out
    lse_out = torch.empty((rows,), dtype=torch.float32, device=dev) if lse_out is None else lse_out
    call("lkv_lse_merge", ptr(outs.contiguous()), ptr(lses.contiguous()), p, rows, d, ptr(out), dtype_code(out.dtype), ptr(lse_out),
         stream_handle(dev))
    return out, lse_out


def lse_merge_packed(parts: torch.Tensor, rows: int, d: int, out_dtype: torch.dtype = torch.float32, out: torch.Tensor | None = None,
                     lse_out: torch.Tensor | None = None) -> tuple[torch.Tensor, torch.Tensor]:
    """Merge partials packed per part as out [rows, d] then lse [rows] (parts [p, rows * (d + 1)], float32)."""
    dev = require_cuda(parts)
    p = parts.shape[0]
    if parts.stride(-1) != 1 or parts.numel() != p * rows * (d + 1) or not parts.is_contiguous():
        raise ValueError("lse_merge_packed: parts must be contiguous [p, rows * (d + 1)] float32")
    out = torch.empty((rows, d), dtype=out_dtype, device=dev) if out is None else out
    lse_out = torch.empty((rows,), dtype=torch.float32, device=dev) if lse_out is None else lse_out
    call("lkv_lse_merge_packed", ptr(parts), p, rows, d, ptr(out), dtype_code(out.dtype), ptr(lse_out), stream_handle(dev))
    return out, lse_out


def bitmap_words(n_blocks: int) -> int:
    """uint32 words of a per-head block bitmap covering block ids [0, n_blocks)."""
    return max(1, math.ceil(n_blocks / 32))


def exact_attention(query: torch.Tensor, k_base: torch.Tensor, v_base: torch.Tensor, strides: tuple[int, int, int], blocks: torch.Tensor,
                    last_fill: int, cold: torch.Tensor, first_block: int, n_blocks: int, scale: float, block_size: int,
                    excluded: torch.Tensor | None = None, slot_of: torch.Tensor | None = None, out_dtype: torch.dtype | None = None,
                    out: torch.Tensor | None = None, lse: torch.Tensor | None = None, parts: tuple[torch.Tensor, torch.Tensor] | None = None,
                    ws_slot: int = 0) -> tuple[torch.Tensor, torch.Tensor]:
    """Hot pass, cold pass and their merge in one launch (plus the combine).

    The hot set is as in `hot_attention`, the cold set as in `cold_attention`; returns the merged
    (out [hq, d] in `out_dtype`, lse [hq] float32). `parts`, when given, receives the per-set float32
    partials (out [2, hq, d], lse [2, hq]), hot first.
    """
    dev = require_cuda(query, k_base, v_base, blocks, cold)
    hq, d = query.shape[-3] if query.dim() == 4 else query.shape[0], query.shape[-1]
    q = query.reshape(hq, d).contiguous()
    h, n = blocks.shape
    out_dtype = out_dtype or q.dtype
    out = torch.empty((hq, d), dtype=out_dtype, device=dev) if out is None else out
    lse = torch.empty((hq,), dtype=torch.float32, device=dev) if lse is None else lse
    ws = workspace(dev, int(L.lib().lkv_exact_attention_workspace(h, hq, d, n, n_blocks)), ws_slot)
    s_row, s_head, s_tok = strides
    hot = L.HotSet(ptr(k_base), ptr(v_base), dtype_code(k_base.dtype), s_row, s_head, s_tok, ptr(blocks), n, ptr(slot_of),
                   0 if slot_of is None else slot_of.stride(0), last_fill, storage_rows(k_base, v_base, strides, h, block_size, d))
    kind = L.LKV_COLD_INT8 if cold.dtype == torch.uint8 else L.LKV_COLD_PAIRS
    cs = L.ColdSet(ptr(cold), kind, first_block, n_blocks, ptr(excluded), 0 if excluded is None else excluded.shape[-1])
    po, pl = (None, None) if parts is None else parts
    call("lkv_exact_attention", ptr(q), hq, h, d, block_size, ctypes.byref(hot), ctypes.byref(cs), scale, ptr(out), dtype_code(out.dtype),
         ptr(lse), ptr(po), ptr(pl), ptr(ws), ws.numel(), stream_handle(dev))
    return out, lse


def device_status(clear: bool = True) -> int:
    """Status word of the kernels with bounded waits (0 = no wait ran out). Synchronises."""
    st = ctypes.c_int(0)
    call("lkv_device_status", ctypes.byref(st), int(clear))
    return st.value


_ATTACHED: set[int] = set()


def status_attach(device: torch.device | int | None = None) -> None:
    """Points the kernels on `device` at the host mirror of the status word (once per device)."""
    idx = torch.cuda.current_device() if device is None else (device if isinstance(device, int) else device.index)
    idx = torch.cuda.current_device() if idx is None else idx
    if idx in _ATTACHED:
        return
    with torch.cuda.device(idx):
        call("lkv_status_attach")
    _ATTACHED.add(idx)


def status_poll(clear: bool = True) -> int:
    """The host mirror of the status word, read without synchronising (0 when nothing was recorded,
    or when no device has been attached yet)."""
    if not _ATTACHED:
        return 0
    st = ctypes.c_int(0)
    call("lkv_status_poll", ctypes.byref(st), int(clear))
    return st.value


class DeviceWaitError(RuntimeError):
    """A kernel's bounded wait ran out (or a CTA's list overflowed): its output was poisoned."""


def raise_on_status(where: str) -> None:
    """Raises DeviceWaitError when the status mirror holds a code (clearing it)."""
    code = status_poll(clear=True)
    if code:
        what = {L.LKV_DEV_WAIT_TIMEOUT: "a bounded wait on the GPU ran out", L.LKV_DEV_LIST_OVERFLOW: "an attention CTA's item list overflowed"}
        raise DeviceWaitError(f"{where}: {what.get(code, f'device status {code}')} (an earlier step's output is not valid)")


def debug_set(key: int, value: int) -> None:
    """Test hooks of the bounded waits (lkv_debug_set)."""
    call("lkv_debug_set", key, value)


def tier_admit(chosen: torch.Tensor, block_slot: torch.Tensor, slot_block: torch.Tensor, last_used: torch.Tensor, evicted_at: torch.Tensor | None,
               step: int, store: torch.Tensor, pool: torch.Tensor, miss_blk: torch.Tensor, miss_slot: torch.Tensor, n_miss: torch.Tensor,
               slots_out: torch.Tensor | None = None, miss_total: torch.Tensor | None = None) -> None:
    """Device-side residency admit of `chosen` [h, k] plus the fetch of the misses (see lkv_tier_admit);
    `miss_total` (int64 scalar on the device, optional) accumulates the misses."""
    dev = require_cuda(chosen, block_slot, slot_block, last_used, store, pool)
    h, k = chosen.shape
    n_slots = slot_block.shape[1]
    bs, d = pool.shape[-2], pool.shape[-1]
    kind = L.LKV_COLD_INT8 if store.dtype == torch.uint8 else L.LKV_COLD_PAIRS
    call("lkv_tier_admit", ptr(chosen), h, k, chosen.stride(0), ptr(block_slot), block_slot.shape[1], ptr(slot_block), ptr(last_used), n_slots,
         ptr(evicted_at), step, ptr(store), kind, ptr(pool), bs, d, dtype_code(pool.dtype), ptr(miss_blk), ptr(miss_slot), ptr(n_miss),
         ptr(slots_out), 0 if slots_out is None else slots_out.stride(0), ptr(miss_total), stream_handle(dev))


def append_tokens(keys: torch.Tensor, values: torch.Tensor, slot: torch.Tensor, fill: int) -> None:
    """keys / values [h, T, d] (unit channel stride) into pool slot [h, 2, bs, d] at token positions
    fill .. fill + T - 1, in one launch (lkv_append_tokens)."""
    dev = require_cuda(keys, values, slot)
    h, t, d = keys.shape
    if values.shape != keys.shape or keys.dtype != slot.dtype or values.dtype != slot.dtype or keys.stride(-1) != 1 or values.stride(-1) != 1:
        raise ValueError("append_tokens needs keys and values [h, T, d] of the slot's dtype with unit channel stride")
    if not slot.is_contiguous() or slot.shape[0] != h or slot.shape[1] != 2 or slot.shape[-1] != d:
        raise ValueError(f"append_tokens needs a contiguous slot [{h}, 2, bs, {d}]")
    call("lkv_append_tokens", ptr(keys), keys.stride(0), keys.stride(1), ptr(values), values.stride(0), values.stride(1), h, t, d,
         dtype_code(slot.dtype), ptr(slot), slot.shape[2], fill, stream_handle(dev))


def mark_blocks(ids: torch.Tensor, bitmap: torch.Tensor) -> torch.Tensor:
    """Clear `bitmap` [h, words] and set the bit of every block id in `ids` [h, k] (int32; -1 is
    skipped), as the selection marks its own choice (lkv_mark_blocks). Returns `bitmap`."""
    dev = require_cuda(ids, bitmap)
    if ids.dtype != torch.int32 or bitmap.dtype != torch.int32 or ids.stride(-1) != 1 or not bitmap.is_contiguous():
        raise ValueError("mark_blocks needs int32 ids with unit column stride and a contiguous int32 bitmap")
    if ids.shape[0] != bitmap.shape[0]:
        raise ValueError(f"ids has {ids.shape[0]} heads, the bitmap {bitmap.shape[0]}")
    call("lkv_mark_blocks", ptr(ids), ids.shape[0], ids.shape[1], ids.stride(0), ptr(bitmap), bitmap.shape[1], stream_handle(dev))
    return bitmap


def quest_topk_admit(query: torch.Tensor, kmin: torch.Tensor, kmax: torch.Tensor, first_block: int, n_cand: int, k: int, chosen: torch.Tensor,
                     bitmap: torch.Tensor | None, block_slot: torch.Tensor, slot_block: torch.Tensor, last_used: torch.Tensor,
                     evicted_at: torch.Tensor | None, step: int, store: torch.Tensor, pool: torch.Tensor, miss_blk: torch.Tensor,
                     miss_slot: torch.Tensor, n_miss: torch.Tensor, slots_out: torch.Tensor | None = None,
                     bound_dtype: torch.dtype | None = None, ws_slot: int = 1, miss_total: torch.Tensor | None = None) -> torch.Tensor:
    """quest_topk in block order into `chosen` [h, k] (and the bitmap), then tier_admit of that
    selection, in one library call (lkv_quest_topk_admit). Returns `chosen`."""
    dev = require_cuda(query, kmin, kmax, chosen, block_slot, slot_block, last_used, store, pool)
    hq, d = query.shape[-3] if query.dim() == 4 else query.shape[0], query.shape[-1]
    q = query.reshape(hq, d).contiguous()
    h = kmin.shape[-3]
    if chosen.stride(-1) != 1 or chosen.shape[-1] < k:
        raise ValueError("quest_topk_admit: chosen must be [h, >=k] int32 with unit column stride")
    bound_dtype = bound_dtype or q.dtype
    ws = workspace(dev, int(L.lib().lkv_quest_topk_workspace(h, n_cand)), ws_slot)
    words = 0 if bitmap is None else bitmap.shape[-1]
    kind = L.LKV_COLD_INT8 if store.dtype == torch.uint8 else L.LKV_COLD_PAIRS
    call("lkv_quest_topk_admit", ptr(q), dtype_code(q.dtype), hq, h, d, ptr(kmin), ptr(kmax), dtype_code(kmin.dtype), kmin.stride(-3), first_block,
         n_cand, k, dtype_code(bound_dtype), ptr(chosen), chosen.stride(0), None, ptr(bitmap), words, ptr(ws), ws.numel(), ptr(block_slot),
         block_slot.shape[1], ptr(slot_block), ptr(last_used), slot_block.shape[1], ptr(evicted_at), step, ptr(store), kind, ptr(pool),
         pool.shape[-2], dtype_code(pool.dtype), ptr(miss_blk), ptr(miss_slot), ptr(n_miss), ptr(slots_out),
         0 if slots_out is None else slots_out.stride(0), ptr(miss_total), stream_handle(dev))
    return chosen
