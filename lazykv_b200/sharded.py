"""Context sharding of the tiered decode hot path over the GPUs of one node.

The softmax partials over disjoint key sets merge exactly by their log-sum-exp
(lazykv/exact.py:69-85), so one layer's sealed blocks are split into contiguous ranges, one per
rank (`shard_plan`); each rank selects among its own candidates, runs the hot and cold passes over
its range and emits (out, lse) for the layer's query rows; the ranks exchange only those partials
(an all-gather of [hq, d + 1] floats per rank) and every rank merges them with the n-way
`lkv_lse_merge`. The reference runs on one GPU; this module has no counterpart there.

Selection across shards has two modes:
  * local budgets (default): rank r selects its share of K among its own candidates
    (`shard_plan`'s k_local, in proportion to its candidates). In the exact tier the output does
    not depend on which blocks are selected (every sealed block is attended once, hot or cold), so
    this is exact and needs no exchange before the attention;
  * global (`GlobalSelection`): every rank's candidate bounds are all-gathered ([h, n_local]
    bf16 per rank, a quarter of the bytes of top-K (bound, id) pairs at a 25% budget) and every
    rank runs the same select over them (`lkv_topk_gathered`), so the selection equals the
    single-GPU one; each rank then admits and attends the selected blocks of its range (a
    different count per head: its lists are padded with -1). The candidate form of the same
    exchange (`local_candidates`, `gather_candidates`, `topk_merge`: top-min(K, n_local)
    (bound, id) pairs, one CTA per head) is kept for callers that hold only their local top-K.
"""

from __future__ import annotations

import ctypes
from dataclasses import dataclass

import numpy as np
import torch
import torch.distributed as dist

from lazykv_b200 import _lib as L
from lazykv_b200 import kernels as K


@dataclass(frozen=True)
class ShardPlan:
    """Rank's part of a layer: sealed blocks [lo, hi), candidates [cand_first, cand_first + n_cand)."""

    lo: int
    hi: int
    cand_first: int
    n_cand: int
    k_local: int
    has_sink: bool
    has_current: bool


def shard_plan(n_sealed: int, k_total: int, world: int, rank: int) -> ShardPlan:
    """The plan of lkv_shard_plan (host arithmetic, no GPU needed)."""
    out = (ctypes.c_int32 * 5)()
    L.call("lkv_shard_plan", n_sealed, k_total, world, rank, out)
    lo, hi, first, n, k = (int(x) for x in out)
    return ShardPlan(lo, hi, first, n, k, lo == 0, rank == world - 1)


def _all_gather(t: torch.Tensor, group: dist.ProcessGroup | None) -> torch.Tensor:
    """[world, *t.shape] on every rank, rank order (all_gather_into_tensor where the backend has it)."""
    world = dist.get_world_size(group)
    out = torch.empty((world, *t.shape), dtype=t.dtype, device=t.device)
    if t.is_cuda:
        dist.all_gather_into_tensor(out, t.contiguous(), group=group)
    else:
        dist.all_gather(list(out.unbind(0)), t.contiguous(), group=group)
    return out


def gather_partials(out: torch.Tensor, lse: torch.Tensor, group: dist.ProcessGroup | None = None) -> tuple[torch.Tensor, torch.Tensor]:
    """All ranks' (out [rows, d], lse [rows]) float32 partials: ([world, rows, d], [world, rows]).

    One collective: out and lse travel together as [rows, d + 1]."""
    rows, d = out.shape
    packed = torch.cat([out.float(), lse.float().view(rows, 1)], dim=1)
    allp = _all_gather(packed, group)
    return allp[:, :, :d], allp[:, :, d]


def merge_partials(outs: torch.Tensor, lses: torch.Tensor, out_dtype: torch.dtype = torch.float32,
                   out: torch.Tensor | None = None) -> tuple[torch.Tensor, torch.Tensor]:
    """The n-way log-sum-exp merge of gathered partials, on the device (lkv_lse_merge)."""
    return K.lse_merge(outs.contiguous(), lses.contiguous(), out_dtype, out=out)


class PackedPartial:
    """A rank's partial as one buffer [rows * (d + 1)] float32: out [rows, d] then lse [rows] (both
    contiguous views), so the exchange is one all-gather into [world, rows * (d + 1)] and the merge
    reads the gathered buffer in place (lkv_lse_merge_packed)."""

    def __init__(self, rows: int, d: int, world: int, device: torch.device) -> None:
        self.rows, self.d = rows, d
        self.buf = torch.zeros(rows * (d + 1), dtype=torch.float32, device=device)
        self.out = self.buf[: rows * d].view(rows, d)
        self.lse = self.buf[rows * d :]
        self.gathered = torch.zeros((world, rows * (d + 1)), dtype=torch.float32, device=device)

    def exchange(self, group: dist.ProcessGroup | None = None) -> None:
        dist.all_gather_into_tensor(self.gathered, self.buf, group=group)

    def merge(self, out_dtype: torch.dtype = torch.bfloat16, out: torch.Tensor | None = None) -> torch.Tensor:
        merged, _ = K.lse_merge_packed(self.gathered, self.rows, self.d, out_dtype, out=out)
        return merged


class PeerExchange:
    """The per-layer exchange of partials by peer stores over NVLink (lkv_exchange_merge): a rank's
    (out, lse) go straight into every peer's inbox and each rank merges what arrived, in one
    launch, instead of an NCCL all-gather and a merge launch. Built collectively: every rank
    allocates its region, the 64-byte IPC handles are all-gathered over `group` (once, at set-up),
    and every rank opens its peers'. `exchange` is graph-capturable. `close` (or garbage
    collection) releases the peers' mappings and the region; every rank must stop calling
    `exchange` first."""

    def __init__(self, rows: int, d: int, group: dist.ProcessGroup | None = None, device: torch.device | None = None) -> None:
        self.rows, self.d = rows, d
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        self.device = device or torch.device("cuda", torch.cuda.current_device())
        base = ctypes.c_void_p()
        handle = (ctypes.c_char * 64)()
        with torch.cuda.device(self.device):
            L.call("lkv_exchange_alloc", rows, d, self.world, ctypes.byref(base), handle)
        self._own = base.value
        handles = [bytes(handle)]
        if self.world > 1:
            handles = [None] * self.world
            dist.all_gather_object(handles, bytes(handle), group=group)
        bases = []
        self._opened = []
        with torch.cuda.device(self.device):
            for r, hb in enumerate(handles):
                if r == self.rank:
                    bases.append(self._own)
                    continue
                peer = ctypes.c_void_p()
                L.call("lkv_exchange_open", (ctypes.c_char * 64).from_buffer_copy(hb), ctypes.byref(peer))
                self._opened.append(peer.value)
                bases.append(peer.value)
        self._bases = (ctypes.c_void_p * self.world)(*bases)
        # This rank's partial, float32: out [rows, d] then lse [rows] (one buffer, as PackedPartial).
        self.buf = torch.zeros(rows * (d + 1), dtype=torch.float32, device=self.device)
        self.out = self.buf[: rows * d].view(rows, d)
        self.lse = self.buf[rows * d :]

    def exchange(self, merged: torch.Tensor, merged_lse: torch.Tensor | None = None) -> torch.Tensor:
        """Push this rank's partial (self.out, self.lse) to every rank, wait for theirs, merge into
        `merged` [rows, d] (bf16 or float32) and optionally `merged_lse` [rows]."""
        L.call("lkv_exchange_merge", L.ptr(self.out), L.ptr(self.lse), self.rows, self.d, self.world, self.rank, self._bases, L.ptr(merged),
               L.dtype_code(merged.dtype), L.ptr(merged_lse), L.stream_handle(self.device))
        return merged

    def close(self) -> None:
        if self._own is None:
            return
        torch.cuda.synchronize(self.device)
        with torch.cuda.device(self.device):
            for p in self._opened:
                L.call("lkv_exchange_close", ctypes.c_void_p(p))
            L.call("lkv_exchange_free", ctypes.c_void_p(self._own))
        self._opened, self._own = [], None

    def __del__(self) -> None:
        try:
            self.close()
        except Exception:  # noqa: BLE001 - interpreter shutdown
            pass


def gather_candidates(ids: torch.Tensor, bounds: torch.Tensor, group: dist.ProcessGroup | None = None) -> tuple[torch.Tensor, torch.Tensor]:
    """Every rank's local candidates (ids [h, k] int32, ascending; bounds [h, k] float32) as
    [h, world * k] in rank order, i.e. ascending id across the node (ranks hold ascending ranges)."""
    h, k = ids.shape
    packed = torch.stack([bounds.float(), ids.to(torch.int32).view(torch.float32)], dim=0)  # [2, h, k], ids bit-cast
    allp = _all_gather(packed, group)  # [world, 2, h, k]
    b = allp[:, 0].permute(1, 0, 2).reshape(h, -1).contiguous()
    i = allp[:, 1].contiguous().view(torch.int32).permute(1, 0, 2).reshape(h, -1).contiguous()
    return i, b


def topk_merge(ids: torch.Tensor, bounds: torch.Tensor, k: int, bound_dtype: torch.dtype = torch.bfloat16, by_block: bool = True,
               out_blocks: torch.Tensor | None = None, bitmap: torch.Tensor | None = None) -> torch.Tensor:
    """Top-k block ids [h, k] over gathered candidates (lkv_topk_merge), ties to the lower id."""
    dev = K.require_cuda(ids, bounds)
    h, n = ids.shape
    out_blocks = torch.empty((h, k), dtype=torch.int32, device=dev) if out_blocks is None else out_blocks
    ws = K.workspace(dev, int(L.lib().lkv_topk_merge_workspace(h, n)), 2)
    words = 0 if bitmap is None else bitmap.shape[-1]
    L.call("lkv_topk_merge", L.ptr(bounds.float().contiguous()), L.ptr(ids.contiguous()), h, n, n, k, L.dtype_code(bound_dtype),
           L.LKV_ORDER_BLOCK if by_block else L.LKV_ORDER_BOUND, L.ptr(out_blocks), out_blocks.stride(0), L.ptr(bitmap), words, L.ptr(ws),
           ws.numel(), L.stream_handle(dev))
    return out_blocks


def local_candidates(query: torch.Tensor, kmin: torch.Tensor, kmax: torch.Tensor, first: int, n_cand: int, k: int,
                     bound_dtype: torch.dtype | None = None) -> tuple[torch.Tensor, torch.Tensor]:
    """This shard's top-min(k, n_cand) candidates (ids ascending) and their bounds, for a global selection."""
    kk = min(k, n_cand)
    ids, bound = K.quest_topk(query, kmin, kmax, first, n_cand, kk, bound_dtype, want_bound=True, by_block=True)
    b = torch.gather(bound, 1, (ids - first).long())
    return ids, b


def shard_hot_list(global_ids: torch.Tensor, plan: ShardPlan, k_pad: int | None = None) -> torch.Tensor:
    """The part of a global selection [h, K] (ascending ids) inside this rank's range, padded with -1
    to a common length per head: [h, k_pad], ids ascending then -1 (device work only)."""
    h, kk = global_ids.shape
    inside = (global_ids >= plan.cand_first) & (global_ids < plan.hi)
    # Stable compaction: inside ids first (they are ascending), padding after.
    key = torch.where(inside, torch.zeros_like(global_ids), torch.ones_like(global_ids))
    order = torch.argsort(key, dim=1, stable=True)
    ids = torch.gather(torch.where(inside, global_ids, torch.full_like(global_ids, -1)), 1, order)
    k_pad = kk if k_pad is None else k_pad
    return ids[:, :k_pad].contiguous()


class GlobalSelection:
    """The global top-k of a context-sharded layer: every rank scores its own candidates into a
    send buffer [h, ld] (lkv_quest_bounds), one all-gather gives every rank all the bounds
    [world, h, ld], and every rank runs the same select over them (lkv_topk_gathered), keeping its
    own part as local ids. The selection is the one lkv_quest_topk makes over the unsharded
    candidates (ties at the k-th bound to the lower block ids), so the ranks agree and their parts
    add up to it. The per-rank hot list then holds between 0 and min(k, n_cand) blocks: `cols`."""

    def __init__(self, plans: list[ShardPlan], rank: int, h: int, k_total: int, device: torch.device,
                 bound_dtype: torch.dtype = torch.bfloat16) -> None:
        self.plans, self.rank, self.k = plans, rank, k_total
        self.plan = plans[rank]
        self.seg_n = [p.n_cand for p in plans]
        self.ld = max(self.seg_n)
        self.cols = min(k_total, self.plan.n_cand)
        self.bound_dtype = bound_dtype
        self.send = torch.zeros((h, self.ld), dtype=bound_dtype, device=device)
        self.gathered = torch.zeros((len(plans), h, self.ld), dtype=bound_dtype, device=device)

    def select(self, query: torch.Tensor, kmin: torch.Tensor, kmax: torch.Tensor, chosen: torch.Tensor, bitmap: torch.Tensor | None = None,
               group: dist.ProcessGroup | None = None, block_slot: torch.Tensor | None = None, hot: torch.Tensor | None = None) -> torch.Tensor:
        """This rank's part of the global selection of `query` into chosen [h, >= cols] (local ids
        ascending, then -1) and the bitmap; kmin/kmax are the rank's metadata (local ids). With
        `block_slot` and `hot`, the resident split (hot: the chosen blocks' current slots or -1; the
        bitmap: only the resident ones)."""
        p = self.plan
        first = p.cand_first - p.lo
        K.quest_bounds(query, kmin, kmax, first, p.n_cand, self.send, self.bound_dtype)
        if len(self.plans) > 1:
            dist.all_gather_into_tensor(self.gathered, self.send, group=group)
        else:
            self.gathered[0].copy_(self.send)
        return K.topk_gathered(self.gathered, self.seg_n, self.k, self.rank, first, chosen, bitmap, out_cols=self.cols, block_slot=block_slot, hot=hot)


class ShardedExactStep:
    """One decode step of one selecting layer over this rank's shard, then the cross-rank merge.

    The shard's stores are the tier's layouts restricted to [lo, hi): metadata [h, n_local, d],
    int8 records [n_local, h, W] (or pairs [n_local, h, 2, bs, d]), and the slot pool with the
    block -> slot map (local ids). `hot_list` [h, n_list] (local ids, -1 padding) is rewritten by
    `select`; the sink (local block 0 on rank 0) and the current block (local id n_local on the
    last rank) are fixed entries.
    """

    def __init__(self, plan: ShardPlan, block_size: int, kmin: torch.Tensor, kmax: torch.Tensor, records: torch.Tensor, pool: torch.Tensor,
                 slot_of: torch.Tensor | None, hot_list: torch.Tensor, bitmap: torch.Tensor, fill: int, scale: float,
                 group: dist.ProcessGroup | None = None) -> None:
        self.plan, self.bs, self.kmin, self.kmax, self.records = plan, block_size, kmin, kmax, records
        self.pool, self.slot_of, self.hot_list, self.bitmap = pool, slot_of, hot_list, bitmap
        self.fill, self.scale, self.group = fill, scale, group
        self.sel_off = int(plan.has_sink)
        h, _, d = kmin.shape
        self.h, self.d = h, d

    def select_local(self, query: torch.Tensor) -> None:
        """Local budget: this rank's k_local best candidates into the hot list and the bitmap."""
        p = self.plan
        K.quest_topk(query, self.kmin, self.kmax, p.cand_first - p.lo, p.n_cand, p.k_local, out_blocks=self.hot_list[:, self.sel_off:],
                     bitmap=self.bitmap, by_block=True)

    def attend(self, query: torch.Tensor, out: torch.Tensor | None = None, lse: torch.Tensor | None = None) -> tuple[torch.Tensor, torch.Tensor]:
        """Hot + cold passes over the shard and their merge: this rank's partial (out, lse), float32."""
        p, d = self.plan, self.d
        strides = (self.h * 2 * self.bs * d, 2 * self.bs * d, d)
        return K.exact_attention(query, self.pool, self.pool[:, :, 1], strides, self.hot_list, self.fill if p.has_current else self.bs,
                                 self.records, p.cand_first - p.lo, p.n_cand, self.scale, self.bs, excluded=self.bitmap, slot_of=self.slot_of,
                                 out_dtype=torch.float32, out=out, lse=lse)

    def step(self, query: torch.Tensor, out_dtype: torch.dtype = torch.bfloat16) -> torch.Tensor:
        """Select, attend, all-gather the partials (one collective), merge: the layer's output
        [hq, d] on every rank."""
        hq = query.shape[-3] if query.dim() == 4 else query.shape[0]
        if getattr(self, "_packed", None) is None:
            self._packed = PackedPartial(hq, self.d, dist.get_world_size(self.group), query.device)
        pk = self._packed
        self.select_local(query)
        self.attend(query, out=pk.out, lse=pk.lse)
        pk.exchange(self.group)
        return pk.merge(out_dtype)


def host_reference_global_topk(ids: np.ndarray, bounds: np.ndarray, k: int) -> np.ndarray:
    """The global selection over gathered candidates on the host (descending bound, ties to the
    lower id), ascending ids [h, k]: what lkv_topk_merge computes, for tests and tooling."""
    h = ids.shape[0]
    out = np.empty((h, k), dtype=np.int64)
    for j in range(h):
        order = np.lexsort((ids[j], -bounds[j].astype(np.float64)))
        out[j] = np.sort(ids[j][order[:k]])
    return out


def gathered_layout(plans: list[ShardPlan]) -> tuple[list[int], int]:
    """The ranks' candidate counts and the common row stride of the gathered bounds buffer
    [world, h, ld] that GlobalSelection all-gathers."""
    seg_n = [p.n_cand for p in plans]
    return seg_n, max(seg_n)


def host_reference_gathered_topk(gathered: np.ndarray, seg_n: list[int], k: int, rank: int, out_base: int) -> np.ndarray:
    """What lkv_topk_gathered writes for `rank`, on the host, for tests and tooling: over every
    rank's bounds (gathered [world, h, ld], rank r's first seg_n[r] entries, in block order), the k
    highest per row with ties to the lower block id; rank's chosen as local ids (out_base + index
    in its range) ascending, then -1, min(k, seg_n[rank]) columns."""
    world, h, _ = gathered.shape
    starts = np.concatenate([[0], np.cumsum(seg_n)])
    cols = min(k, seg_n[rank])
    out = np.full((h, cols), -1, dtype=np.int64)
    for j in range(h):
        row = np.concatenate([gathered[r, j, : seg_n[r]].astype(np.float64) for r in range(world)])
        row = np.where(row == 0.0, 0.0, row)  # +0 and -0 tie
        order = np.lexsort((np.arange(len(row)), -row))[: min(k, len(row))]
        mine = np.sort(order[(order >= starts[rank]) & (order < starts[rank + 1])]) - starts[rank]
        out[j, : len(mine)] = mine + out_base
    return out
