"""The tier: HBM slot pool, pinned host store, and a decode step that never returns to the host.

API of lazykv/tiered.py (TieredLayer :150-535, TieredCache :538-860, allocate_host_pools :874-882)
with the same layouts: the pool [n_slots + 2, h, 2, bs, d] in the model dtype (slot 0 the sink,
the last slot the block being filled), the host store [cap, h, 2, bs, d] in the model dtype or
[cap, h, packed_pair_bytes] int8 records, metadata [1, h, cap, d], and the reference's residency
tables (slot_block, block_slot, last_used, evicted_at).

What changes is where the work runs. Per selecting layer and decode step:
  1. selection: Quest bound + top-K on the device (lkv_quest_topk); indices stay there;
  2. residency: the reference's LRU admit as a device kernel, which also fetches the misses from
     the host store (zero-copy loads; int8 records dequantised exactly as unpack) into their slots
     (lkv_tier_admit), so the tables live on the device;
  3. attention over [sink, selected, current] read in place from the pool (lkv_hot_attention), or,
     in the exact tier, that and the cold pass over every other sealed block with the merge, in one
     launch (lkv_exact_attention).
Sealing a block packs or copies it into the host store with a kernel and updates its metadata on
the device, asynchronously. The host only tracks lengths.

Cold placement: the store the exact pass and the fetches read is the pinned host store through its
device view (`cold_placement="host"`, zero-copy over the link), or a device copy kept alongside it
(`"device"`).

Record and replay (tiered.py:620-621, 715-724, 832-836): `record_selection=True` keeps a device
copy of every selecting layer's chosen ids per step, read back by recorded_selection();
`replay_selection` feeds such a map back in place of the selection (loaded, admitted and attended
as the selection's own choice), which repeats the recorded run's fetches and outputs exactly.
"""

from __future__ import annotations

import ctypes
import time
import weakref
from collections.abc import Mapping
from dataclasses import asdict, dataclass, field
from typing import Any

import numpy as np
import torch
from transformers import PreTrainedModel
from transformers.cache_utils import Cache

from lazykv_b200 import _lib as L
from lazykv_b200 import kernels as K
from lazykv_b200.cache import CacheStats, FullGPUCache
from lazykv_b200.pinned import device_view, pinned_empty
from lazykv_b200.quant import packed_pair_bytes
from lazykv_b200.selection import QUEST_DENSE_LAYERS, current_block_mask

NEVER = -(2**40)  # "evicted at" of pairs never evicted (tiered.py:69)
PREFETCH_WS_SLOT = 8  # selection workspace of the prefetch stream (the compute stream's selections use slot 1)
BOUNDARY_CHUNK = 128  # blocks packed at once at the boundary (tiered.py:70)


@dataclass
class TierCounters:
    """What the tier did (the reference's tiered.py:76-109, less its host-time split)."""

    host_select_s: float = 0.0
    selections: int = 0
    selected_pairs: int = 0
    hit_pairs: int = 0
    fetched_pairs: int = 0
    fetch_transfers: int = 0
    fetch_bytes: int = 0
    seals: int = 0
    seal_bytes: int = 0
    boundary_d2h_s: float = 0.0
    boundary_d2h_bytes: int = 0
    zerocopy_bytes: int = 0
    ingest_forwards: int = 0
    ingest_tokens: int = 0
    ingest_h2d_bytes: int = 0
    # The layer-ahead prefetch (tiered.py:94-97): pairs its speculative admits fetched, its admits
    # (one fetch launch each), their bytes, and how many of those pairs the real selection then chose.
    host_prefetch_s: float = 0.0
    prefetched_pairs: int = 0
    prefetch_transfers: int = 0
    prefetch_bytes: int = 0
    prefetch_used_pairs: int = 0
    fetched_pairs_per_step: list[int] = field(default_factory=list)


class TieredLayer:
    """One selecting layer: GPU slot pool, pinned host store, metadata and device residency tables."""

    def __init__(self, keys: torch.Tensor, values: torch.Tensor, k_blocks: int, block_size: int, capacity_tokens: int,
                 host: torch.Tensor | None = None, n_slots: int | None = None, quant: str | None = None, cold_placement: str = "host") -> None:
        """The layer at the boundary from its whole prompt KV [1, h, T, d] (lazykv/tiered.py:161-206):
        every sealed block into the store with its metadata, the newest blocks seeded into slots,
        the exact sink and the unsealed tail into the pool."""
        self._open_boundary(keys, keys.shape[2], k_blocks, block_size, capacity_tokens, host, n_slots, quant, cold_placement)
        self.close_boundary(keys, values)

    @classmethod
    def open_boundary(cls, like: torch.Tensor, total_tokens: int, k_blocks: int, block_size: int, capacity_tokens: int,
                      host: torch.Tensor | None = None, n_slots: int | None = None, quant: str | None = None,
                      cold_placement: str = "host") -> TieredLayer:
        """A layer whose boundary is written while its prompt is still being prefilled: `ingest` after
        each chunk stores the blocks that chunk completed, `close_boundary` after the last one. `like`
        ([1, h, *, d]) gives the heads, head_dim, dtype and device; `total_tokens` is the prompt's length."""
        self = cls.__new__(cls)
        self._open_boundary(like, total_tokens, k_blocks, block_size, capacity_tokens, host, n_slots, quant, cold_placement)
        return self

    def _open_boundary(self, like: torch.Tensor, total_tokens: int, k_blocks: int, bs: int, capacity_tokens: int, host: torch.Tensor | None,
                       n_slots: int | None, quant: str | None, cold_placement: str) -> None:
        n_blocks = total_tokens // bs
        self._allocate(like.shape[1], like.shape[3], n_blocks, k_blocks, bs, capacity_tokens, like.device, like.dtype, host, n_slots, quant,
                       cold_placement)
        self._bd_tokens, self._bd_blocks = total_tokens, n_blocks
        self._bd_seed = min(self.n_slots, n_blocks - 1)  # the newest blocks start resident (tiered.py:176-180)
        self._bd_done = 0  # blocks already in the store
        self._bd_s = 0.0

    def ingest(self, keys: torch.Tensor, values: torch.Tensor, upto: int) -> None:
        """Stores the sealed blocks that tokens [0, upto) of keys/values [1, h, >= upto, d] complete
        and that are not stored yet, in pieces of BOUNDARY_CHUNK blocks; a block among the seeded
        newest ones also goes to its slot, holding what a fetch of it would (its dequantised record
        under int8). Nothing here waits for the device."""
        t0 = time.perf_counter()
        bs = self.bs
        last = min(upto // bs, self._bd_blocks)
        first_seeded = self._bd_blocks - self._bd_seed
        while self._bd_done < last:
            c0 = self._bd_done
            c1 = min(last, c0 + BOUNDARY_CHUNK)
            span = slice(c0 * bs, c1 * bs)
            pairs = torch.stack((keys[0, :, span], values[0, :, span]), dim=1).unflatten(2, (c1 - c0, bs)).permute(2, 0, 1, 3, 4).contiguous()
            resident = self._store_blocks(pairs, c0)
            a = max(c0, first_seeded)
            if a < c1 and self._bd_seed > 0:
                self.pool[1 + a - first_seeded : 1 + c1 - first_seeded] = resident[a - c0 :]
            self._bd_done = c1
        self._bd_s += time.perf_counter() - t0

    def _store_blocks(self, pairs: torch.Tensor, c0: int) -> torch.Tensor:
        """Blocks c0 .. c0 + n of `pairs` [n, h, 2, bs, d] into the store, with their min/max key
        metadata; returns the values a slot holds for them. The int8 records are written straight
        into the pinned store through its device view, and their metadata is taken over the
        dequantised keys (tiered.py:182-197)."""
        c1 = c0 + pairs.shape[0]
        if self.quant is None:
            self.host[c0:c1].copy_(pairs, non_blocking=True)
            if self.dev_store is not None:
                self.dev_store[c0:c1].copy_(pairs)
            K.block_minmax(pairs[:, :, 0].transpose(0, 1), self.bs, self.kmin[0], self.kmax[0], first_block=c0)
            return pairs
        deq = torch.empty_like(pairs)
        K.pack_int8(pairs, records=self.host_dev[c0:c1], kmin=self.kmin[0], kmax=self.kmax[0], first_block=c0, deq=deq)
        if self.dev_store is not None:
            self.dev_store[c0:c1].copy_(self.host_dev[c0:c1])
        return deq

    def close_boundary(self, keys: torch.Tensor, values: torch.Tensor) -> None:
        """The boundary's end: any blocks not yet stored, the sink (which never leaves VRAM and stays
        exact, even under int8: tiered.py:200-202), the unsealed tail into the current slot, and the
        residency tables. Waits for the device once."""
        self.ingest(keys, values, self._bd_tokens)
        t0 = time.perf_counter()
        bs, n_blocks = self.bs, self._bd_blocks
        tail = self._bd_tokens - n_blocks * bs
        for half, src in enumerate((keys, values)):
            self.pool[0, :, half] = src[0, :, :bs]
            if tail:
                self.pool[self.tail_slot, :, half, :tail] = src[0, :, n_blocks * bs : self._bd_tokens]
        torch.cuda.synchronize(self.pool.device)
        self.boundary_d2h_s = self._bd_s + time.perf_counter() - t0
        self.boundary_d2h_bytes = n_blocks * self.h * self.pair_bytes
        self._finish(n_blocks, tail, self._bd_seed)

    @classmethod
    def from_store(cls, host: torch.Tensor, n_blocks: int, tail: torch.Tensor, k_blocks: int, block_size: int, capacity_tokens: int,
                   device: torch.device, n_slots: int | None = None, quant: str | None = None, sink: torch.Tensor | None = None,
                   cold_placement: str = "host") -> TieredLayer:
        """A layer whose pinned host store already holds its `n_blocks` sealed blocks (a restored
        snapshot); the classmethod of lazykv/tiered.py:209-241, extended to the int8 store.

        The result is the layer the constructor builds from the same KV: the metadata and the seeded
        slots are derived on the device from the store's bytes (the bf16 pairs, or the int8 records
        dequantised as a fetch does, whose min/max are the metadata the constructor writes), and the
        residency tables are seeded the same way. `tail` is the unsealed block [h, 2, fill, d]. An
        int8 store also needs `sink`, the exact first block [h, 2, bs, d]: its record is lossy and the
        sink stays exact in VRAM. Nothing here waits for the device.
        """
        if (quant == "int8") != (host.dtype == torch.uint8):
            raise ValueError(f"a {host.dtype} store does not hold a quant={quant!r} tier")
        if quant == "int8" and sink is None:
            raise ValueError("an int8 store needs the exact sink block: its record is lossy")
        self = cls.__new__(cls)
        h, bs, fill = host.shape[1], block_size, tail.shape[2]
        d, dt = tail.shape[3], tail.dtype
        self._allocate(h, d, n_blocks, k_blocks, bs, capacity_tokens, device, dt, host, n_slots, quant, cold_placement)
        seed = min(self.n_slots, n_blocks - 1)
        lo_seed = n_blocks - seed
        for c0 in range(0, n_blocks, BOUNDARY_CHUNK):
            c1 = min(n_blocks, c0 + BOUNDARY_CHUNK)
            g = host[c0:c1].to(device, non_blocking=True)  # [n, h, 2, bs, d] pairs or [n, h, W] records
            if self.dev_store is not None:
                self.dev_store[c0:c1].copy_(g)
            pairs = g if quant is None else K.unpack_int8(g.flatten(0, 1), bs, d, dt).view(c1 - c0, h, 2, bs, d)
            K.block_minmax(pairs[:, :, 0].transpose(0, 1), bs, self.kmin[0], self.kmax[0], first_block=c0)
            lo = max(c0, lo_seed)
            if lo < c1 and seed > 0:
                self.pool[1 + lo - lo_seed : 1 + c1 - lo_seed] = pairs[lo - c0 :]
            if c0 == 0 and quant is None:
                self.pool[0] = pairs[0]
        if quant is not None:
            self.pool[0] = sink.to(device, non_blocking=True)
        if fill:
            self.pool[self.tail_slot, :, :, :fill] = tail.to(device, non_blocking=True)
        self.boundary_d2h_s, self.boundary_d2h_bytes = 0.0, 0  # nothing crossed device to host
        self._finish(n_blocks, fill, seed)
        return self

    # -- set-up ----------------------------------------------------------------------------------

    def _allocate(self, h: int, d: int, n_blocks: int, k_blocks: int, bs: int, capacity_tokens: int, dev: torch.device, dt: torch.dtype,
                  host: torch.Tensor | None, n_slots: int | None, quant: str | None, cold_placement: str) -> None:
        if n_blocks - 1 <= k_blocks:
            raise ValueError(f"budget of {k_blocks} blocks covers all {n_blocks - 1} candidate blocks; the tier needs selection")
        n_slots = k_blocks if n_slots is None else n_slots
        if 0 < n_slots < k_blocks:
            raise ValueError(f"{n_slots} slots cannot hold a selection of {k_blocks} blocks")
        if quant not in (None, "int8"):
            raise ValueError(f"unknown tier precision {quant!r}")
        if cold_placement not in ("host", "device"):
            raise ValueError(f"unknown cold placement {cold_placement!r}")
        self.h, self.d, self.bs, self.k, self.n_slots = h, d, bs, k_blocks, n_slots
        self.quant, self.cold_placement = quant, cold_placement
        self.cap_blocks = -(-capacity_tokens // bs)
        self.tail_slot = n_slots + 1
        self.pool = torch.zeros((n_slots + 2, h, 2, bs, d), dtype=dt, device=dev)
        self.kmin = torch.empty((1, h, self.cap_blocks, d), dtype=dt, device=dev)
        self.kmax = torch.empty_like(self.kmin)
        self.logical_pair_bytes = 2 * bs * d * self.pool.element_size()
        shape = (self.cap_blocks, h, 2, bs, d) if quant is None else (self.cap_blocks, h, packed_pair_bytes(bs, d))
        want = dt if quant is None else torch.uint8
        if host is None:
            host = pinned_empty(shape, want)
        elif tuple(host.shape) != shape or host.dtype != want or not host.is_pinned():
            raise ValueError(f"host pool must be pinned {want} with shape {shape}, got {host.dtype} {tuple(host.shape)}")
        self.host = host
        self.host_dev = device_view(host)  # the pinned store as kernels see it (zero-copy)
        # The store the exact pass and the fetches read: the pinned store itself (zero-copy), or a
        # device copy written alongside it.
        self.dev_store = torch.empty(shape, dtype=want, device=dev) if cold_placement == "device" else None
        self.store = self.dev_store if self.dev_store is not None else self.host_dev
        self.pair_bytes = self.logical_pair_bytes if quant is None else packed_pair_bytes(bs, d)

    def _finish(self, n_blocks: int, fill: int, seed: int) -> None:
        h, dev = self.h, self.pool.device
        self.n_sealed, self.fill, self.length = n_blocks, fill, n_blocks * self.bs + fill
        recent = torch.arange(n_blocks - seed, n_blocks, device=dev, dtype=torch.int32)
        ns = max(self.n_slots, 1)
        self._slot_block = torch.full((h, ns), -1, dtype=torch.int32, device=dev)
        self._block_slot = torch.full((h, self.cap_blocks), -1, dtype=torch.int32, device=dev)
        self._last_used = torch.full((h, ns), -2, dtype=torch.int64, device=dev)
        self._evicted_at = torch.full((h, self.cap_blocks), NEVER, dtype=torch.int64, device=dev)
        if seed > 0:
            self._slot_block[:, :seed] = recent
            self._block_slot[:, n_blocks - seed : n_blocks] = torch.arange(1, seed + 1, device=dev, dtype=torch.int32)
            self._last_used[:, :seed] = -1
        k2 = self.k + 2
        self.hot_list = torch.zeros((h, k2), dtype=torch.int32, device=dev)  # pool slots: sink, selected, current
        self.hot_list[:, -1] = self.tail_slot
        self.chosen = torch.zeros((h, self.k), dtype=torch.int32, device=dev)
        self.words = K.bitmap_words(self.cap_blocks + 1)
        self.bitmap = torch.zeros((h, self.words), dtype=torch.int32, device=dev)
        self.miss_blk = torch.zeros((h, self.k), dtype=torch.int32, device=dev)
        self.miss_slot = torch.zeros((h, self.k), dtype=torch.int32, device=dev)
        self.n_miss = torch.zeros((h,), dtype=torch.int32, device=dev)
        self.fetched_total = torch.zeros((), dtype=torch.int64, device=dev)
        self.ends = torch.tensor([0, self.tail_slot], dtype=torch.int32, device=dev).repeat(h, 1).contiguous()  # sink, current
        self.out: torch.Tensor | None = None  # [hq, d] float32, allocated on first use
        self.out_q: torch.Tensor | None = None  # [hq, d] in the query dtype: the fused exact call writes it
        self.lse: torch.Tensor | None = None

    # -- residency tables, as numpy copies (synchronising) -----------------------------------------

    def _get(self, t: torch.Tensor) -> np.ndarray:
        ev = self.__dict__.get("_split_ev")
        if ev is not None:
            L.lib().lkv_split_wait(ev)  # an admit beside the attention may still be writing the tables
        return t.cpu().numpy()

    # -- the admit beside the attention (exact tier, resident split) ---------------------------------

    admit_stream: torch.cuda.Stream | None = None  # set by the cache: the exact pass attends before the admit

    def _split_events(self) -> ctypes.c_void_p:
        """The library-owned events (lkv_split_events) that order this layer's admits beside its
        attentions; made on first use, with the tier's device current."""
        ev = self.__dict__.get("_split_ev")
        if ev is None:
            ev = ctypes.c_void_p()
            with torch.cuda.device(self.pool.device):
                rc = L.lib().lkv_split_events_create(ctypes.byref(ev))
            if rc != 0:
                raise L.LkvError(f"lkv_split_events_create failed ({rc}): {L.last_error()}")
            self._split_ev = ev
            weakref.finalize(self, L.lib().lkv_split_events_destroy, ev.value)
        return ev

    def join_admit(self) -> None:
        """The current stream waits for this layer's last admit beside the attention (tables, slots
        and the fetch counter it writes)."""
        ev = self.__dict__.get("_split_ev")
        if ev is not None:
            rc = L.lib().lkv_split_join(ev, L.stream_handle(self.pool.device))
            if rc != 0:
                raise L.LkvError(f"lkv_split_join failed ({rc}): {L.last_error()}")

    def _resident_listing(self) -> None:
        """For a selection loaded into self.chosen: the hot list gets each chosen block's slot, or -1
        where it is not resident, and the bitmap marks only the resident ones (what
        lkv_quest_topk_resident writes for its own selection)."""
        slots = torch.gather(self._block_slot, 1, self.chosen.long())
        resident = slots >= 1
        self.hot_list[:, 1 : self.k + 1] = torch.where(resident, slots, -1)
        K.mark_blocks(torch.where(resident, self.chosen, -1), self.bitmap)

    @property
    def slot_block(self) -> np.ndarray:
        return self._get(self._slot_block)[:, : self.n_slots]

    @property
    def block_slot(self) -> np.ndarray:
        return self._get(self._block_slot)

    @property
    def last_used(self) -> np.ndarray:
        return self._get(self._last_used)[:, : self.n_slots]

    @property
    def evicted_at(self) -> np.ndarray:
        return self._get(self._evicted_at)

    def set_tables(self, slot_block: np.ndarray | None = None, block_slot: np.ndarray | None = None, last_used: np.ndarray | None = None) -> None:
        """Overwrite residency tables from host arrays (tests and tooling)."""
        for src, dst in ((slot_block, self._slot_block), (block_slot, self._block_slot), (last_used, self._last_used)):
            if src is not None:
                dst[:, : src.shape[1]].copy_(torch.from_numpy(np.ascontiguousarray(src)).to(dst.dtype))

    # -- writes (tiered.py:306-375) ---------------------------------------------------------------

    def _write_tokens(self, keys: torch.Tensor, values: torch.Tensor, counters: TierCounters) -> None:
        """Tokens [1, h, T, d] into the current block, in spans that fit it. A full block is sealed
        lazily, when the next token needs its space (tiered.py:306-334), so the block being filled
        is always the pool's current slot."""
        done, total = 0, keys.shape[2]
        while done < total:
            if self.fill == self.bs:
                self._seal(counters)
            span = min(self.bs - self.fill, total - done)
            dst = self.pool[self.tail_slot, :, :, self.fill : self.fill + span]  # [h, 2, span, d]
            for half, src in enumerate((keys, values)):
                dst[:, half].copy_(src[0, :, done : done + span])
            self.fill += span
            self.length += span
            done += span

    def append(self, key: torch.Tensor, value: torch.Tensor, counters: TierCounters) -> None:
        """One decode token's KV [1, h, 1, d]: one launch writes both halves into the current block
        (lkv_append_tokens); KV of another dtype goes through the converting copies."""
        pool = self.pool
        if key.dtype != pool.dtype or value.dtype != pool.dtype or key.stride(-1) != 1 or value.stride(-1) != 1 or key.device != pool.device:
            self._write_tokens(key, value, counters)
            return
        if self.fill == self.bs:
            self._seal(counters)
        fast = self.__dict__.get("_append_args")
        if fast is None:
            fast = self._append_args = (L.lib().lkv_append_tokens, L.dtype_code(pool.dtype), pool[self.tail_slot].data_ptr())
        fn, code, tail = fast
        rc = fn(key.data_ptr(), key.stride(1), key.stride(2), value.data_ptr(), value.stride(1), value.stride(2), self.h, 1, self.d, code, tail,
                self.bs, self.fill, L.stream_handle(pool.device))
        if rc != 0:
            raise L.LkvError(f"lkv_append_tokens failed ({rc}): {L.last_error()}")
        self.fill += 1
        self.length += 1

    def tail_views(self) -> tuple[torch.Tensor, torch.Tensor]:
        """The current block's keys and values [1, h, bs, d] as views of the pool (what update()
        returns for a decode token; the device attention never reads them)."""
        views = self.__dict__.get("_tail_views")
        if views is None:
            t = self.tail_slot
            views = self._tail_views = (self.pool[t : t + 1, :, 0], self.pool[t : t + 1, :, 1])
        return views

    def extend(self, keys: torch.Tensor, values: torch.Tensor, counters: TierCounters) -> None:
        """A multi-token forward's KV [1, h, T, d], as T appends would write it."""
        self._write_tokens(keys, values, counters)

    def dense_kv(self, keys: torch.Tensor, values: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor, int]:
        """The layer's whole KV from the host store, then the tail and `keys`/`values` (bf16 tier)."""
        if self.quant is not None:
            raise NotImplementedError("dense ingestion is implemented for the bf16 tier only")
        n = self.n_sealed
        g = self.host[:n].to(keys.device, non_blocking=True).permute(1, 2, 0, 3, 4).reshape(self.h, 2, n * self.bs, self.d)
        tail = self.pool[self.tail_slot, :, :, : self.fill]
        k = torch.cat([g[:, 0], tail[:, 0], keys[0]], dim=1).unsqueeze(0)
        v = torch.cat([g[:, 1], tail[:, 1], values[0]], dim=1).unsqueeze(0)
        return k, v, n * self.h * self.pair_bytes

    def _seal(self, counters: TierCounters) -> None:
        b = self.n_sealed
        if b >= self.cap_blocks:
            raise RuntimeError(f"host pool full: {self.cap_blocks} blocks")
        tail = self.pool[self.tail_slot : self.tail_slot + 1]  # [1, h, 2, bs, d]
        if self.quant is None:
            self.host[b].copy_(tail[0], non_blocking=True)
            if self.dev_store is not None:
                self.dev_store[b].copy_(tail[0])
            K.block_minmax(tail[0, :, 0], self.bs, self.kmin[0], self.kmax[0], first_block=b)
        else:
            K.pack_int8(tail, records=self.host_dev[b : b + 1], kmin=self.kmin[0], kmax=self.kmax[0], first_block=b)
            if self.dev_store is not None:
                self.dev_store[b].copy_(self.host_dev[b])
        self.n_sealed += 1
        self.fill = 0
        counters.seals += 1
        counters.seal_bytes += self.h * self.pair_bytes

    # -- the device decode step ------------------------------------------------------------------------

    def candidates(self) -> tuple[int, int]:
        """(n_full, fill): blocks 1..n_full-1 are selectable, block n_full is the current one."""
        return self.n_sealed, self.fill

    def choose(self, query: torch.Tensor, bitmap: bool = False) -> torch.Tensor:
        """Top-K block ids [h, K] on the device (ascending id), optionally marking the bitmap."""
        n_full, _ = self.candidates()
        K.quest_topk(query, self.kmin[0], self.kmax[0], 1, n_full - 1, self.k, out_blocks=self.chosen, bitmap=self.bitmap if bitmap else None,
                     by_block=True)
        return self.chosen

    def choose_and_admit(self, query: torch.Tensor, step: int, bitmap: bool = False) -> torch.Tensor:
        """choose() then admit_device() in one library call (lkv_quest_topk_admit)."""
        n_full, _ = self.candidates()
        K.quest_topk_admit(query, self.kmin[0], self.kmax[0], 1, n_full - 1, self.k, self.chosen, self.bitmap if bitmap else None, self._block_slot,
                           self._slot_block, self._last_used, self._evicted_at, step, self.store, self.pool, self.miss_blk, self.miss_slot,
                           self.n_miss, slots_out=self.hot_list[:, 1 : self.k + 1], miss_total=self.fetched_total)
        return self.chosen

    def prefetch_device(self, query: torch.Tensor, step: int, prefetched_total: torch.Tensor) -> None:
        """The layer-ahead prefetch of this layer (tiered.py:749-798), on the current stream: the
        selection a speculated query makes, admitted (misses fetched into slots) with the step's
        LRU stamp, so that the real selection finds those blocks resident. Its own buffers and
        selection workspace, as it runs on a side stream beside the previous layer."""
        if getattr(self, "spec_chosen", None) is None:
            dev = self.pool.device
            self.spec_chosen = torch.zeros((self.h, self.k), dtype=torch.int32, device=dev)
            self.spec_miss_blk = torch.zeros((self.h, self.k), dtype=torch.int32, device=dev)
            self.spec_miss_slot = torch.zeros((self.h, self.k), dtype=torch.int32, device=dev)
            self.spec_n_miss = torch.zeros((self.h,), dtype=torch.int32, device=dev)
            self.spec_bitmap = torch.zeros((self.h, self.words), dtype=torch.int32, device=dev)
            self.spec_lane = torch.arange(self.k, device=dev, dtype=torch.int32)
        n_full, _ = self.candidates()
        K.quest_topk(query, self.kmin[0], self.kmax[0], 1, n_full - 1, self.k, out_blocks=self.spec_chosen, by_block=True, ws_slot=PREFETCH_WS_SLOT)
        K.tier_admit(self.spec_chosen, self._block_slot, self._slot_block, self._last_used, self._evicted_at, step, self.store, self.pool,
                     self.spec_miss_blk, self.spec_miss_slot, self.spec_n_miss, miss_total=prefetched_total)
        self.pending_prefetch = True

    def count_prefetch_used(self, used_total: torch.Tensor) -> None:
        """After the real selection (self.chosen): adds to `used_total` the pairs the pending
        prefetch fetched that it chose (tiered.py:731-734), on the device."""
        K.mark_blocks(self.chosen, self.spec_bitmap)
        blk = self.spec_miss_blk
        words = torch.gather(self.spec_bitmap, 1, (blk >> 5).long())
        hit = ((words >> (blk & 31)) & 1).bool() & (self.spec_lane[None, :] < self.spec_n_miss[:, None])
        used_total += hit.sum()
        self.pending_prefetch = False

    def admit_device(self, step: int) -> None:
        """Device-side admit of self.chosen and the fetch of its misses; fills the hot list."""
        K.tier_admit(self.chosen, self._block_slot, self._slot_block, self._last_used, self._evicted_at, step, self.store, self.pool,
                     self.miss_blk, self.miss_slot, self.n_miss, slots_out=self.hot_list[:, 1 : self.k + 1], miss_total=self.fetched_total)

    def load_chosen(self, chosen: np.ndarray, bitmap: bool = False) -> None:
        """A selection made elsewhere (a recorded one, replayed) into self.chosen, and into the
        bitmap the cold pass skips when `bitmap`. The ids [h, K] must be distinct candidates
        (1..n_full-1) per head. The upload goes through a pinned stage that is rewritten only after
        the previous step's copy from it has completed, so the host may run steps ahead."""
        arr = np.asarray(chosen)
        n_full, _ = self.candidates()
        if arr.shape != (self.h, self.k):
            raise ValueError(f"a selection of this layer is [{self.h}, {self.k}] block ids, got {list(arr.shape)}")
        if arr.size and (arr.min() < 1 or arr.max() >= n_full):
            raise ValueError(f"selected block ids must lie in 1..{n_full - 1}")
        if any(len(np.unique(row)) != self.k for row in arr):
            raise ValueError("a head's selected block ids must be distinct")
        stage, ev = getattr(self, "_stage", None), getattr(self, "_stage_done", None)
        if stage is None:
            stage = self._stage = torch.empty((self.h, self.k), dtype=torch.int32, pin_memory=True)
        if ev is not None:
            ev.synchronize()  # the last copy out of the stage has finished
        stage.numpy()[:] = arr
        self.chosen.copy_(stage, non_blocking=True)
        ev = self._stage_done = torch.cuda.Event()
        ev.record()
        if bitmap:
            K.mark_blocks(self.chosen, self.bitmap)

    def attend(self, query: torch.Tensor, scale: float, step: int, exact: bool, zerocopy: bool = False,
               out_dtype: torch.dtype = torch.float32, chosen: np.ndarray | None = None) -> torch.Tensor:
        """One decode step of this layer on the device; returns out [hq, d] float32, or in `out_dtype`
        (bf16 or float32) from the exact tier's fused call, which then writes that dtype directly.
        `chosen` [h, K] replaces the step's selection (a replayed one): it is loaded, admitted and
        attended exactly as the device selection's own choice would be."""
        hq, d = query.shape[1], self.d
        if self.out is None or self.out.shape != (hq, d):
            self.out = torch.empty((hq, d), dtype=torch.float32, device=query.device)
            self.lse = torch.empty((hq,), dtype=torch.float32, device=query.device)
        if out_dtype == torch.float32:
            self.out_q = self.out
        elif self.out_q is None or self.out_q.shape != (hq, d) or self.out_q.dtype != out_dtype:
            self.out_q = torch.empty((hq, d), dtype=out_dtype, device=query.device)
        pool_strides = (self.h * 2 * self.bs * d, 2 * self.bs * d, d)
        if zerocopy:
            if chosen is not None:
                raise ValueError("the zero-copy fetch has no residency to replay")
            self.choose(query, bitmap=exact)
            return self._attend_zerocopy(query, scale, exact, pool_strides)
        split = exact and self.admit_stream is not None
        if chosen is not None:
            if split:
                self.join_admit()  # the last admit beside the attention still reads self.chosen
            self.load_chosen(chosen, bitmap=exact and not split)
            if not split:
                self.admit_device(step)
        if exact:  # choose_and_admit, then K.exact_attention into out_q: the two calls, argument lists cached
            return self._exact_step(query, scale, step, selected=chosen is not None)
        if chosen is None:
            self.choose_and_admit(query, step, bitmap=exact)
        K.hot_attention(query, self.pool, self.pool[:, :, 1], pool_strides, self.hot_list, self.fill, scale, self.bs, out=self.out, lse=self.lse)
        return self.out

    def _exact_step(self, query: torch.Tensor, scale: float, step: int, selected: bool = False) -> torch.Tensor:
        """choose_and_admit then the fused exact attention, as two library calls whose argument
        lists are built once per (query shape, dtype, sealed count) and only patched per step (the
        query's address, the step, the current block's fill, the stream): a decode step's host cost
        is then little more than the two calls. Same launches and results as the wrappers.
        `selected`: the step's selection is already loaded and admitted; only the attention runs."""
        hq, d = query.shape[1], self.d
        dev = self.pool.device
        q = query.reshape(hq, d)
        if not q.is_contiguous():
            q = q.contiguous()
        key = (hq, query.dtype, self.n_sealed, self.out_q.data_ptr())
        plan = self.__dict__.get("_plan")
        # The plan holds the workspaces' addresses: it is rebuilt when the sealed count (and so the
        # sizes) changes, or when another call grew and so replaced a workspace.
        if plan is None or plan["key"] != key or K.current_workspace(dev, 1) is not plan["ws_t"][0] or K.current_workspace(dev, 0) is not plan["ws_t"][1]:
            n_cand = self.n_sealed - 1
            ws_sel = K.workspace(dev, self._ws_bytes(("sel", n_cand), lambda: int(L.lib().lkv_quest_topk_workspace(self.h, n_cand))), 1)
            n_list = self.hot_list.shape[1]
            ws_att = K.workspace(dev, self._ws_bytes(("att", hq, n_cand), lambda: int(L.lib().lkv_exact_attention_workspace(self.h, hq, d, n_list, n_cand))),
                                 0)
            plan = self._plan = self._build_plan(key, q, n_cand, ws_sel, ws_att)
            plan["ws_t"] = (ws_sel, ws_att)
        stream = L.stream_handle(dev)
        sel, att, hot = plan["sel"], plan["att"], plan["hot"]
        if self.admit_stream is not None:
            # Resident split, one library call: the selection lists the resident slots, the attention
            # covers the misses from their records, and the admit runs beside it on the admit stream.
            if selected:
                self.join_admit()
                self._resident_listing()
            args = plan["split"]
            args.q = q.data_ptr()
            args.scale = scale
            args.step = step
            args.selected = 1 if selected else 0
            hot.last_fill = self.fill
            rc = plan["split_fn"](plan["split_ref"], self._split_events(), stream, plan["side"])
            if rc != 0:
                raise L.LkvError(f"lkv_split_step failed ({rc}): {L.last_error()}")
            return self.out_q
        if not selected:
            sel[0] = q.data_ptr()
            sel[26] = step
            sel[-1] = stream
            rc = plan["sel_fn"](*sel)
            if rc != 0:
                raise L.LkvError(f"lkv_quest_topk_admit failed ({rc}): {L.last_error()}")
        hot.last_fill = self.fill
        att[0] = q.data_ptr()
        att[7] = scale
        att[-1] = stream
        rc = plan["att_fn"](*att)
        if rc != 0:
            raise L.LkvError(f"lkv_exact_attention failed ({rc}): {L.last_error()}")
        return self.out_q

    def _ws_bytes(self, key: tuple, size_of) -> int:  # noqa: ANN001
        cache = self.__dict__.setdefault("_ws_cache", {})
        v = cache.get(key)
        if v is None:
            v = cache[key] = size_of()
        return v

    def _build_plan(self, key: tuple, q: torch.Tensor, n_cand: int, ws_sel: torch.Tensor, ws_att: torch.Tensor) -> dict:
        hq, d, h = q.shape[0], self.d, self.h
        kind = L.LKV_COLD_INT8 if self.store.dtype == torch.uint8 else L.LKV_COLD_PAIRS
        kmin, kmax = self.kmin[0], self.kmax[0]
        slots = self.hot_list[:, 1 : self.k + 1]
        qd = L.dtype_code(q.dtype)
        sel = [q.data_ptr(), qd, hq, h, d, kmin.data_ptr(), kmax.data_ptr(), L.dtype_code(kmin.dtype), kmin.stride(-3), 1, n_cand, self.k, qd,
               self.chosen.data_ptr(), self.chosen.stride(0), None, self.bitmap.data_ptr(), self.bitmap.shape[-1], ws_sel.data_ptr(), ws_sel.numel(),
               self._block_slot.data_ptr(), self._block_slot.shape[1], self._slot_block.data_ptr(), self._last_used.data_ptr(),
               self._slot_block.shape[1], self._evicted_at.data_ptr(), 0, self.store.data_ptr(), kind, self.pool.data_ptr(), self.pool.shape[-2],
               L.dtype_code(self.pool.dtype), self.miss_blk.data_ptr(), self.miss_slot.data_ptr(), self.n_miss.data_ptr(), slots.data_ptr(),
               slots.stride(0), self.fetched_total.data_ptr(), 0]
        strides = (h * 2 * self.bs * d, 2 * self.bs * d, d)
        hot = L.HotSet(self.pool.data_ptr(), self.pool[:, :, 1].data_ptr(), L.dtype_code(self.pool.dtype), strides[0], strides[1], strides[2],
                       self.hot_list.data_ptr(), self.hot_list.shape[1], None, 0, self.fill,
                       K.storage_rows(self.pool, self.pool[:, :, 1], strides, h, self.bs, d))
        cold = L.ColdSet(self.store.data_ptr(), kind, 1, n_cand, self.bitmap.data_ptr(), self.bitmap.shape[-1])
        att = [q.data_ptr(), hq, h, d, self.bs, ctypes.byref(hot), ctypes.byref(cold), 1.0, self.out_q.data_ptr(), L.dtype_code(self.out_q.dtype),
               self.lse.data_ptr(), None, None,
               ws_att.data_ptr(), ws_att.numel(), 0]
        lib = L.lib()
        plan = {"key": key, "ws": (ws_sel.data_ptr(), ws_att.data_ptr()), "sel": sel, "att": att, "hot": hot, "cold": cold,
                "sel_fn": lib.lkv_quest_topk_admit, "att_fn": lib.lkv_exact_attention}
        if self.admit_stream is not None:
            # The resident split's one call (lkv_split_step): the resident selection, the attention and
            # the admit without slots_out, their arguments in one struct patched per step.
            a = L.SplitStepArgs(q=q.data_ptr(), q_dtype=qd, hq=hq, h=h, d=d, kmin=kmin.data_ptr(), kmax=kmax.data_ptr(),
                                meta_dtype=L.dtype_code(kmin.dtype), m_head=kmin.stride(-3), first_block=1, n_cand=n_cand, k=self.k,
                                bound_mode=qd, chosen=self.chosen.data_ptr(), chosen_ld=self.chosen.stride(0), block_slot=self._block_slot.data_ptr(),
                                cap=self._block_slot.shape[1], hot=slots.data_ptr(), hot_ld=slots.stride(0), bitmap=self.bitmap.data_ptr(),
                                bitmap_words=self.bitmap.shape[-1], sel_workspace=ws_sel.data_ptr(), sel_workspace_bytes=ws_sel.numel(),
                                bs=self.bs, hot_set=ctypes.addressof(hot), cold_set=ctypes.addressof(cold), scale=1.0,
                                out=self.out_q.data_ptr(), out_dtype=L.dtype_code(self.out_q.dtype), lse=self.lse.data_ptr(),
                                att_workspace=ws_att.data_ptr(), att_workspace_bytes=ws_att.numel(), slot_block=self._slot_block.data_ptr(),
                                last_used=self._last_used.data_ptr(), n_slots=self._slot_block.shape[1], evicted_at=self._evicted_at.data_ptr(),
                                step=0, store=self.store.data_ptr(), store_kind=kind, pool=self.pool.data_ptr(), pool_dtype=L.dtype_code(self.pool.dtype),
                                miss_blk=self.miss_blk.data_ptr(), miss_slot=self.miss_slot.data_ptr(), n_miss=self.n_miss.data_ptr(),
                                miss_total=self.fetched_total.data_ptr(), selected=0)
            plan.update(split=a, split_ref=ctypes.byref(a), split_fn=lib.lkv_split_step, side=self.admit_stream.cuda_stream)
        return plan

    def _attend_zerocopy(self, query: torch.Tensor, scale: float, exact: bool, pool_strides: tuple[int, int, int]) -> torch.Tensor:
        """No slots: the selected blocks are read in place from the host store, the sink and the
        current block from the pool; the partials are merged."""
        d = self.d
        o1, l1 = K.hot_attention(query, self.pool, self.pool[:, :, 1], pool_strides, self.ends, self.fill, scale, self.bs)
        if self.quant is None:
            st = self.host_dev
            o2, l2 = K.hot_attention(query, st, st[:, :, 1], (self.h * 2 * self.bs * d, 2 * self.bs * d, d), self.chosen, self.bs, scale, self.bs)
        else:
            raise ValueError("the zero-copy fetch reads bf16 blocks in place; the int8 tier needs fetch='gather'")
        parts_o, parts_l = [o1, o2], [l1, l2]
        if exact:
            o3, l3 = K.cold_attention(query, self.store, self.bs, 1, self.n_sealed - 1, scale, excluded=self.bitmap)
            parts_o.append(o3)
            parts_l.append(l3)
        K.lse_merge(torch.stack(parts_o), torch.stack(parts_l), torch.float32, out=self.out, lse_out=self.lse)
        return self.out

    def gather_zerocopy(self, query: torch.Tensor, mask_cache: dict[str, Any], bitmap: bool = False) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
        """Attention inputs read by the GPU straight from the pinned store (tiered.py:489-511): the
        selection on the device in rank order (marking the bitmap when `bitmap`), the selected pairs
        gathered through the store's device view (loads over the link), between the sink and the
        current block from the pool. No slots, no host sync; the blocks and order of gather()."""
        if self.quant is not None:
            raise ValueError("the zero-copy fetch reads bf16 blocks in place; the int8 tier needs fetch='gather'")
        n_full, _ = self.candidates()
        top, _ = K.quest_topk(query, self.kmin[0], self.kmax[0], 1, n_full - 1, self.k, out_blocks=self.chosen,
                              bitmap=self.bitmap if bitmap else None)
        dev = self.pool.device
        heads = torch.arange(self.h, device=dev)
        rows = (top.long() * self.h + heads[:, None]).reshape(-1)
        sel = self.host_dev.view(-1, 2, self.bs, self.d).index_select(0, rows).view(self.h, self.k, 2, self.bs, self.d)
        ends = self.pool[[0, self.tail_slot]].permute(1, 0, 2, 3, 4)  # [h, 2 (sink, current), 2, bs, d]
        blocks = torch.cat([ends[:, :1], sel, ends[:, 1:]], dim=1)  # [h, K + 2, 2, bs, d]
        k2 = self.k + 2
        shape = (1, self.h, k2 * self.bs, self.d)
        k_sel = blocks[:, :, 0].reshape(shape)
        v_sel = blocks[:, :, 1].reshape(shape)
        fill = self.fill
        if mask_cache.get("fill") != fill or mask_cache.get("total") != k2 * self.bs:
            mask_cache["mask"] = current_block_mask(k2 * self.bs, self.bs, fill, query.dtype, query.device)
            mask_cache["fill"], mask_cache["total"] = fill, k2 * self.bs
        return k_sel, v_sel, mask_cache["mask"]

    # -- the reference's host-facing calls (synchronising) ------------------------------------------

    def rank(self, query: torch.Tensor, bitmap: bool = False) -> np.ndarray:
        """Top-K block ids [h, K] for a query, descending bound (tiered.py:383-387), optionally
        marking them in the bitmap the cold pass skips. Syncs."""
        n_full, _ = self.candidates()
        top, _ = K.quest_topk(query, self.kmin[0], self.kmax[0], 1, n_full - 1, self.k, bitmap=self.bitmap if bitmap else None)
        return top.cpu().numpy().astype(np.int64)

    def admit(self, chosen: np.ndarray, step: int, counters: TierCounters, stream: Any = None, stage: Any = None) -> tuple[np.ndarray, np.ndarray, int]:
        """Make every (head, block) in `chosen` [h, K] resident (tiered.py:389-463), on the device.

        Returns the fetched pairs (heads, blocks) in the reference's order and the number of fetch
        launches. Synchronises to read the misses back.
        """
        ch = torch.from_numpy(np.ascontiguousarray(chosen)).to(device=self.pool.device, dtype=torch.int32)
        K.tier_admit(ch, self._block_slot, self._slot_block, self._last_used, self._evicted_at, step, self.store, self.pool,
                     self.miss_blk, self.miss_slot, self.n_miss, miss_total=self.fetched_total)
        n = self.n_miss.cpu().numpy()
        blk = self.miss_blk.cpu().numpy()
        # Head-major, chosen order within a head: the order of np.nonzero(miss) in the reference.
        mh = np.concatenate([np.full(n[j], j, dtype=np.int64) for j in range(self.h)])
        mb = np.concatenate([blk[j, : n[j]].astype(np.int64) for j in range(self.h)])
        return mh, mb, int(n.sum() > 0)

    def gather(self, chosen: np.ndarray, step: int, query: torch.Tensor, mask_cache: dict[str, Any]) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
        """Attention inputs for `chosen` after admit: sink, chosen blocks in the given order, current block."""
        slots = self.hot_list[:, 1 : self.k + 1].long()  # written by the admit
        idx = torch.cat([torch.zeros((self.h, 1), dtype=torch.long, device=slots.device), slots,
                         torch.full((self.h, 1), self.tail_slot, dtype=torch.long, device=slots.device)], dim=1)
        flat = idx * self.h + torch.arange(self.h, device=slots.device)[:, None]
        pool_flat = self.pool.view(-1, 2, self.bs, self.d)
        k2 = self.k + 2
        shape = (1, self.h, k2 * self.bs, self.d)
        k_sel = pool_flat[flat.reshape(-1), 0].view(shape)
        v_sel = pool_flat[flat.reshape(-1), 1].view(shape)
        fill = self.fill
        if mask_cache.get("fill") != fill or mask_cache.get("total") != k2 * self.bs:
            mask_cache["mask"] = current_block_mask(k2 * self.bs, self.bs, fill, query.dtype, query.device)
            mask_cache["fill"], mask_cache["total"] = fill, k2 * self.bs
        return k_sel, v_sel, mask_cache["mask"]

    # -- accounting -------------------------------------------------------------------------------------

    def gpu_bytes(self) -> int:
        return self.pool.numel() * self.pool.element_size()

    def metadata_bytes(self) -> int:
        return 2 * self.kmin.numel() * self.kmin.element_size()

    def host_bytes(self) -> int:
        return self.n_sealed * self.h * self.pair_bytes

    def not_resident_pairs(self) -> int:
        return (self.n_sealed - 1) * self.h - int((self._slot_block[:, : self.n_slots] >= 0).sum().item())

    def not_resident_bytes(self) -> int:
        return self.not_resident_pairs() * self.pair_bytes

    def not_resident_logical_bytes(self) -> int:
        return self.not_resident_pairs() * self.logical_pair_bytes


class TieredCache(Cache):
    """Decode-time cache: dense layers share the prefilled FullGPUCache, selecting layers are tiered.

    Constructor of lazykv/tiered.py:546-565 (plus `cold_placement`). The residency decision runs on
    the device. `prefetch=True` adds the reference's layer-ahead prefetch (rung 7): a pre-hook on
    each decoder layer before a selecting one speculates the next layer's query and runs its
    selection and admit on a side stream; the real selection then waits for it and finds those
    blocks resident. Outputs do not change (the attention reads the same values wherever a block
    sits); `close()` removes the hooks.
    """

    def __init__(self, full: FullGPUCache, k_blocks: int, block_size: int, capacity_tokens: int, model: PreTrainedModel | None = None,
                 prefetch: bool = False, dense_layers: int = QUEST_DENSE_LAYERS, host_pools: list[torch.Tensor] | None = None,
                 thrash_window: int = 16, instrument: bool = False, n_slots: int | None = None, fetch: str = "runs", stages: Any = None,
                 quant: str | None = None, record_selection: bool = False, replay_selection: Any = None,
                 tiers: dict[int, TieredLayer] | None = None, cold_placement: str = "host") -> None:
        super().__init__(layers=full.layers)
        if prefetch and model is None:
            raise ValueError("prefetch needs the model, to speculate the next layer's query")
        if fetch not in ("runs", "gather", "zerocopy"):
            raise ValueError(f"unknown fetch mode {fetch!r}")
        if quant is not None and fetch != "gather":
            raise ValueError(f"the int8 tier needs fetch='gather', got {fetch!r}")
        if fetch == "zerocopy":
            if prefetch or record_selection or replay_selection is not None:
                raise ValueError("the zero-copy fetch has no residency to prefetch, record or replay")
            n_slots = 0 if n_slots is None else n_slots
        if replay_selection is not None and not isinstance(replay_selection, Mapping):
            raise ValueError("replay_selection maps (layer, step) to the chosen block ids [h, K] of that step")
        # (layer, step) -> chosen block ids [h, K]; recorded as device copies, read back on demand
        # (tiered.py:620-621, 715-724). Scripts may assign both attributes directly, as the reference's do.
        self._record: dict[tuple[int, int], Any] | None = {} if record_selection else None
        self._replay: Mapping[tuple[int, int], np.ndarray] | None = replay_selection
        self.full, self.k_blocks, self.block_size, self.dense_layers = full, k_blocks, block_size, dense_layers
        self.thrash_window, self.instrument, self.quant, self.fetch = thrash_window, instrument, quant, fetch
        self.prefetch = bool(prefetch)
        self.policy_name = "tiered_int8" if quant else ("tiered_prefetch" if prefetch else ("tiered_zerocopy" if fetch == "zerocopy" else "tiered_sync"))
        self.counters = TierCounters()
        if tiers is None:
            tiers = {}
            for i in range(dense_layers, len(full.layers)):
                src = full.layers[i]
                n = src.get_seq_length()
                host = None if host_pools is None else host_pools[i - dense_layers]
                tiers[i] = TieredLayer(src.keys[:, :, :n], src.values[:, :, :n], k_blocks, block_size, capacity_tokens, host, n_slots, quant=quant,
                                       cold_placement=cold_placement)
        elif sorted(tiers) != list(range(dense_layers, len(full.layers))):
            raise ValueError(f"prebuilt tiers must cover layers {dense_layers}..{len(full.layers) - 1}, got {sorted(tiers)}")
        self.tiers: dict[int, TieredLayer] = tiers
        for layer in tiers.values():
            self.counters.boundary_d2h_s += layer.boundary_d2h_s
            self.counters.boundary_d2h_bytes += layer.boundary_d2h_bytes
        self.n_slots = next(iter(self.tiers.values())).n_slots
        # The kernels' bounded waits report to a host-mapped status word, polled once per step.
        K.status_attach(next(iter(self.tiers.values())).pool.device)
        self._mask_cache: dict[str, Any] = {}
        self._step = 0
        self._step_marks: list[torch.Tensor] = []  # device totals of fetched pairs at each step's end
        # One running count of fetched pairs for every tier, added to by the admit kernels themselves.
        self._fetched = sum(t.fetched_total for t in self.tiers.values()).clone()  # what they fetched before, if anything
        for t in self.tiers.values():
            t.fetched_total = self._fetched
        self._last_chosen: torch.Tensor | None = None
        # The layer-ahead prefetch (tiered.py:625-638): a pre-hook on decoder layer L speculates layer
        # L + 1's query and runs that layer's selection and admit on a side stream while layer L computes.
        self._hooks: list[Any] = []
        self._copy_events: dict[int, torch.cuda.Event] = {}
        self._window: dict[int, tuple[torch.cuda.Event, torch.cuda.Event, torch.cuda.Event]] = {}
        self._timed: list[tuple[torch.cuda.Event, torch.cuda.Event, torch.cuda.Event, torch.cuda.Event]] = []
        self.copy_stream: torch.cuda.Stream | None = None
        if self.prefetch:
            dev = next(iter(self.tiers.values())).pool.device
            self._prefetched = torch.zeros((), dtype=torch.int64, device=dev)
            self._prefetch_used = torch.zeros((), dtype=torch.int64, device=dev)
            self.copy_stream = torch.cuda.Stream(device=dev)
            decoder = model.model.layers  # type: ignore[union-attr]
            for src in range(max(dense_layers - 1, 0), len(decoder) - 1):
                if src + 1 in self.tiers:
                    self._hooks.append(decoder[src].register_forward_pre_hook(self._make_hook(src + 1, decoder[src + 1]), with_kwargs=True))

    # -- transformers plumbing ------------------------------------------------------------------------

    def update(self, key_states: torch.Tensor, value_states: torch.Tensor, layer_idx: int, *args: object, **kwargs: object) -> tuple[torch.Tensor, torch.Tensor]:
        if layer_idx == 0:
            self._begin_step()
        tier = self.tiers.get(layer_idx)
        if tier is None:
            return self.full.layers[layer_idx].update(key_states, value_states)
        if key_states.shape[-2] != 1:
            # A multi-token forward attends to the layer's whole KV (tiered.py:649-663).
            k, v, moved = tier.dense_kv(key_states, value_states)
            tier.extend(key_states, value_states, self.counters)
            c = self.counters
            c.ingest_forwards += 1
            c.ingest_tokens += key_states.shape[-2]
            c.ingest_h2d_bytes += moved
            return k, v
        tier.append(key_states, value_states, self.counters)
        return tier.tail_views()

    def get_seq_length(self, layer_idx: int = 0) -> int:
        tier = self.tiers.get(layer_idx)
        return tier.length if tier is not None else self.full.layers[layer_idx].get_seq_length()

    def model_kwargs(self) -> dict[str, object]:
        return {"lazykv_selector": self}

    def close(self) -> None:
        for h in self._hooks:
            h.remove()
        self._hooks.clear()
        if self._step > 0:
            self._flush_step()
            self._step = 0

    def _make_hook(self, target: int, target_layer: torch.nn.Module):  # noqa: ANN202
        """The pre-hook of the layer before `target` (tiered.py:749-798): layer target's query as it
        would be if the layer in between changed nothing (the residual stream through target's own
        norm, projection and rotary embedding), its selection and admit on the copy stream."""
        attn, norm = target_layer.self_attn, target_layer.input_layernorm

        def hook(module: torch.nn.Module, args: tuple[Any, ...], kwargs: dict[str, Any]) -> None:
            hidden = args[0] if args else kwargs["hidden_states"]
            if hidden.shape[1] != 1 or target not in self.tiers or kwargs.get("past_key_values", self) is not self:
                return  # not a decode step, or a forward over another cache
            t0 = time.perf_counter()
            tier = self.tiers[target]
            cos, sin = kwargs["position_embeddings"]
            q = attn.q_proj(norm(hidden)).view(1, 1, -1, tier.d).transpose(1, 2)
            half = tier.d // 2
            q = q * cos.unsqueeze(1) + torch.cat((-q[..., half:], q[..., :half]), dim=-1) * sin.unsqueeze(1)
            stream = self.copy_stream
            assert stream is not None
            ws = torch.cuda.Event(enable_timing=True) if self.instrument else None
            if ws is not None:
                ws.record()
            stream.wait_stream(torch.cuda.current_stream(stream.device))
            with torch.cuda.stream(stream):
                start = torch.cuda.Event(enable_timing=self.instrument)
                start.record()
                tier.prefetch_device(q, self._step, self._prefetched)
                done = torch.cuda.Event(enable_timing=self.instrument)
                done.record()
            q.record_stream(stream)
            self._copy_events[target] = done
            if ws is not None:
                self._window[target] = (ws, start, done)
            self.counters.prefetch_transfers += 1
            self.counters.host_prefetch_s += time.perf_counter() - t0

        return hook

    def _await_prefetch(self, layer_idx: int) -> None:
        """The selection below reads the tables and slots the layer's prefetch may still be writing."""
        ev = self._copy_events.pop(layer_idx, None)
        if ev is None:
            return
        win = self._window.pop(layer_idx, None)
        if win is not None:
            we = torch.cuda.Event(enable_timing=True)
            we.record()  # the compute stream reaches the target layer
            self._timed.append((win[0], win[1], win[2], we))
        torch.cuda.current_stream().wait_event(ev)

    def overlap(self) -> dict[str, Any]:
        """Measured overlap of each prefetch with the compute it was launched beside (tiered.py:
        802-830): per prefetch, its interval on the copy stream and the compute stream's interval
        from the launch until the target layer began selecting; the overlap fraction is the share
        of the prefetch inside that window, the stall how long the target layer waited for it.
        Needs `instrument=True`; synchronises the device."""
        if not self._timed:
            return {"prefetches_timed": 0}
        torch.cuda.synchronize()
        fractions, copy_ms, stall_ms, window_ms = [], [], [], []
        for ws, cs_ev, ce_ev, we_ev in self._timed:
            cs, ce, we = ws.elapsed_time(cs_ev), ws.elapsed_time(ce_ev), ws.elapsed_time(we_ev)
            dur = ce - cs
            inside = max(0.0, min(ce, we) - max(cs, 0.0))
            fractions.append(1.0 if dur <= 0 else inside / dur)
            copy_ms.append(dur)
            stall_ms.append(max(0.0, ce - we))
            window_ms.append(we)
        return {"prefetches_timed": len(self._timed), "overlap_fraction": fractions, "copy_ms": copy_ms, "stall_ms": stall_ms, "window_ms": window_ms}

    def _begin_step(self) -> None:
        # A bounded wait that ran out on the device during an earlier step poisoned that step's
        # selection; it surfaces here, without a device synchronisation.
        K.raise_on_status("TieredCache")
        if self._step > 0:
            self._flush_step()
        self._step += 1

    def _join_admits(self) -> None:
        """The current stream waits for every admit still running beside an attention."""
        for t in self.tiers.values():
            if t.admit_stream is not None:
                t.join_admit()

    def _flush_step(self) -> None:
        # The step's fetch total stays on the device until the counters are read: no host sync here.
        if self.fetch != "zerocopy":
            self._join_admits()
            self._step_marks.append(self._fetched.clone())

    # -- decode ---------------------------------------------------------------------------------------------

    exact_pass = False  # True in the exact tier: the cold blocks are attended and merged too

    def decode(self, layer_idx: int, query: torch.Tensor, key: torch.Tensor, value: torch.Tensor, scaling: float | None) -> torch.Tensor | None:
        """The whole decode step of a selecting layer on the device; out [1, Hq, 1, d] in the model dtype."""
        tier = self.tiers.get(layer_idx)
        if tier is None or query.shape[-2] != 1:
            return None
        t0 = time.perf_counter()
        scale = scaling if scaling is not None else tier.d**-0.5
        out_dtype = query.dtype if self.exact_pass and self.fetch != "zerocopy" else torch.float32
        replay = None if self._replay is None else self._replay[(layer_idx, self._step)]
        self._await_prefetch(layer_idx)
        out = tier.attend(query, scale, self._step, self.exact_pass, zerocopy=self.fetch == "zerocopy", out_dtype=out_dtype, chosen=replay)
        if getattr(tier, "pending_prefetch", False):
            tier.count_prefetch_used(self._prefetch_used)
        if self._record is not None:
            self._record[(layer_idx, self._step)] = tier.chosen.clone()  # a device copy: no host sync per step
        c = self.counters
        c.selections += 1
        c.selected_pairs += tier.h * tier.k
        if self.fetch == "zerocopy":
            c.zerocopy_bytes += tier.h * tier.k * tier.pair_bytes
        c.host_select_s += time.perf_counter() - t0
        return out.to(query.dtype).view(1, query.shape[1], 1, tier.d)

    def select(self, layer_idx: int, query: torch.Tensor, key: torch.Tensor, value: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor] | None:
        """The reference's protocol (tiered.py:694-747): gathered (key, value, mask) after the admit."""
        tier = self.tiers.get(layer_idx)
        if tier is None or query.shape[-2] != 1:
            return None
        if self.fetch == "zerocopy":
            out = tier.gather_zerocopy(query, self._mask_cache, bitmap=self.exact_pass)
            c = self.counters
            c.selections += 1
            c.selected_pairs += tier.h * tier.k
            c.zerocopy_bytes += tier.h * tier.k * tier.pair_bytes
            return out
        self._await_prefetch(layer_idx)
        if self._replay is None:
            chosen = tier.rank(query, bitmap=self.exact_pass)
            tier.chosen.copy_(torch.from_numpy(chosen).to(torch.int32))
        else:
            chosen = np.asarray(self._replay[(layer_idx, self._step)])
            tier.load_chosen(chosen, bitmap=self.exact_pass)
        if self._record is not None:
            self._record[(layer_idx, self._step)] = chosen
        tier.admit_device(self._step)
        if getattr(tier, "pending_prefetch", False):
            tier.count_prefetch_used(self._prefetch_used)
        self._last_chosen = tier.chosen.clone()
        self.counters.selections += 1
        self.counters.selected_pairs += chosen.size
        return tier.gather(chosen, self._step, query, self._mask_cache)

    def recorded_selection(self) -> dict[tuple[int, int], np.ndarray]:
        """The (layer, step) -> chosen-blocks [h, K] map a `record_selection=True` run captured
        (tiered.py:832-836). Device records are read back here (one sync), as int64 block ids:
        ascending ids from decode() (the order the device selection hands its admit), rank order
        from select(). Replaying the map through `replay_selection` repeats the run exactly."""
        if self._record is None:
            raise RuntimeError("this cache was not built with record_selection=True")
        for key, v in self._record.items():
            if isinstance(v, torch.Tensor):
                self._record[key] = v.cpu().numpy().astype(np.int64)
        return self._record

    # -- accounting --------------------------------------------------------------------------------------

    def counters_dict(self) -> dict[str, Any]:
        self._join_admits()
        if self.fetch != "zerocopy":
            marks = [int(m.item()) for m in self._step_marks]
            self.counters.fetched_pairs_per_step = [b - a for a, b in zip([0] + marks[:-1], marks)]
            total = int(self._fetched.item())
            self.counters.fetched_pairs = total
            self.counters.hit_pairs = self.counters.selected_pairs - total
            self.counters.fetch_bytes = total * next(iter(self.tiers.values())).pair_bytes
        if self.prefetch:
            self.counters.prefetched_pairs = int(self._prefetched.item())
            self.counters.prefetch_bytes = self.counters.prefetched_pairs * next(iter(self.tiers.values())).pair_bytes
            self.counters.prefetch_used_pairs = int(self._prefetch_used.item())
        return asdict(self.counters)

    def stats(self) -> CacheStats:
        dense = sum(self.full.layers[i].resident_bytes() for i in range(self.dense_layers))
        gpu = dense + sum(t.gpu_bytes() + t.metadata_bytes() for t in self.tiers.values())
        not_resident = sum(t.not_resident_bytes() for t in self.tiers.values())
        return CacheStats(seq_len=self.get_seq_length(self.dense_layers), gpu_resident_kv_bytes=gpu, host_kv_bytes=not_resident, gpu_allocated_kv_bytes=gpu)

    def host_logical_bytes(self) -> int:
        return sum(t.not_resident_logical_bytes() for t in self.tiers.values())

    def host_pinned_bytes(self) -> int:
        return sum(t.host.numel() * t.host.element_size() for t in self.tiers.values())


def allocate_stages(cap_pairs: int, heads: int, head_dim: int, block_size: int, dtype: torch.dtype = torch.bfloat16,
                    quant: str | None = None) -> tuple[None, None]:
    """The reference's gather-mode staging buffers (tiered.py:863-871), for drop-in calls: the
    device admit fetches with loads from the store, with no host-side gather or staging copy, so
    there is nothing to allocate; TieredCache accepts the returned pair as `stages` and ignores it."""
    del cap_pairs, heads, head_dim, block_size, dtype, quant
    return None, None


def allocate_host_pools(n_layers: int, heads: int, head_dim: int, block_size: int, capacity_tokens: int, dtype: torch.dtype = torch.bfloat16,
                        quant: str | None = None) -> list[torch.Tensor]:
    """Exact-size pinned host stores, one per selecting layer (tiered.py:874-882)."""
    blocks = -(-capacity_tokens // block_size)
    shape, dt = ((blocks, heads, 2, block_size, head_dim), dtype) if quant is None else ((blocks, heads, packed_pair_bytes(block_size, head_dim)), torch.uint8)
    return [pinned_empty(shape, dt) for _ in range(n_layers)]

