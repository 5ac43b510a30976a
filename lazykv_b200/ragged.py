"""Ragged continuous batching: many sequences of different lengths decoded together, each through
its own block table over one paged store.

The reference decodes one sequence at a time (its tier is batch-1); this layer runs, for every
active sequence at once, what its decode step runs for one: the Quest bound and top-K over the
sequence's sealed blocks (lazykv/selection.py:38-62), the fetch of the kept blocks into HBM slots
as a fetch dequantises them (lazykv/tiered.py:429-447), and the exact attention over the hot set
[sink, kept blocks, current block] merged with the int8 cold set, every other sealed block
(lazykv/exact.py:225-264). Per sequence the result is the reference's composition of those pieces
(`oracle.restatement.tiered_decode`); the batch only changes how many launches it takes: one
selection (two kernels: scores over a flattened list of 256-candidate chunks, then one top-K CTA
per row), one fetch and one attention launch whose CTAs a host-built schedule spreads over the
rows in proportion to their blocks.

Layout (one selecting layer):
  - store: int8 records [store_blocks, h, W] in device memory, metadata kmin / kmax [h, store_blocks,
    d] over the dequantised keys; a sealed block takes any free store row;
  - block tables [max_seqs, max_blocks + 1] int32: logical block b of sequence slot s -> store row;
  - pool [max_seqs * (k_max + 2), h, 2, bs, d] in the model dtype: per sequence slot s, pool row
    s * (k_max + 2) holds the exact sink, the next k_max rows the blocks kept this step, the last
    the current (unsealed) block.
With `cold_placement="host"` the store is pinned host memory instead (written and read through
its device view); each step the records the attention reads are read over the link with mapped
loads into an HBM stage (lkv_ragged_stage_records, the zero-copy read of the cold tier of
lazykv/tiered.py:489-511), and the attention reads the stage: the same values, bit for bit.
Wherever the store lives, by default the kept blocks are attended in place: their records are
dequantised in the attention kernel exactly as a fetch would dequantise them into a slot, so the
step attends [sink, current] from the pool and every candidate block from the store (kept or not),
which is the same set of values as the hot/cold split; the selection is still computed and returned
(for a caller whose residency decides what to fetch). `decode(..., fetch=True)` runs the split as
the batch-1 tier does instead: the kept blocks are fetched into the sequence's HBM slots every step
(fetch-on-select, no cross-step LRU) and excluded from the cold pass.
"""

from __future__ import annotations

import ctypes
from dataclasses import dataclass, field

import numpy as np
import torch

from lazykv_b200 import _lib as L
from lazykv_b200 import kernels as K
from lazykv_b200._lib import call, dtype_code, ptr, require_cuda, stream_handle
from lazykv_b200.selection import blocks_for_budget

CHUNK = 256  # candidates per CTA of the ragged score kernel


def work_list(n_cand: np.ndarray) -> np.ndarray:
    """The score kernel's chunks [n, 2] int32: (row, first candidate) for every CHUNK candidates of
    each row, rows in order (a row with n candidates has ceil(n / CHUNK) chunks at 0, CHUNK, ...)."""
    n_cand = np.asarray(n_cand, dtype=np.int64)
    per_row = (n_cand + CHUNK - 1) // CHUNK
    starts = np.cumsum(per_row) - per_row
    row_of = np.repeat(np.arange(len(n_cand)), per_row)
    first = (np.arange(int(per_row.sum())) - np.repeat(starts, per_row)) * CHUNK
    return np.stack([row_of, first], axis=1).astype(np.int32)


def schedule(row_items: np.ndarray, n_sms: int) -> tuple[np.ndarray, int]:
    """The ragged attention's CTAs (lkv_ragged_schedule, host only): [n, 4] int32 rows of (row, index
    in the row, the row's CTAs, the row's first partial), and the number of partials."""
    items = np.ascontiguousarray(row_items, dtype=np.int32)
    max_ctas = int(items.sum()) // 64 + len(items) + 1
    sched = np.zeros((max_ctas, 4), dtype=np.int32)
    n_parts = ctypes.c_int(0)
    n = L.lib().lkv_ragged_schedule(items.ctypes.data, len(items), n_sms, sched.ctypes.data, max_ctas, ctypes.byref(n_parts))
    if n <= 0:
        raise L.LkvError(f"lkv_ragged_schedule failed ({n}): {L.last_error()}")
    return sched[:n], n_parts.value


@dataclass
class _Seq:
    length: int
    n_sealed: int
    fill: int
    rows: list[int] = field(default_factory=list)  # store row of each sealed block


class RaggedTier:
    """One selecting layer's KV for up to `max_seqs` sequences of up to `max_tokens` tokens each.

    `budget` is the fraction of a sequence's tokens attended from HBM: K = blocks_for_budget(budget,
    length, bs) blocks are kept per KV head (capped by its candidates).
    """

    def __init__(self, heads: int, group: int, head_dim: int, block_size: int, max_seqs: int, max_tokens: int, store_blocks: int,
                 budget: float, device: torch.device | str = "cuda", dtype: torch.dtype = torch.bfloat16, cold_placement: str = "device") -> None:
        if dtype != torch.bfloat16 or head_dim != 64 or block_size != 16 or group not in (1, 2, 4, 8):
            raise ValueError("ragged batching runs the bf16 tensor-core path: head_dim 64, block size 16, a query group of 1, 2, 4 or 8")
        if cold_placement not in ("device", "host"):
            raise ValueError(f"cold_placement is 'device' or 'host', got {cold_placement!r}")
        self.h, self.g, self.d, self.bs = heads, group, head_dim, block_size
        self.dev, self.dtype, self.budget = torch.device(device), dtype, budget
        self.max_seqs, self.max_tokens = max_seqs, max_tokens
        self.max_blocks = -(-max_tokens // block_size)
        if self.max_blocks > 16384:
            raise ValueError(f"{max_tokens} tokens is more than 16,384 blocks per sequence")
        self.k_max = blocks_for_budget(budget, max_tokens, block_size)
        self.per_seq = self.k_max + 2
        self.W = K.packed_pair_bytes(block_size, head_dim)
        self.cold_placement = cold_placement
        if cold_placement == "host":
            # The store in pinned host memory; kernels write and read it through its device view.
            from lazykv_b200.pinned import device_view, pinned_empty

            with torch.cuda.device(self.dev):
                self.records_host = pinned_empty((store_blocks, heads, self.W), torch.uint8)
                self.records = device_view(self.records_host)
            self.stage: torch.Tensor | None = None  # the step's cold records, staged in HBM
            self.stage_table = torch.full((max_seqs, self.max_blocks + 1), -1, dtype=torch.int32, device=self.dev)
        else:
            self.records = torch.zeros((store_blocks, heads, self.W), dtype=torch.uint8, device=self.dev)
        self.kmin = torch.zeros((heads, store_blocks, head_dim), dtype=dtype, device=self.dev)
        self.kmax = torch.zeros_like(self.kmin)
        self.pool = torch.zeros((max_seqs * self.per_seq, heads, 2, block_size, head_dim), dtype=dtype, device=self.dev)
        self.table = torch.full((max_seqs, self.max_blocks + 1), -1, dtype=torch.int32, device=self.dev)
        self.words = K.bitmap_words(self.max_blocks + 1)
        self._free_rows = list(range(store_blocks - 1, -1, -1))
        self._free_seqs = list(range(max_seqs - 1, -1, -1))
        self.seqs: dict[int, _Seq] = {}

    # -- sequences -----------------------------------------------------------------------------------

    def _base(self, s: int) -> int:
        return s * self.per_seq

    def _take_rows(self, n: int) -> list[int]:
        if n > len(self._free_rows):
            raise RuntimeError(f"store full: {n} blocks wanted, {len(self._free_rows)} free")
        return [self._free_rows.pop() for _ in range(n)]

    def _store(self, pairs: torch.Tensor, rows: list[int]) -> None:
        """Pack pairs [n, h, 2, bs, d] into the given store rows, with their metadata."""
        n = pairs.shape[0]
        kmin = torch.empty((self.h, n, self.d), dtype=self.dtype, device=self.dev)
        kmax = torch.empty_like(kmin)
        rec = K.pack_int8(pairs, kmin=kmin, kmax=kmax, first_block=0)
        idx = torch.tensor(rows, dtype=torch.long, device=self.dev)
        self.records[idx] = rec
        self.kmin[:, idx] = kmin
        self.kmax[:, idx] = kmax

    def add(self, keys: torch.Tensor, values: torch.Tensor) -> int:
        """A new sequence from its prefilled KV [h, L, d]; returns its slot id."""
        require_cuda(keys, values)
        h, length, d = keys.shape
        if (h, d) != (self.h, self.d) or keys.dtype != self.dtype or values.shape != keys.shape:
            raise ValueError(f"expected [{self.h}, L, {self.d}] {self.dtype} keys and values")
        if not 0 < length <= self.max_tokens or length < 2 * self.bs:
            raise ValueError(f"a sequence needs {2 * self.bs} to {self.max_tokens} tokens, got {length}")
        if not self._free_seqs:
            raise RuntimeError(f"all {self.max_seqs} sequence slots are taken")
        n, fill = divmod(length, self.bs)
        rows = self._take_rows(n)
        s = self._free_seqs.pop()
        pairs = torch.stack([keys[:, : n * self.bs], values[:, : n * self.bs]], dim=1)  # [h, 2, n*bs, d]
        pairs = pairs.unflatten(2, (n, self.bs)).permute(2, 0, 1, 3, 4).contiguous()  # [n, h, 2, bs, d]
        self._store(pairs, rows)
        self.table[s, :n] = torch.tensor(rows, dtype=torch.int32, device=self.dev)
        base = self._base(s)
        self.pool[base] = pairs[0]  # the sink stays exact in HBM
        tail = self.pool[base + self.per_seq - 1]
        tail.zero_()
        if fill:
            tail[:, 0, :fill] = keys[:, n * self.bs :]
            tail[:, 1, :fill] = values[:, n * self.bs :]
        self.seqs[s] = _Seq(length, n, fill, rows)
        return s

    def drop(self, s: int) -> None:
        """Retire sequence slot `s`: its store rows and the slot are free again."""
        seq = self.seqs.pop(s)
        self._free_rows.extend(reversed(seq.rows))
        self.table[s].fill_(-1)
        self._free_seqs.append(s)

    def append(self, s: int, key: torch.Tensor, value: torch.Tensor) -> None:
        """One decode token's KV [h, d] for sequence `s`; the current block is sealed first when full."""
        seq = self.seqs[s]
        if seq.length >= self.max_tokens:
            raise RuntimeError(f"sequence {s} is at its {self.max_tokens}-token capacity")
        tail = self.pool[self._base(s) + self.per_seq - 1]
        if seq.fill == self.bs:
            (row,) = self._take_rows(1)
            self._store(tail.unsqueeze(0), [row])
            self.table[s, seq.n_sealed] = row
            seq.rows.append(row)
            seq.n_sealed += 1
            seq.fill = 0
        tail[:, 0, seq.fill] = key
        tail[:, 1, seq.fill] = value
        seq.fill += 1
        seq.length += 1

    # -- the decode step -----------------------------------------------------------------------------

    def k_of(self, s: int) -> int:
        seq = self.seqs[s]
        return max(0, min(blocks_for_budget(self.budget, seq.length, self.bs), seq.n_sealed - 1))

    def decode(self, seq_ids: list[int], query: torch.Tensor, scale: float, fetch: bool = False) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
        """Attention of `query` [n * h * g, d] (sequence seq_ids[i]'s query heads in block i) over each
        sequence's tier: out [n * h * g, d] float32, lse [n * h * g] float32 and the kept blocks
        [n * h, k_max] (row i * h + head; entries past the row's K are unspecified)."""
        require_cuda(query)
        n, h, g = len(seq_ids), self.h, self.g
        rows = n * h
        if query.shape != (rows * g, self.d) or query.dtype != self.dtype:
            raise ValueError(f"expected query [{rows * g}, {self.d}] {self.dtype}")
        for s in seq_ids:
            if self.seqs[s].n_sealed < 2:
                raise ValueError(f"sequence {s} has no candidate block")
        dev = self.dev
        n_cand = np.array([self.seqs[s].n_sealed - 1 for s in seq_ids], dtype=np.int32).repeat(h)
        k = np.array([self.k_of(s) for s in seq_ids], dtype=np.int32).repeat(h)
        fill = np.array([self.seqs[s].fill for s in seq_ids], dtype=np.int32).repeat(h)
        # host-built arrays, uploaded together: row_sel, work, row_info, sched
        work = work_list(n_cand)
        n_hot = (k + 2) if fetch else np.full_like(k, 2)  # [sink, kept..., current] or [sink, current]
        items = (n_hot + n_cand - (k if fetch else 0)).astype(np.int32)
        sm = torch.cuda.get_device_properties(dev).multi_processor_count
        sched, n_parts = schedule(items, sm)
        n_ctas = sched.shape[0]
        row_sel = np.stack([n_cand, k], axis=1)
        row_info = np.stack([n_hot, fill, n_cand, np.zeros_like(k)], axis=1)
        seq_cand = n_cand[::h].astype(np.int64)
        stage_first = np.cumsum(seq_cand) - seq_cand  # staged row of each sequence's first candidate (host cold tier)
        host = np.concatenate([row_sel.ravel(), work.ravel(), row_info.ravel(), sched.ravel(), stage_first]).astype(np.int32)
        dmeta = torch.from_numpy(host).to(dev, non_blocking=False)
        o1 = row_sel.size
        o2 = o1 + work.size
        o3 = o2 + row_info.size
        o4 = o3 + sched.size
        d_row_sel, d_work, d_row_info, d_sched, d_stage_first = dmeta[:o1], dmeta[o1:o2], dmeta[o2:o3], dmeta[o3:o4], dmeta[o4:]
        if o2 % 4 or o3 % 4:  # 16-byte alignment of row_info and sched
            d_row_info, d_sched = d_row_info.clone(), d_sched.clone()
        sid = torch.tensor(seq_ids, dtype=torch.long, device=dev)
        table = self.table.index_select(0, sid).contiguous()  # the batch's tables, row i = seq_ids[i]
        # 1. selection
        sel = torch.empty((rows, self.k_max), dtype=torch.int32, device=dev)
        bitmap = torch.empty((rows, self.words), dtype=torch.int32, device=dev)
        max_cand = int(n_cand.max())
        ws = K.workspace(dev, L.lib().lkv_ragged_topk_workspace(rows, max_cand), slot=5)
        call("lkv_ragged_quest_topk", ptr(query), dtype_code(query.dtype), rows, g, self.d, h, ptr(self.kmin), ptr(self.kmax), dtype_code(self.dtype),
             self.kmin.stride(0), self.kmin.shape[1], ptr(table), table.stride(0), ptr(d_row_sel), max_cand, ptr(d_work), work.shape[0],
             dtype_code(self.dtype), ptr(sel), sel.stride(0), ptr(bitmap), self.words, ptr(ws), ws.numel(), stream_handle(dev))
        b_of_row = torch.arange(rows, device=dev) // h
        base = (sid * self.per_seq)[b_of_row]
        if fetch:
            # 2. fetch-on-select: kept block i of row (seq b, head j) -> pool row base(seq) + 1 + i
            kk = torch.from_numpy(k).to(dev).long()
            i = torch.arange(self.k_max, device=dev)
            last = sel.gather(1, (kk - 1).clamp(min=0)[:, None])
            blk = torch.where(i[None, :] < kk[:, None], sel, last).long()  # past K: repeat the last kept block (same copy)
            i_c = torch.minimum(i[None, :], (kk - 1).clamp(min=0)[:, None])
            head = torch.arange(rows, device=dev) % h
            src = table.long()[b_of_row[:, None], blk] * h + head[:, None]
            dst = (base[:, None] + 1 + i_c) * h + head[:, None]
            K.fetch_pairs(self.records.view(-1, self.W), src.reshape(-1).contiguous(), self.pool.view(-1, 2, self.bs, self.d),
                          dst.reshape(-1).contiguous(), self.bs, self.d)
            # 3. attention: hot list of pool rows [sink, kept..., current], the kept blocks excluded from the store pass
            hot = (base[:, None] + torch.arange(self.k_max + 2, device=dev)[None, :]).to(torch.int32)
            hot[torch.arange(rows, device=dev), kk + 1] = (base + self.per_seq - 1).to(torch.int32)
            excluded = bitmap
        else:
            # 3. attention: [sink, current] from the pool, every candidate from the store
            hot = torch.stack([base, base + self.per_seq - 1], dim=1).to(torch.int32)
            excluded = None
        hot = hot.contiguous()
        out = torch.empty((rows * g, self.d), dtype=torch.float32, device=dev)
        lse = torch.empty((rows * g,), dtype=torch.float32, device=dev)
        s_row, s_head, s_tok = h * 2 * self.bs * self.d, 2 * self.bs * self.d, self.d
        hs = L.HotSet(ptr(self.pool), ptr(self.pool[:, :, 1]), dtype_code(self.dtype), s_row, s_head, s_tok, ptr(hot), hot.shape[1], None, 0, 0,
                      self.pool.shape[0])
        ws2 = K.workspace(dev, L.lib().lkv_ragged_attention_workspace(g, n_parts), slot=6)
        records, att_table = self.records, table
        if self.cold_placement == "host":
            # 4. the records the attention reads (every candidate not in the hot set), read over the
            # link with mapped loads and staged in HBM; the attention then reads them there.
            n_stage = int(seq_cand.sum())
            if self.stage is None or self.stage.shape[0] < n_stage:
                self.stage = torch.empty((max(n_stage, 1), h, self.W), dtype=torch.uint8, device=dev)
            att_table = self.stage_table[:n]
            call("lkv_ragged_stage_records", ptr(self.records), self.records.shape[0], h, self.W, ptr(table), table.stride(0), ptr(d_work),
                 work.shape[0], ptr(d_row_info), ptr(excluded), self.words, ptr(self.stage), self.stage.shape[0], ptr(d_stage_first),
                 ptr(att_table), att_table.stride(0), stream_handle(dev))
            records = self.stage
        call("lkv_ragged_exact_attention", ptr(query), rows, g, self.d, self.bs, h, ctypes.byref(hs), ptr(records), records.shape[0],
             ptr(att_table), att_table.stride(0), ptr(excluded), self.words, ptr(d_row_info), ptr(d_sched), n_ctas, n_parts, float(scale), ptr(out),
             L.LKV_F32, ptr(lse), ptr(ws2), ws2.numel(), stream_handle(dev))
        return out, lse, sel
