"""Query-aware block selection (Quest-style), on the device: the API of lazykv/selection.py.

`quest_bound` and `top_blocks` keep the reference's signatures and shapes (selection.py:38-62) but
run as one sm_100a scoring kernel plus a device-side radix top-k (`lkv_quest_topk`), so indices
never come back to the host. The bound is the reference's, max over the KV head's query group of
q+ . kmax + q- . kmin without 1/sqrt(d), computed with a fixed float32 accumulation order and, in
bf16, the same two roundings as the reference's bf16 matmuls; among equal bounds the lower block
id ranks first.
"""

from __future__ import annotations

import math

import torch

from lazykv_b200 import kernels as K

QUEST_DENSE_LAYERS = 2  # selection.py:35: the first two layers stay dense


def _bound_inputs(query: torch.Tensor, kmin: torch.Tensor, kmax: torch.Tensor, dtype: torch.dtype | None) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor, torch.dtype]:
    if dtype is not None and dtype != query.dtype:
        # The reference casts all three operands before its matmuls (selection.py:47-48).
        query, kmin, kmax = query.to(dtype), kmin.to(dtype), kmax.to(dtype)
    mode = dtype or query.dtype
    if kmin.stride(-1) != 1 or kmin.stride() != kmax.stride():
        kmin, kmax = kmin.contiguous(), kmax.contiguous()
    return query, kmin, kmax, mode


def quest_bound(query: torch.Tensor, kmin: torch.Tensor, kmax: torch.Tensor, dtype: torch.dtype | None = None) -> torch.Tensor:
    """Quest's upper bound [1, kv, n] on each candidate block's score, per KV head (selection.py:38-53).

    `query` [1, n_q, 1, d]; `kmin`/`kmax` [1, kv, n, d] over the candidate blocks.
    """
    q, mn, mx, mode = _bound_inputs(query, kmin, kmax, dtype)
    n = mn.shape[-2]
    _, bound = K.quest_topk(q, mn[0], mx[0], 0, n, 1, mode, want_bound=True)
    return bound.to(mode).unsqueeze(0)


def top_blocks(query: torch.Tensor, kmin: torch.Tensor, kmax: torch.Tensor, k: int, dtype: torch.dtype | None = None) -> torch.Tensor:
    """Indices [1, kv, k] (int64) of the k candidates with the highest bound, descending (selection.py:56-62)."""
    q, mn, mx, mode = _bound_inputs(query, kmin, kmax, dtype)
    idx, _ = K.quest_topk(q, mn[0], mx[0], 0, mn.shape[-2], k, mode)
    return idx.long().unsqueeze(0)


def current_block_mask(total: int, block_size: int, fill: int, dtype: torch.dtype, device: torch.device, reuse: torch.Tensor | None = None) -> torch.Tensor:
    """Additive mask [1, 1, 1, total] hiding the unfilled part of the current block (selection.py:65-69)."""
    mask = torch.zeros((1, 1, 1, total), dtype=dtype, device=device) if reuse is None else reuse.zero_()
    mask[..., total - block_size + fill :] = float("-inf")
    return mask


def blocks_for_budget(fraction: float, total_tokens: int, block_size: int) -> int:
    """Selected blocks K such that sink + K blocks + the current block stay within the budget (selection.py:72-74)."""
    return max(1, math.floor(fraction * total_tokens / block_size) - 2)


# -- QuestView: rung 5 over a fully resident cache (lazykv/selection.py:77-183) ---------------------

import time  # noqa: E402
from dataclasses import dataclass  # noqa: E402

from transformers.cache_utils import Cache  # noqa: E402

from lazykv_b200.cache import CacheStats, FullGPUCache  # noqa: E402


@dataclass
class SelectorCounters:
    host_select_s: float = 0.0
    selections: int = 0


class _LayerState:
    def __init__(self) -> None:
        self.kmin: torch.Tensor | None = None  # [h, cap_blocks, d]
        self.kmax: torch.Tensor | None = None
        self.n_meta = 0
        self.blocks: torch.Tensor | None = None  # [h, K + 2] hot list: sink, selected, current


class QuestView(Cache):
    """Decode-time view over a prefilled FullGPUCache that attends only to selected blocks.

    Shares the full cache's layers (decode appends to them). Per selecting layer and step: the
    metadata of newly completed blocks is computed on the device, the top-K blocks are chosen on
    the device, and `decode` attends to [sink, selected, current] in place in the cache storage
    (no gather). `select` keeps the reference's protocol and returns the gathered key set.
    """

    def __init__(self, full: FullGPUCache, k_blocks: int, block_size: int, dense_layers: int = QUEST_DENSE_LAYERS,
                 bound_dtype: torch.dtype | None = None) -> None:
        super().__init__(layers=full.layers)
        self.full, self.k_blocks, self.block_size, self.dense_layers = full, k_blocks, block_size, dense_layers
        self.bound_dtype = bound_dtype
        self.counters = SelectorCounters()
        self.policy_name = "quest" if bound_dtype is None else f"quest_{str(bound_dtype).removeprefix('torch.')}"
        self._state = [_LayerState() for _ in full.layers]
        self._mask: torch.Tensor | None = None
        self._mask_key: tuple[int, int] | None = None
        for i, layer in enumerate(full.layers):
            if getattr(layer, "is_initialized", False):
                self._refresh_metadata(i, layer.keys, layer.get_seq_length())

    def update(self, key_states: torch.Tensor, value_states: torch.Tensor, layer_idx: int, *args: object, **kwargs: object) -> tuple[torch.Tensor, torch.Tensor]:
        return self.full.layers[layer_idx].update(key_states, value_states)

    def get_seq_length(self, layer_idx: int = 0) -> int:
        return self.full.layers[layer_idx].get_seq_length()

    def model_kwargs(self) -> dict[str, object]:
        return {"lazykv_selector": self}

    def stats(self) -> CacheStats:
        return self.full.stats()

    def attended_tokens(self) -> int:
        return (self.k_blocks + 2) * self.block_size

    def _refresh_metadata(self, layer_idx: int, keys: torch.Tensor, length: int) -> None:
        st = self._state[layer_idx]
        bs = self.block_size
        n_full = length // bs
        if st.kmin is None:
            cap = -(-keys.shape[2] // bs)
            st.kmin = torch.empty((keys.shape[1], cap, keys.shape[3]), dtype=keys.dtype, device=keys.device)
            st.kmax = torch.empty_like(st.kmin)
        if n_full > st.n_meta:
            K.block_minmax(keys[0, :, st.n_meta * bs : n_full * bs], bs, st.kmin, st.kmax, first_block=st.n_meta)
            st.n_meta = n_full

    def _plan(self, layer_idx: int, query: torch.Tensor, key: torch.Tensor, by_block: bool) -> tuple[int, int, torch.Tensor] | None:
        """(n_full, fill, hot list [h, K + 2]) for this decode step, or None to attend densely.

        The selected blocks are listed in rank order, or by ascending id when `by_block` (the order
        the tier attends in, so the two give the same bits)."""
        if query.shape[-2] != 1 or layer_idx < self.dense_layers:
            return None
        bs = self.block_size
        length = key.shape[2]
        n_full, fill = divmod(length, bs)
        if fill == 0:  # the newest block just completed: it is the current block
            n_full, fill = n_full - 1, bs
        if n_full - 1 <= self.k_blocks:
            return None  # the budget covers every block: dense is exact and cheaper
        st = self._state[layer_idx]
        layer = self.full.layers[layer_idx]
        self._refresh_metadata(layer_idx, layer.keys, n_full * bs)
        h = key.shape[1]
        if st.blocks is None or st.blocks.shape != (h, self.k_blocks + 2):
            st.blocks = torch.zeros((h, self.k_blocks + 2), dtype=torch.int32, device=key.device)
        st.blocks[:, -1] = n_full
        q, mn, mx, mode = _bound_inputs(query, st.kmin, st.kmax, self.bound_dtype)
        K.quest_topk(q, mn, mx, 1, n_full - 1, self.k_blocks, mode, out_blocks=st.blocks[:, 1 : self.k_blocks + 1], by_block=by_block)
        return n_full, fill, st.blocks

    def decode(self, layer_idx: int, query: torch.Tensor, key: torch.Tensor, value: torch.Tensor, scaling: float | None) -> torch.Tensor | None:
        t0 = time.perf_counter()
        plan = self._plan(layer_idx, query, key, by_block=True)
        if plan is None:
            return None
        n_full, fill, blocks = plan
        layer = self.full.layers[layer_idx]
        bs, d = self.block_size, query.shape[-1]
        scale = scaling if scaling is not None else d**-0.5
        strides = (bs * d, layer.keys.stride(1), d)
        out, _ = K.hot_attention(query, layer.keys, layer.values, strides, blocks, fill, scale, bs)
        self.counters.host_select_s += time.perf_counter() - t0
        self.counters.selections += 1
        return out.to(query.dtype).view(1, query.shape[1], 1, d)

    def select(self, layer_idx: int, query: torch.Tensor, key: torch.Tensor, value: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor] | None:
        """Gathered (key, value, additive mask) for this decode step, or None to attend densely."""
        plan = self._plan(layer_idx, query, key, by_block=False)
        if plan is None:
            return None
        n_full, fill, blocks = plan
        bs = self.block_size
        layer = self.full.layers[layer_idx]
        idx = (blocks.long().unsqueeze(-1) * bs + torch.arange(bs, device=key.device)).flatten(1)  # [h, (K+2)*bs]
        idx = idx.unsqueeze(0).unsqueeze(-1).expand(-1, -1, -1, key.shape[-1])
        k_sel = torch.gather(layer.keys, 2, idx)
        v_sel = torch.gather(layer.values, 2, idx)
        total = (self.k_blocks + 2) * bs
        if self._mask_key != (total, fill):
            self._mask = current_block_mask(total, bs, fill, query.dtype, query.device, None)
            self._mask_key = (total, fill)
        self.counters.selections += 1
        assert self._mask is not None
        return k_sel, v_sel, self._mask
