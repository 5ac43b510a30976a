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
