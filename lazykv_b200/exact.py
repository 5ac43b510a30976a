"""Exact attention over the tier: the API of lazykv/exact.py, with the cold pass on the GPU.

The reference attends to the blocks the GPU did not gather on the CPU, over a float32 mirror, and
merges the two partials by their log-sum-exp (exact.py:69-127, :225-264). Here the cold pass reads
the cold tier where it lives (pinned host memory through zero-copy loads, or a device copy), with
int8 records dequantised in the kernel, and the hot pass, the cold pass and the merge are one launch
(lkv_exact_attention). The set split is the reference's: hot = sink + the K selected blocks + the
current block; cold = every other sealed block (exact.py:116-123).

Unlike the reference, an int8 cold tier is allowed (the reference refuses it, exact.py:165-168):
every sealed block except the sink is then attended as unpack(record) in the model dtype, whether a
fetch put it in a slot or the cold pass dequantises it from the record, which is the reference's
rule for its mirror ("attends to what a fetch would have produced", exact.py:189-192); the result
does not depend on which blocks were selected beyond float32 rounding. The zero-copy fetch is
allowed too: the selection never has to reach the host.
"""

from __future__ import annotations

import time
from dataclasses import dataclass
from typing import Any

import numpy as np
import torch

from lazykv_b200 import kernels as K
from lazykv_b200.cache import FullGPUCache
from lazykv_b200.tiered import TieredCache

NEG_INF = float("-inf")


@dataclass
class ExactCounters:
    """What the exact pass costs (exact.py:56-66). There is no mirror and no CPU pass, so the mirror
    times stay 0; cpu_tokens counts the tokens the cold pass walks (the name is the reference's)."""

    merges: int = 0
    cpu_attention_s: float = 0.0
    host_merge_s: float = 0.0
    mirror_s: float = 0.0
    boundary_mirror_s: float = 0.0
    cpu_tokens: int = 0
    cold_tokens: int = 0
    returned_bytes: int = 0


def merge_lse(out_a: torch.Tensor, lse_a: torch.Tensor, out_b: torch.Tensor, lse_b: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """Combine two partial attentions [..., d] with their log-sum-exps [...] (exact.py:69-85).

    Exact for disjoint key sets; a partial with lse = -inf contributes nothing; both empty gives
    out = 0 and lse = -inf. Float32, on the device.
    """
    shape = out_a.shape
    d = shape[-1]
    outs = torch.stack([out_a.reshape(-1, d).float(), out_b.reshape(-1, d).float()])
    lses = torch.stack([lse_a.reshape(-1).float(), lse_b.reshape(-1).float()])
    out, lse = K.lse_merge(outs, lses, torch.float32)
    return out.view(shape), lse.view(lse_a.shape)


def cpu_partial_attention(keys: torch.Tensor, values: torch.Tensor, query: torch.Tensor, scaling: float, block_size: int,
                          excluded: np.ndarray) -> tuple[torch.Tensor, torch.Tensor]:
    """Attention of query [h, g, d] over keys/values [h, n_blocks * bs, d] minus `excluded` [h, e]
    block ids per head (exact.py:88-127). Same contract, computed on the GPU by the split-decode
    kernel (the name is kept for drop-in use): out [h, g, d] and lse [h, g] float32; a head with
    nothing left gets out = 0 and lse = -inf. Every head must keep the same number of blocks."""
    h, total, d = keys.shape
    g = query.shape[1]
    n_blocks = total // block_size
    keep = [np.setdiff1d(np.arange(n_blocks), np.asarray(excluded[j])) for j in range(h)]
    n_keep = {len(x) for x in keep}
    if len(n_keep) != 1:
        raise ValueError("every KV head must exclude the same number of blocks")
    if n_keep.pop() == 0:
        return torch.zeros((h, g, d), device=keys.device), torch.full((h, g), NEG_INF, device=keys.device)
    blocks = torch.from_numpy(np.stack(keep).astype(np.int32)).to(keys.device)
    k, v = keys.contiguous(), values.contiguous()
    q = query.reshape(h * g, d).to(k.dtype)
    out, lse = K.hot_attention(q, k, v, (block_size * d, total * d, d), blocks, block_size, scaling, block_size)
    return out.view(h, g, d), lse.view(h, g)


class ExactTieredCache(TieredCache):
    """Rung 9 on the device: the tier of TieredCache, made exact by attending to every cold block.

    Constructor of lazykv/exact.py:164 (`mirrors` and `threads` are accepted for drop-in calls and
    unused: there is no host mirror and no CPU pass). A prefetch is refused, as in the reference.

    `resident_split=True` (an addition): each decode step selects with the resident slots listed
    (lkv_quest_topk_resident), attends at once, the chosen blocks not resident yet from their cold
    records, and runs the admit and the fetch of the misses beside the attention on a second stream.
    The attention then no longer waits for the admit. Outputs equal the admit-first order's within
    float32 rounding, but which blocks come from slots and which from records depends on residency,
    so the last bits do too: a session restored from a snapshot (which reseeds residency) continues
    bit for bit only with the default admit-first order.
    """

    exact_pass = True

    def __init__(self, full: FullGPUCache, *args: Any, mirrors: Any = None, threads: int | None = 8, resident_split: bool = False,
                 **kwargs: Any) -> None:
        if kwargs.get("prefetch"):
            raise ValueError("rung 9 does not prefetch; the cold set is attended, not fetched")
        super().__init__(full, *args, **kwargs)
        self.policy_name = "tiered_exact" if self.quant is None else "tiered_exact_int8"
        self.exact = ExactCounters()
        self.threads = threads
        self.mirrors: dict[int, Any] = {}
        self.resident_split = bool(resident_split) and self.fetch != "zerocopy" and all(t.h <= 64 for t in self.tiers.values())
        if self.resident_split:
            stream = torch.cuda.Stream(device=next(iter(self.tiers.values())).pool.device)
            for t in self.tiers.values():
                t.admit_stream = stream

    def _count(self, layer_idx: int) -> None:
        tier = self.tiers[layer_idx]
        c = self.exact
        c.merges += 1
        c.cpu_tokens += (tier.n_sealed - 1) * tier.bs * tier.h
        c.cold_tokens += (tier.n_sealed - 1 - tier.k) * tier.bs * tier.h

    def decode(self, layer_idx: int, query: torch.Tensor, key: torch.Tensor, value: torch.Tensor, scaling: float | None) -> torch.Tensor | None:
        out = super().decode(layer_idx, query, key, value, scaling)
        if out is not None:
            self._count(layer_idx)
        return out

    def merge(self, layer_idx: int, query: torch.Tensor, key: torch.Tensor, out: torch.Tensor, scaling: float | None,
              mask: torch.Tensor | None) -> torch.Tensor:
        """Fold the cold blocks into `out`, attention over the gathered set alone (exact.py:225-264).

        For callers of the select/attend protocol: the gathered set's lse is recomputed from `key`
        in float32 (exact.py:380-393); the cold partial comes from the cold pass on the device, over
        the blocks select() did not mark in the tier's bitmap.
        """
        tier = self.tiers.get(layer_idx)
        if tier is None or query.shape[-2] != 1:
            return out
        t0 = time.perf_counter()
        scale = scaling if scaling is not None else tier.d**-0.5
        n_q, h = query.shape[1], tier.h
        q = query.view(1, h, n_q // h, tier.d).float()
        scores = torch.matmul(q, key.float().transpose(-1, -2)) * scale
        if mask is not None:
            scores = scores + mask.float().view(1, 1, 1, -1)
        lse_gpu = torch.logsumexp(scores, dim=-1).view(n_q)
        cold, cold_lse = K.cold_attention(query, tier.store, tier.bs, 1, tier.n_sealed - 1, scale, excluded=tier.bitmap, dtype=query.dtype)
        merged, _ = merge_lse(out[0, :, 0].float(), lse_gpu, cold, cold_lse)
        self._count(layer_idx)
        self.exact.host_merge_s += time.perf_counter() - t0
        return merged.to(out.dtype).view(1, n_q, 1, tier.d)

    def mirror_bytes(self) -> int:
        """Host RAM the exactness costs on top of the tier's stores: none, there is no mirror."""
        return 0

    def exact_counters_dict(self) -> dict[str, Any]:
        d = dict(self.exact.__dict__)
        d["threads"] = self.threads
        d["mirror_bytes"] = self.mirror_bytes()
        return d


def allocate_mirrors(*args: Any, **kwargs: Any) -> list[Any]:
    """The reference's float32 host mirrors (exact.py:412-418) have no role here: nothing to allocate."""
    return []
