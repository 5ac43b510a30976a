"""Layer-major prefill straight into the tier (lazykv/tiered_prefill.py:69-130).

All chunks run through layer L before layer L+1, so only one layer's prompt KV is in VRAM at a
time; when a selecting layer finishes, its KV goes to TieredLayer (pack or copy into the host store,
metadata and seeded slots on the device) and the scratch buffer is reused. Every kernel sees the
same chunk boundaries and KV prefix as a chunk-major prefill, so the KV and the last logits match
the FullGPUCache path bit for bit.
"""

from __future__ import annotations

import time
from dataclasses import dataclass, field

import torch
from transformers import PreTrainedModel
from transformers.cache_utils import Cache

from lazykv_b200.cache import FullGPUCache, PreallocatedLayer
from lazykv_b200.selection import QUEST_DENSE_LAYERS
from lazykv_b200.tiered import TieredCache, TieredLayer


class _OneLayerCache(Cache):
    """Routes each layer's update: dense layers to `full`, the selecting layer being run to `scratch`."""

    def __init__(self, full: FullGPUCache, scratch: PreallocatedLayer, dense_layers: int) -> None:
        super().__init__(layers=full.layers)
        self.full, self.scratch, self.dense_layers = full, scratch, dense_layers

    def update(self, key_states: torch.Tensor, value_states: torch.Tensor, layer_idx: int, *args: object, **kwargs: object) -> tuple[torch.Tensor, torch.Tensor]:
        store = self.full.layers[layer_idx] if layer_idx < self.dense_layers else self.scratch
        return store.update(key_states, value_states)


@dataclass
class TieredPrefillResult:
    last_logits: torch.Tensor  # [vocab] float32
    cache: TieredCache
    full: FullGPUCache
    wall_s: float
    chunks: int
    boundary_s: float
    layer_s: list[float] = field(default_factory=list)


@torch.inference_mode()
def tiered_prefill(model: PreTrainedModel, input_ids: torch.Tensor, chunk_size: int, k_blocks: int, block_size: int, capacity_tokens: int,
                   dense_layers: int = QUEST_DENSE_LAYERS, host_pools: list[torch.Tensor] | None = None, n_slots: int | None = None,
                   quant: str | None = None, cache_cls: type[TieredCache] = TieredCache, cold_placement: str = "host",
                   **cache_kwargs: object) -> TieredPrefillResult:
    """Prefill `input_ids` layer by layer and return a decode-ready tiered cache (`cache_cls`)."""
    inner = model.model
    layers = inner.layers
    ids = input_ids.to(model.device).view(1, -1)
    n = ids.shape[1]
    if n > capacity_tokens:
        raise ValueError(f"prompt of {n} tokens exceeds capacity {capacity_tokens}")
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    full = FullGPUCache(len(layers), capacity_tokens)
    scratch = PreallocatedLayer(n)
    router = _OneLayerCache(full, scratch, dense_layers)
    bounds = [(s, min(n, s + chunk_size)) for s in range(0, n, chunk_size)]
    hidden = inner.embed_tokens(ids)
    rope = []
    for s, e in bounds:
        pos = torch.arange(s, e, device=ids.device).unsqueeze(0)
        rope.append((pos, inner.rotary_emb(hidden[:, s:e], position_ids=pos)))
    tiers: dict[int, TieredLayer] = {}
    layer_s: list[float] = []
    boundary_s = 0.0
    for i, layer in enumerate(layers):
        tl = time.perf_counter()
        scratch.reset()
        for (s, e), (pos, pe) in zip(bounds, rope):
            out = layer(hidden[:, s:e], attention_mask=None, position_ids=pos, past_key_values=router, use_cache=True, position_embeddings=pe)
            hidden[:, s:e] = out[0] if isinstance(out, tuple) else out
        if i >= dense_layers:
            host = None if host_pools is None else host_pools[i - dense_layers]
            tiers[i] = TieredLayer(scratch.keys[:, :, :n], scratch.values[:, :, :n], k_blocks, block_size, capacity_tokens, host, n_slots, quant=quant,
                                   cold_placement=cold_placement)
            boundary_s += tiers[i].boundary_d2h_s
        torch.cuda.synchronize()
        layer_s.append(time.perf_counter() - tl)
    del scratch, router
    s, e = bounds[-1]
    logits = model.lm_head(inner.norm(hidden[:, s:e])[:, -1:])
    last = logits[0, -1].float()
    del hidden
    cache = cache_cls(full, k_blocks, block_size, capacity_tokens, model=model, dense_layers=dense_layers, n_slots=n_slots, quant=quant, tiers=tiers,
                      **cache_kwargs)  # type: ignore[arg-type]
    torch.cuda.synchronize()
    return TieredPrefillResult(last, cache, full, time.perf_counter() - t0, len(bounds), boundary_s, layer_s)
