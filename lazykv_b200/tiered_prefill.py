"""Layer-major prefill straight into the tier (the API of lazykv/tiered_prefill.py:69-130).

Every chunk of the prompt runs through layer L before any chunk reaches layer L+1, so only one
selecting layer's prompt KV is ever in VRAM: a scratch layer that the running layer attends over.
While that layer runs, its tier is written as the prompt advances: after each chunk, the blocks that
chunk completed are packed (int8) or copied (bf16) into the host store with their metadata, and the
newest ones seeded into slots (`TieredLayer.ingest`), so the boundary's work overlaps the next
chunks instead of waiting for the layer's end; after the last chunk only the sink, the unsealed tail
and the residency tables remain (`TieredLayer.close_boundary`). Each kernel sees the chunk
boundaries and KV prefix that a chunk-major prefill gives it, so the KV, the tier and the last
logits match the FullGPUCache path bit for bit.
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


class _RouteTo(Cache):
    """The cache a decoder layer sees during the layer-major pass: every update goes to one store
    (the running selecting layer's scratch, or a dense layer's own FullGPUCache layer)."""

    def __init__(self, full: FullGPUCache, store: PreallocatedLayer) -> None:
        super().__init__(layers=full.layers)
        self.store = store

    def update(self, key_states: torch.Tensor, value_states: torch.Tensor, layer_idx: int, *args: object, **kwargs: object) -> tuple[torch.Tensor, torch.Tensor]:
        return self.store.update(key_states, value_states)


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
    """Prefill `input_ids` layer by layer, writing each selecting layer's tier as its chunks complete,
    and return a decode-ready tiered cache (`cache_cls`)."""
    decoder = model.model
    ids = input_ids.to(model.device).view(1, -1)
    n = ids.shape[1]
    if n > capacity_tokens:
        raise ValueError(f"prompt of {n} tokens exceeds capacity {capacity_tokens}")
    torch.cuda.synchronize()
    t_start = time.perf_counter()
    spans = [(s, min(n, s + chunk_size)) for s in range(0, n, chunk_size)]
    full = FullGPUCache(len(decoder.layers), capacity_tokens)
    scratch = PreallocatedLayer(n)  # the running selecting layer's prompt KV
    hidden = decoder.embed_tokens(ids)
    # Positions and rotary embeddings are the same for every layer: computed once per chunk.
    chunk_inputs = []
    for s, e in spans:
        pos = torch.arange(s, e, device=ids.device).unsqueeze(0)
        chunk_inputs.append((s, e, pos, decoder.rotary_emb(hidden[:, s:e], position_ids=pos)))
    tiers: dict[int, TieredLayer] = {}
    layer_s: list[float] = []
    for i, layer in enumerate(decoder.layers):
        t_layer = time.perf_counter()
        selecting = i >= dense_layers
        if selecting:
            scratch.reset()
        route = _RouteTo(full, scratch if selecting else full.layers[i])
        tier: TieredLayer | None = None
        for s, e, pos, rope in chunk_inputs:
            out = layer(hidden[:, s:e], attention_mask=None, position_ids=pos, past_key_values=route, use_cache=True, position_embeddings=rope)
            hidden[:, s:e] = out[0] if isinstance(out, tuple) else out
            if selecting:
                if tier is None:
                    host = None if host_pools is None else host_pools[i - dense_layers]
                    tier = TieredLayer.open_boundary(scratch.keys, n, k_blocks, block_size, capacity_tokens, host, n_slots, quant=quant,
                                                     cold_placement=cold_placement)
                tier.ingest(scratch.keys, scratch.values, e)
        if tier is not None:
            tier.close_boundary(scratch.keys, scratch.values)
            tiers[i] = tier
        torch.cuda.synchronize()
        layer_s.append(time.perf_counter() - t_layer)
    del scratch
    logits = model.lm_head(decoder.norm(hidden[:, spans[-1][0] : spans[-1][1]])[:, -1:])
    last = logits[0, -1].float()
    del hidden
    cache = cache_cls(full, k_blocks, block_size, capacity_tokens, model=model, dense_layers=dense_layers, n_slots=n_slots, quant=quant, tiers=tiers,
                      **cache_kwargs)  # type: ignore[arg-type]
    torch.cuda.synchronize()
    boundary_s = sum(t.boundary_d2h_s for t in tiers.values())
    return TieredPrefillResult(last, cache, full, time.perf_counter() - t_start, len(spans), boundary_s, layer_s)
