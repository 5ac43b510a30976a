"""The attention function registered with transformers' AttentionInterface (lazykv/attention.py:139-182).

Contract of the reference's hook: no attention mask is ever passed (the function owns causality),
batch size 1, and a selector object in kwargs["lazykv_selector"]. For a decode step on a selecting
layer the selector's `decode` runs the whole hot path on the device (selection, residency, the
attention over the hot blocks and, for the exact tier, the cold pass and the merge) and returns
the output directly. A selector without `decode` goes through the reference's protocol: `select`
returns gathered (key, value, additive mask) and an optional `merge` folds in the rest. Prefill and
the dense layers attend densely with torch's scaled_dot_product_attention (lower-right causal).
"""

from __future__ import annotations

import torch
from torch.nn.attention import SDPBackend, sdpa_kernel
from torch.nn.attention.bias import causal_lower_right
from transformers import AttentionInterface

IMPLEMENTATION_NAME = "lazykv_b200"
_DECODE_BACKENDS = [SDPBackend.FLASH_ATTENTION, SDPBackend.EFFICIENT_ATTENTION, SDPBackend.MATH]


def attend(query: torch.Tensor, key: torch.Tensor, value: torch.Tensor, scaling: float | None, mask: torch.Tensor | None = None) -> torch.Tensor:
    """Exact attention of `query` over all of `key`/`value`: lower-right causal for q_len > 1 (a
    chunk's queries sit at the end of the KV), an optional additive mask for decode."""
    q_len, kv_len = query.shape[-2], key.shape[-2]
    F = torch.nn.functional.scaled_dot_product_attention
    if q_len > 1:
        return F(query, key, value, attn_mask=causal_lower_right(q_len, kv_len), scale=scaling, enable_gqa=True)
    if mask is not None:
        # A masked GQA decode falls to SDPA's math kernel, which would round the probabilities to
        # the model dtype; the gathered set is small, so it is attended in float32 instead, as the
        # device decode path does.
        return F(query.float(), key.float(), value.float(), attn_mask=mask.float(), scale=scaling, enable_gqa=True).to(query.dtype)
    # A dense decode step (the dense layers) grows the KV by one token every step: a backend that
    # builds an execution plan per shape (cuDNN's) would build one every step, so it is left out.
    with sdpa_kernel(_DECODE_BACKENDS):
        return F(query, key, value, scale=scaling, enable_gqa=True)


def lazykv_attention_forward(module: torch.nn.Module, query: torch.Tensor, key: torch.Tensor, value: torch.Tensor,
                             attention_mask: torch.Tensor | None, dropout: float = 0.0, scaling: float | None = None,
                             **kwargs: object) -> tuple[torch.Tensor, None]:
    if attention_mask is not None:
        raise RuntimeError("lazykv attention owns causality; a mask should never be passed")
    if query.shape[0] != 1:
        raise RuntimeError("batch size 1 only")
    selector = kwargs.get("lazykv_selector")
    if selector is not None and query.shape[-2] == 1:
        layer = int(getattr(module, "layer_idx"))
        decode = getattr(selector, "decode", None)
        if decode is not None:
            out = decode(layer, query, key, value, scaling)
            if out is not None:
                return out.transpose(1, 2).contiguous(), None
        chosen = selector.select(layer, query, key, value)
        if chosen is not None:
            k_sel, v_sel, mask = chosen
            out = attend(query, k_sel, v_sel, scaling, mask)
            merge = getattr(selector, "merge", None)
            if merge is not None:
                out = merge(layer, query, k_sel, out, scaling, mask)
            return out.transpose(1, 2).contiguous(), None
    return attend(query, key, value, scaling).transpose(1, 2).contiguous(), None


def install(strategy: str | None = None, n_q_heads: int | None = None, n_kv_heads: int | None = None, head_dim: int | None = None,
            bucket: int = 64) -> tuple[str, list[object]]:
    """Register the attention function; models opt in with model.set_attn_implementation(IMPLEMENTATION_NAME).

    Signature of lazykv/attention.py:269. The reference picks among several dense-attention
    strategies after verifying them; here there is one decode path (the device hot path) and one
    prefill path (SDPA), so `strategy` and `bucket` only have to name no other. Returns the
    strategy in use and an empty list of checks.
    """
    if strategy not in (None, IMPLEMENTATION_NAME, "sdpa", "cudnn_bucketed", "efficient"):
        raise RuntimeError(f"requested attention strategy {strategy!r} is not available")
    AttentionInterface.register(IMPLEMENTATION_NAME, lazykv_attention_forward)
    return IMPLEMENTATION_NAME, []
