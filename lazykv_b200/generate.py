"""Chunked prefill and decode drivers (the callers of the hot path, after lazykv/generate.py:97-184)."""

from __future__ import annotations

from collections.abc import Iterator
from dataclasses import dataclass

import torch
from transformers import PreTrainedModel
from transformers.cache_utils import Cache


def cache_model_kwargs(cache: Cache) -> dict[str, object]:
    fn = getattr(cache, "model_kwargs", None)
    return fn() if fn is not None else {}


@dataclass
class PrefillResult:
    last_logits: torch.Tensor  # [vocab] float32
    chunks: int


@torch.inference_mode()
def prefill(model: PreTrainedModel, cache: Cache, input_ids: torch.Tensor, chunk_size: int) -> PrefillResult:
    """Chunked prefill keeping only the last position's logits."""
    ids = input_ids.to(model.device).view(1, -1)
    logits, chunks = None, 0
    for s in range(0, ids.shape[1], chunk_size):
        out = model(input_ids=ids[:, s : s + chunk_size], past_key_values=cache, use_cache=True, logits_to_keep=1)
        logits, chunks = out.logits, chunks + 1
    assert logits is not None
    return PrefillResult(logits[0, -1].float(), chunks)


@torch.inference_mode()
def teacher_forced_decode(model: PreTrainedModel, cache: Cache, first_logits: torch.Tensor, continuation_ids: torch.Tensor) -> Iterator[torch.Tensor]:
    """Log-probs at each forced continuation position, one single-token decode step each."""
    yield torch.log_softmax(first_logits.float(), dim=-1)
    ids = torch.empty((1, 1), dtype=torch.long, device=model.device)
    extra = cache_model_kwargs(cache)
    for tok in continuation_ids.view(-1).tolist()[:-1]:
        ids.fill_(tok)
        out = model(input_ids=ids, past_key_values=cache, use_cache=True, logits_to_keep=1, **extra)
        yield torch.log_softmax(out.logits[0, -1].float(), dim=-1)


@torch.inference_mode()
def greedy_decode(model: PreTrainedModel, cache: Cache, first_logits: torch.Tensor, n_tokens: int) -> list[int]:
    tok = int(torch.argmax(first_logits).item())
    toks = [tok]
    ids = torch.empty((1, 1), dtype=torch.long, device=model.device)
    extra = cache_model_kwargs(cache)
    for _ in range(n_tokens):
        ids.fill_(tok)
        out = model(input_ids=ids, past_key_values=cache, use_cache=True, logits_to_keep=1, **extra)
        tok = int(torch.argmax(out.logits[0, -1]).item())
        toks.append(tok)
    return toks
