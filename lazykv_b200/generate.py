"""Chunked prefill and decode drivers (the callers of the hot path, after lazykv/generate.py:97-184)."""

from __future__ import annotations

import time
from collections.abc import Iterator
from dataclasses import dataclass, field

import torch
from transformers import PreTrainedModel
from transformers.cache_utils import Cache


def cache_model_kwargs(cache: Cache) -> dict[str, object]:
    fn = getattr(cache, "model_kwargs", None)
    return fn() if fn is not None else {}


@dataclass
class PrefillResult:
    last_logits: torch.Tensor  # [vocab] float32
    wall_s: float  # host clock around the prefill, synchronised on both sides
    event_s: float  # device time between CUDA events (0.0 on a CPU model)
    chunks: int


class _Clock:
    """Wall time and, for a CUDA model, event time of one region (both synchronised)."""

    def __init__(self, device: torch.device) -> None:
        self.cuda = device.type == "cuda"

    def __enter__(self) -> _Clock:
        if self.cuda:
            self.a, self.b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            torch.cuda.synchronize()
            self.a.record()
        self.t0 = time.perf_counter()
        return self

    def stop(self) -> tuple[float, float]:
        if self.cuda:
            self.b.record()
            torch.cuda.synchronize()
        wall = time.perf_counter() - self.t0
        return wall, (self.a.elapsed_time(self.b) / 1e3 if self.cuda else 0.0)

    def __exit__(self, *exc: object) -> None:
        return None


@torch.inference_mode()
def prefill(model: PreTrainedModel, cache: Cache, input_ids: torch.Tensor, chunk_size: int, observer: object | None = None) -> PrefillResult:
    """Chunked prefill keeping only the last position's logits (lazykv/generate.py:97-125)."""
    if observer is not None:
        raise ValueError("attention observers (prefill scoring) are not built")
    ids = input_ids.to(model.device).view(1, -1)
    logits, chunks = None, 0
    with _Clock(model.device) as clock:
        for s in range(0, ids.shape[1], chunk_size):
            out = model(input_ids=ids[:, s : s + chunk_size], past_key_values=cache, use_cache=True, logits_to_keep=1)
            logits, chunks = out.logits, chunks + 1
        assert logits is not None
        last = logits[0, -1].float()
        wall, ev = clock.stop()
    return PrefillResult(last, wall, ev, chunks)


@dataclass
class DecodeResult:
    tokens: list[int]
    wall_s: list[float] = field(default_factory=list)  # per token, host sync included
    event_s: list[float] = field(default_factory=list)  # per token, CUDA events (0.0 on a CPU model)


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
def greedy_decode(model: PreTrainedModel, cache: Cache, first_logits: torch.Tensor, n_tokens: int) -> DecodeResult:
    """Greedy decode (lazykv/generate.py:134-154): token 0 from the prefill logits, then n_tokens
    single-token steps, each timed; the token reaches the host every step, as in generation."""
    tok = int(torch.argmax(first_logits).item())
    res = DecodeResult(tokens=[tok])
    ids = torch.empty((1, 1), dtype=torch.long, device=model.device)
    extra = cache_model_kwargs(cache)
    for _ in range(n_tokens):
        ids.fill_(tok)
        with _Clock(model.device) as clock:
            out = model(input_ids=ids, past_key_values=cache, use_cache=True, logits_to_keep=1, **extra)
            nxt = torch.argmax(out.logits[0, -1])
            wall, ev = clock.stop()
        tok = int(nxt.item())
        res.wall_s.append(wall)
        res.event_s.append(ev)
        res.tokens.append(tok)
    return res


def teacher_forced_steps(model: PreTrainedModel, cache: Cache, context_ids: torch.Tensor, continuation_ids: torch.Tensor,
                         chunk_size: int) -> Iterator[torch.Tensor]:
    """Log-probs (float32) at each continuation position: row i is the distribution over
    continuation token i given the context and continuation[:i], scored through single-token
    decode steps after a chunked prefill of the context (lazykv/generate.py:157-168)."""
    pre = prefill(model, cache, context_ids, chunk_size)
    yield from teacher_forced_decode(model, cache, pre.last_logits, continuation_ids)


def teacher_forced_logprobs(model: PreTrainedModel, cache: Cache, context_ids: torch.Tensor, continuation_ids: torch.Tensor,
                            chunk_size: int) -> torch.Tensor:
    """Every row of teacher_forced_steps as one float32 CPU tensor [positions, vocab], filled in
    place (lazykv/generate.py:186-197)."""
    rows: torch.Tensor | None = None
    for i, row in enumerate(teacher_forced_steps(model, cache, context_ids, continuation_ids, chunk_size)):
        if rows is None:
            rows = torch.empty((continuation_ids.numel(), row.numel()), dtype=torch.float32)
        rows[i].copy_(row)
    assert rows is not None
    return rows
