"""Seeded synthetic inputs shared by the golden-vector script and the tests.

Everything is drawn with torch's CPU generator, which is deterministic for a given seed, so the
inputs are regenerated on any machine instead of being stored; the fixtures hold only outputs and
input checksums (`checksum`) that catch a generator change.

Conventions (restated): K and V ~ N(0, 1); keys get a per-(head, channel) mean
offset ~ N(0, 0.5), i.e. variance 0.5 (`offset * sqrt(0.5)`); the query ~ N(0, 1).
"""

from __future__ import annotations

import math

import numpy as np
import torch

HQ, HKV, D, BS = 32, 8, 64, 16  # Llama-3.2-1B attention shapes, 16-token blocks


def kv_with_offset(gen: torch.Generator, h: int, t: int, d: int) -> tuple[torch.Tensor, torch.Tensor]:
    off = torch.randn(h, 1, d, generator=gen) * math.sqrt(0.5)
    k = torch.randn(h, t, d, generator=gen) + off
    v = torch.randn(h, t, d, generator=gen)
    return k, v


def config1(seed: int = 0, t: int = 8192) -> dict[str, torch.Tensor]:
    """Config 1: one layer, fp32 K/V [8, t, 64], query [32, 64]."""
    g = torch.Generator().manual_seed(seed)
    k, v = kv_with_offset(g, HKV, t, D)
    q = torch.randn(HQ, D, generator=g)
    return {"k": k, "v": v, "q": q}


def bf16_layer(seed: int, t: int, h: int = HKV, hq: int = HQ, d: int = D) -> dict[str, torch.Tensor]:
    """One bf16 layer: K/V [h, t, d] with the key offset, query [hq, d], all rounded to bf16."""
    g = torch.Generator().manual_seed(seed)
    k, v = kv_with_offset(g, h, t, d)
    q = torch.randn(hq, d, generator=g)
    return {"k": k.bfloat16(), "v": v.bfloat16(), "q": q.bfloat16()}


def pairs_from_kv(k: torch.Tensor, v: torch.Tensor, bs: int) -> torch.Tensor:
    """[h, n*bs, d] keys/values -> [n, h, 2, bs, d] pairs, the host pool's layout."""
    h, t, d = k.shape
    n = t // bs
    x = torch.stack([k[:, : n * bs], v[:, : n * bs]], dim=1)  # [h, 2, n*bs, d]
    return x.unflatten(2, (n, bs)).permute(2, 0, 1, 3, 4).contiguous()


def checksum(x: torch.Tensor) -> np.ndarray:
    """Three numbers that change if the generator does: sum, sum of squares, a strided sample."""
    f = x.double().flatten()
    return np.array([f.sum().item(), (f * f).sum().item(), f[:: max(1, f.numel() // 97)].sum().item()])


def bf16_np(x: torch.Tensor) -> np.ndarray:
    """bf16 tensor -> its 16-bit patterns as uint16 (half the bytes of a float32 copy)."""
    return x.detach().cpu().contiguous().view(torch.int16).numpy().view(np.uint16)


def from_bf16_np(u: np.ndarray) -> np.ndarray:
    """uint16 bf16 patterns -> float32 values."""
    return (u.astype(np.uint32) << 16).view(np.float32)


def to_np(x: torch.Tensor) -> np.ndarray:
    """float32 numpy copy (bf16 values widen exactly)."""
    return x.detach().float().cpu().numpy()
