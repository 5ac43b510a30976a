"""Full-GPU KV store for the dense layers, and the source the tier is built from at the boundary.

The API is lazykv/cache.py's (PreallocatedLayer :20-77, FullGPUCache :80-102, CacheStats
:105-115): a layer holds [1, kv_heads, max_len, head_dim] keys and values, allocated once when the
first states arrive and zero-filled, and `update` returns views of the filled prefix. Here each
layer keeps its keys and values in ONE allocation, [2, 1, h, max_len, d] (`kv`), with `keys` and
`values` as views of its two halves, so a layer is one block of device memory and its byte counts
follow from that block's shape.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch
from transformers.cache_utils import Cache, CacheLayerMixin


@dataclass(frozen=True)
class CacheStats:
    """Byte counts of a cache at one sequence length (the fields of lazykv/cache.py:105-115)."""

    seq_len: int
    gpu_resident_kv_bytes: int
    host_kv_bytes: int
    gpu_allocated_kv_bytes: int

    @property
    def gpu_residency_fraction(self) -> float:
        """Share of the KV bytes that live on the GPU (1.0 for an empty cache)."""
        stored = self.gpu_resident_kv_bytes + self.host_kv_bytes
        return self.gpu_resident_kv_bytes / stored if stored else 1.0


class PreallocatedLayer(CacheLayerMixin):
    """One layer's keys and values in a single zeroed [2, 1, h, max_len, d] block, filled in order.

    Zeroed rather than left uninitialised: a reader that runs past `length` (a padded or bucketed
    kernel) then sees finite values that a mask can hide."""

    def __init__(self, max_len: int, **kwargs: object) -> None:
        super().__init__()
        self.max_len = max_len
        self.length = 0
        self.kv: torch.Tensor | None = None

    def lazy_initialization(self, key_states: torch.Tensor, value_states: torch.Tensor) -> None:
        if key_states.shape[0] != 1 or value_states.shape[0] != 1:
            raise ValueError(f"LazyKV is batch-size-1 only (v1 scope), got batch {key_states.shape[0]}")
        if key_states.shape != value_states.shape:
            raise ValueError(f"keys {tuple(key_states.shape)} and values {tuple(value_states.shape)} differ in shape")
        _, heads, _, dim = key_states.shape
        self.dtype, self.device = key_states.dtype, key_states.device
        self.kv = torch.zeros((2, 1, heads, self.max_len, dim), dtype=key_states.dtype, device=key_states.device)
        self.keys, self.values = self.kv[0], self.kv[1]
        self.is_initialized = True

    def update(self, key_states: torch.Tensor, value_states: torch.Tensor, *args: object, **kwargs: object) -> tuple[torch.Tensor, torch.Tensor]:
        """Append [1, h, n, d] states; returns the filled prefixes [1, h, length, d]."""
        if not self.is_initialized:
            self.lazy_initialization(key_states, value_states)
        start, n = self.length, key_states.shape[-2]
        if start + n > self.max_len:
            raise RuntimeError(f"KV cache overflow: {start + n} > max_len {self.max_len}")
        for half, states in ((self.keys, key_states), (self.values, value_states)):
            half.narrow(2, start, n).copy_(states)
        self.length = start + n
        return self.keys.narrow(2, 0, self.length), self.values.narrow(2, 0, self.length)

    def get_mask_sizes(self, query_length: int) -> tuple[int, int]:
        return self.length + query_length, 0

    def get_seq_length(self) -> int:
        return self.length

    def get_max_length(self) -> int:
        return self.max_len

    def get_max_cache_shape(self) -> int:
        return self.max_len

    def reset(self) -> None:
        """Forget every token (the block is kept; only the prefix below `length` is ever read)."""
        self.length = 0

    def truncate(self, length: int) -> None:
        """Keep the first `length` tokens, so one prefill can be decoded from more than once."""
        if length < 0 or length > self.length:
            raise ValueError(f"cannot truncate length {self.length} to {length}")
        self.length = length

    def _bytes_per_token(self) -> int:
        # keys and values of every head at one position: the block's bytes over its max_len
        return 0 if self.kv is None else self.kv.numel() * self.kv.element_size() // self.max_len

    def resident_bytes(self) -> int:
        """Bytes of the filled prefix (keys and values)."""
        return self._bytes_per_token() * self.length

    def allocated_bytes(self) -> int:
        """Bytes of the whole block."""
        return self._bytes_per_token() * self.max_len


class FullGPUCache(Cache):
    """Every token of every layer on the GPU: the exact baseline, and the dense layers' store."""

    def __init__(self, num_layers: int, max_len: int) -> None:
        super().__init__(layers=[PreallocatedLayer(max_len) for _ in range(num_layers)])
        self.max_len = max_len

    def truncate(self, length: int) -> None:
        for layer in self.layers:
            layer.truncate(length)

    def stats(self) -> CacheStats:
        own = [x for x in self.layers if isinstance(x, PreallocatedLayer)]
        return CacheStats(
            seq_len=own[0].get_seq_length() if own else 0,
            gpu_resident_kv_bytes=sum(x.resident_bytes() for x in own),
            host_kv_bytes=0,
            gpu_allocated_kv_bytes=sum(x.allocated_bytes() for x in own),
        )
