"""Preallocated full-GPU KV cache: the dense layers' store and the source of the tier's boundary.

API of lazykv/cache.py (PreallocatedLayer :20-77, FullGPUCache :80-102, CacheStats :105-115):
one [1, kv_heads, max_len, head_dim] buffer pair per layer, allocated once and zero-filled (so
padding reads are finite), whose update returns views of the filled prefix.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch
from transformers.cache_utils import Cache, CacheLayerMixin


@dataclass(frozen=True)
class CacheStats:
    seq_len: int
    gpu_resident_kv_bytes: int
    host_kv_bytes: int
    gpu_allocated_kv_bytes: int

    @property
    def gpu_residency_fraction(self) -> float:
        total = self.gpu_resident_kv_bytes + self.host_kv_bytes
        return 1.0 if total == 0 else self.gpu_resident_kv_bytes / total


class PreallocatedLayer(CacheLayerMixin):
    """One layer's KV: [1, h, max_len, d] keys and values, filled from the front."""

    def __init__(self, max_len: int, **kwargs: object) -> None:
        super().__init__()
        self.max_len = max_len
        self.length = 0

    def lazy_initialization(self, key_states: torch.Tensor, value_states: torch.Tensor) -> None:
        b, h, _, d = key_states.shape
        if b != 1:
            raise ValueError("LazyKV is batch-size-1 only (v1 scope)")
        self.dtype, self.device = key_states.dtype, key_states.device
        self.keys = torch.zeros((1, h, self.max_len, d), dtype=key_states.dtype, device=key_states.device)
        self.values = torch.zeros((1, value_states.shape[1], self.max_len, value_states.shape[3]), dtype=value_states.dtype, device=value_states.device)
        self.is_initialized = True

    def update(self, key_states: torch.Tensor, value_states: torch.Tensor, *args: object, **kwargs: object) -> tuple[torch.Tensor, torch.Tensor]:
        if not self.is_initialized:
            self.lazy_initialization(key_states, value_states)
        end = self.length + key_states.shape[-2]
        if end > self.max_len:
            raise RuntimeError(f"KV cache overflow: {end} > max_len {self.max_len}")
        self.keys[:, :, self.length : end].copy_(key_states)
        self.values[:, :, self.length : end].copy_(value_states)
        self.length = end
        return self.keys[:, :, :end], self.values[:, :, :end]

    def get_mask_sizes(self, query_length: int) -> tuple[int, int]:
        return self.length + query_length, 0

    def get_seq_length(self) -> int:
        return self.length

    def get_max_length(self) -> int:
        return self.max_len

    def get_max_cache_shape(self) -> int:
        return self.max_len

    def reset(self) -> None:
        self.length = 0

    def truncate(self, length: int) -> None:
        """Forget tokens past `length`, so one prefill can be decoded from more than once."""
        if not 0 <= length <= self.length:
            raise ValueError(f"cannot truncate length {self.length} to {length}")
        self.length = length

    def resident_bytes(self) -> int:
        if not self.is_initialized:
            return 0
        per_token = self.keys[0, :, 0].numel() * self.keys.element_size() + self.values[0, :, 0].numel() * self.values.element_size()
        return per_token * self.length


class FullGPUCache(Cache):
    """Every token of every layer on the GPU: the exact reference, and the dense layers' store."""

    def __init__(self, num_layers: int, max_len: int) -> None:
        super().__init__(layers=[PreallocatedLayer(max_len) for _ in range(num_layers)])
        self.max_len = max_len

    def truncate(self, length: int) -> None:
        for layer in self.layers:
            layer.truncate(length)

    def stats(self) -> CacheStats:
        layers = [x for x in self.layers if isinstance(x, PreallocatedLayer)]
        allocated = sum(x.keys.numel() * x.keys.element_size() + x.values.numel() * x.values.element_size() for x in layers if x.is_initialized)
        return CacheStats(layers[0].get_seq_length() if layers else 0, sum(x.resident_bytes() for x in layers), 0, allocated)
