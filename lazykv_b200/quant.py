"""int8 records for the cold tier: the API of lazykv/quant.py (:46-105) on the device.

`pack` and `unpack` keep the reference's record (kq | vq | k_scale | k_zero | v_scale | v_zero,
float16 scales, keys per channel and values per token) and its float32 arithmetic, bit for bit with
the reference's CPU pack, through the lkv_pack_int8 / lkv_unpack_int8 kernels.
"""

from __future__ import annotations

import torch

from lazykv_b200 import kernels as K

SCALE_DTYPE = torch.float16


def packed_pair_bytes(block_size: int, head_dim: int) -> int:
    """Bytes one packed (block, head) pair occupies (quant.py:46-49)."""
    return 2 * block_size * head_dim + 2 * SCALE_DTYPE.itemsize * head_dim + 2 * SCALE_DTYPE.itemsize * block_size


def pack(blocks: torch.Tensor) -> torch.Tensor:
    """Pack KV pairs [..., 2, block_size, head_dim] (CUDA) into uint8 records [..., packed_pair_bytes]."""
    *lead, two, bs, d = blocks.shape
    if two != 2:
        raise ValueError(f"expected a [..., 2, block_size, head_dim] KV pair, got {tuple(blocks.shape)}")
    flat = blocks.reshape(-1, 1, 2, bs, d)
    rec = K.pack_int8(flat)
    return rec.view(*lead, rec.shape[-1])


def unpack(packed: torch.Tensor, block_size: int, head_dim: int, dtype: torch.dtype) -> torch.Tensor:
    """Dequantise uint8 records [m, packed_pair_bytes] (CUDA) to [m, 2, block_size, head_dim] in `dtype`."""
    if packed.ndim != 2 or packed.shape[1] != packed_pair_bytes(block_size, head_dim):
        raise ValueError(f"expected [m, {packed_pair_bytes(block_size, head_dim)}] uint8 records, got {tuple(packed.shape)}")
    return K.unpack_int8(packed, block_size, head_dim, dtype)
