"""The allocation-free top-k entry point, lkv_quest_topk_noalloc, called through the C ABI.

It exists for callers that cannot allocate device memory when they select blocks (an
allocator-free runtime, code inside an allocator callback, a process that reserved all device
memory up front): its scratch lives in a fixed array inside the library. Its results must equal
lkv_quest_topk's (given a workspace) bit for bit, on two calls in a row with different inputs, so
that what the first call leaves in the shared array cannot leak into the second. This file is
collected last, so a run that stops at the first failure has run every other test first.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

DEV = "cuda"


def _case(seed: int, h: int, nb: int, hq: int, d: int, dtype: torch.dtype) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    g = torch.Generator(device=DEV).manual_seed(seed)
    keys = (torch.randn(h, nb, 16, d, device=DEV, generator=g) + torch.randn(h, 1, 1, d, device=DEV, generator=g)).to(dtype)
    q = torch.randn(hq, d, device=DEV, generator=g).to(dtype)
    return q, keys.amin(2).contiguous(), keys.amax(2).contiguous()


def _run(entry: str, q, kmin, kmax, first: int, n_cand: int, k: int, mode: int, order: int = 0):  # noqa: ANN001, ANN202
    from lazykv_b200 import _lib

    h, _, d = kmin.shape
    out = torch.full((h, k), -1, dtype=torch.int32, device=DEV)
    bound = torch.full((h, n_cand), float("nan"), dtype=torch.float32, device=DEV)
    words = (kmin.shape[1] + 31) // 32
    bitmap = torch.full((h, words), -1, dtype=torch.int32, device=DEV)
    common = (q.data_ptr(), _lib.dtype_code(q.dtype), q.shape[0], h, d, kmin.data_ptr(), kmax.data_ptr(), _lib.dtype_code(kmin.dtype),
              kmin.stride(0), first, n_cand, k, mode, order, out.data_ptr(), k, bound.data_ptr(), bitmap.data_ptr(), words)
    stream = torch.cuda.current_stream().cuda_stream
    if entry == "noalloc":
        before = torch.cuda.memory_stats().get("allocation.all.allocated", 0)
        _lib.call("lkv_quest_topk_noalloc", *common, stream)
        assert torch.cuda.memory_stats().get("allocation.all.allocated", 0) == before
    else:
        ws = torch.zeros(_lib.lib().lkv_quest_topk_workspace(h, n_cand), dtype=torch.uint8, device=DEV)
        _lib.call("lkv_quest_topk", *common, ws.data_ptr(), ws.numel(), stream)
    torch.cuda.synchronize()
    return out.cpu().numpy(), bound.cpu().numpy(), bitmap.cpu().numpy()


def test_noalloc_top_k_equals_the_workspace_entry_point_on_two_calls_in_a_row() -> None:
    from lazykv_b200 import _lib

    _lib.lib()
    # Call 1: the metric geometry (8 heads x 8,190 candidates, K = 2,046, bf16 bound).
    q, kmin, kmax = _case(1, 8, 8192, 32, 64, torch.bfloat16)
    a = _run("noalloc", q, kmin, kmax, 1, 8190, 2046, _lib.LKV_BF16)
    b = _run("workspace", q, kmin, kmax, 1, 8190, 2046, _lib.LKV_BF16)
    for x, y in zip(a, b):
        assert np.array_equal(x, y)
    assert (a[0] >= 1).all() and (a[0] <= 8190).all()
    # Call 2: other sizes, float32, a float32 bound; the array still holds call 1's keys.
    q, kmin, kmax = _case(2, 4, 600, 16, 128, torch.float32)
    a = _run("noalloc", q, kmin, kmax, 1, 598, 100, _lib.LKV_F32)
    b = _run("workspace", q, kmin, kmax, 1, 598, 100, _lib.LKV_F32)
    for x, y in zip(a, b):
        assert np.array_equal(x, y)


def test_noalloc_block_order_equals_the_workspace_entry_point() -> None:
    """Ascending block-id order, both of its paths, each twice in a row and bit for bit: bf16 at
    head_dim 64 (one launch, a thread-block cluster per head, no scratch) and bf16 at head_dim 128
    (scores, then a cluster select that counts in the array's first-pass counters, which must read
    zero on entry and which every complete call leaves zero)."""
    from lazykv_b200 import _lib

    _lib.lib()
    for seed, d, nb, k in ((3, 64, 8192, 2046), (4, 64, 4100, 1000), (5, 128, 8192, 2046), (6, 128, 3000, 700)):
        q, kmin, kmax = _case(seed, 8, nb, 32, d, torch.bfloat16)
        a = _run("noalloc", q, kmin, kmax, 1, nb - 2, k, _lib.LKV_BF16, _lib.LKV_ORDER_BLOCK)
        b = _run("workspace", q, kmin, kmax, 1, nb - 2, k, _lib.LKV_BF16, _lib.LKV_ORDER_BLOCK)
        for x, y in zip(a, b):
            assert np.array_equal(x, y), (seed, d)
        assert (np.diff(a[0], axis=1) > 0).all()


def test_noalloc_rejects_inputs_beyond_its_fixed_scratch() -> None:
    from lazykv_b200 import _lib

    lib = _lib.lib()
    # 8 heads x 65,537 candidates need 524,296 keys; the array holds 524,288.
    rc = lib.lkv_quest_topk_noalloc(None, 1, 32, 8, 64, None, None, 1, 0, 1, 65537, 16, 1, 0, None, 16, None, None, 0, None)
    assert rc == 1  # LKV_ERR_ARG
    assert "fixed" in _lib.last_error() and "524288" in _lib.last_error()
