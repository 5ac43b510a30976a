"""Failure detection of the bounded waits, on the GPU, without a fault.

The selection's TMA scoring waits on shared-memory barriers for its tile copies. Its test hook makes
the next call first wait on a barrier that nothing completes, with a short bound, so that the wait
runs out. The call must then record status 1 in the status word and in its host-mapped mirror
(polled without a synchronisation), write the failure's poison (every listed id -1, an empty bitmap)
and leave the GPU usable: the next call, with nothing stalled, selects exactly as before.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _layer(seed: int = 5, h: int = 8, n: int = 8192, g: int = 4, d: int = 64):  # noqa: ANN202
    gen = torch.Generator(device=DEV).manual_seed(seed)
    keys = (torch.randn(h, n, 16, d, device=DEV, generator=gen) + torch.randn(h, 1, 1, d, device=DEV, generator=gen)).bfloat16()
    q = torch.randn(h * g, d, device=DEV, generator=gen).bfloat16()
    return q, keys.amin(2).contiguous(), keys.amax(2).contiguous()


def test_a_selection_wait_that_runs_out_is_reported_and_poisons_only_that_call() -> None:
    from lazykv_b200 import _lib
    from lazykv_b200 import kernels as K

    K.status_attach()
    assert K.device_status(clear=True) == 0
    K.status_poll(clear=True)
    q, kmin, kmax = _layer()
    h, nb = kmin.shape[0], kmin.shape[1]
    n_cand, k = nb - 2, 2046
    words = K.bitmap_words(nb)
    ref, _ = K.quest_topk(q, kmin, kmax, 1, n_cand, k, by_block=True)
    ref = ref.clone()
    torch.cuda.synchronize()

    out = torch.full((h, k), 7, dtype=torch.int32, device=DEV)
    bm = torch.full((h, words), -1, dtype=torch.int32, device=DEV)
    K.debug_set(_lib.LKV_DEBUG_SELECT_WAIT_ITERS, 64)  # about 64 us of waiting at most
    K.debug_set(_lib.LKV_DEBUG_SELECT_STALL_NEXT, 1)
    try:
        K.quest_topk(q, kmin, kmax, 1, n_cand, k, out_blocks=out, bitmap=bm, by_block=True)
        torch.cuda.synchronize()
    finally:
        K.debug_set(_lib.LKV_DEBUG_SELECT_STALL_NEXT, 0)
        K.debug_set(_lib.LKV_DEBUG_SELECT_WAIT_ITERS, 1 << 21)
    # The host mirror shows it without a synchronising read; the status word agrees.
    assert K.status_poll(clear=False) == _lib.LKV_DEV_WAIT_TIMEOUT
    assert K.device_status(clear=True) == _lib.LKV_DEV_WAIT_TIMEOUT
    assert (out.cpu() == -1).all()
    assert (bm.cpu() == 0).all()
    # What a decode loop does once per step: the mirror's code becomes an exception (and is cleared).
    with pytest.raises(K.DeviceWaitError):
        K.raise_on_status("test")
    assert K.status_poll(clear=False) == 0

    # The GPU is usable and nothing is left over: the next call selects exactly as before.
    out2 = torch.full((h, k), 7, dtype=torch.int32, device=DEV)
    bm2 = torch.full((h, words), -1, dtype=torch.int32, device=DEV)
    K.quest_topk(q, kmin, kmax, 1, n_cand, k, out_blocks=out2, bitmap=bm2, by_block=True)
    torch.cuda.synchronize()
    assert torch.equal(out2, ref)
    bits = np.unpackbits(bm2.cpu().numpy().view(np.uint8), bitorder="little").reshape(h, -1)
    for j in range(h):
        assert np.array_equal(np.nonzero(bits[j])[0], ref[j].cpu().numpy())
    assert K.device_status(clear=True) == 0
    assert K.status_poll(clear=True) == 0


def test_a_poisoned_selection_still_gives_the_exact_output() -> None:
    """With every listed id -1 and an empty bitmap, the hot pass attends only the sink and the
    current block and the cold pass every candidate: the merged output is the exact one."""
    from lazykv_b200 import _lib
    from lazykv_b200 import kernels as K

    K.status_attach()
    h, g, d, bs, n_sealed = 8, 4, 64, 16, 1025
    gen = torch.Generator(device=DEV).manual_seed(11)
    kv = torch.randn(n_sealed, h, 2, bs, d, device=DEV, generator=gen).bfloat16()
    cur = torch.randn(h, 2, bs, d, device=DEV, generator=gen).bfloat16()
    q = torch.randn(h * g, d, device=DEV, generator=gen).bfloat16()
    kmin = torch.empty((h, n_sealed, d), dtype=torch.bfloat16, device=DEV)
    kmax = torch.empty_like(kmin)
    deq = torch.empty_like(kv)
    rec = K.pack_int8(kv, kmin=kmin, kmax=kmax, deq=deq)
    k = 100
    n_cand = n_sealed - 1
    lst = torch.zeros((h, k + 2), dtype=torch.int32, device=DEV)
    lst[:, -1] = n_sealed
    bm = torch.zeros((h, K.bitmap_words(n_sealed + 1)), dtype=torch.int32, device=DEV)
    pool = torch.zeros((n_sealed + 1, h, 2, bs, d), dtype=torch.bfloat16, device=DEV)
    pool[:n_sealed] = deq
    pool[0] = kv[0]
    pool[n_sealed] = cur
    strides = (h * 2 * bs * d, 2 * bs * d, d)
    outs = []
    for stall in (0, 1):
        if stall:
            K.debug_set(_lib.LKV_DEBUG_SELECT_WAIT_ITERS, 64)
            K.debug_set(_lib.LKV_DEBUG_SELECT_STALL_NEXT, 1)
        try:
            K.quest_topk(q, kmin, kmax, 1, n_cand, k, out_blocks=lst[:, 1 : k + 1], bitmap=bm, by_block=True)
        finally:
            K.debug_set(_lib.LKV_DEBUG_SELECT_STALL_NEXT, 0)
            K.debug_set(_lib.LKV_DEBUG_SELECT_WAIT_ITERS, 1 << 21)
        o, _ = K.exact_attention(q, pool, pool[:, :, 1], strides, lst, bs, rec, 1, n_cand, d**-0.5, bs, excluded=bm, out_dtype=torch.float32)
        torch.cuda.synchronize()
        outs.append(o.clone())
        if stall:
            assert (lst[:, 1 : k + 1] == -1).all().item()
    assert K.device_status(clear=True) == _lib.LKV_DEV_WAIT_TIMEOUT
    K.status_poll(clear=True)
    a, b = outs[0].double(), outs[1].double()
    assert float((a - b).abs().max() / a.abs().max()) < 1e-5
