"""lkv_quest_topk_admit against lkv_quest_topk followed by lkv_tier_admit.

Over a run of decode steps whose queries select overlapping but different blocks, from the same
starting state, the one call and the two must leave the same selection and bitmap, the same
residency tables (block_slot, slot_block, last_used, evicted_at), the same miss lists and hot-list
slots, and the same slot pool, bit for bit, at head_dim 64 (the TMA-scored selection, the staged
admit and the vectorised fetch) and 128 (the other selection and fetch paths).
"""

from __future__ import annotations

import pytest
import torch

from tests.parity import lru_admit

pytestmark = pytest.mark.gpu
DEV = "cuda"
NEVER = -(2**40)


def _state(h: int, nblk: int, k: int, d: int, seed: int):  # noqa: ANN202
    from lazykv_b200 import kernels as K

    g = torch.Generator(device=DEV).manual_seed(seed)
    kv = torch.randn(nblk, h, 2, 16, d, device=DEV, generator=g)
    kv[:, :, 0] += torch.randn(1, h, 1, d, device=DEV, generator=g) * 0.7
    kv = kv.bfloat16()
    kmin = torch.empty((h, nblk, d), dtype=torch.bfloat16, device=DEV)
    kmax = torch.empty_like(kmin)
    rec = K.pack_int8(kv, kmin=kmin, kmax=kmax)
    q_base = torch.randn(4 * h, d, device=DEV, generator=g)
    queries = [(q_base + 0.2 * torch.randn(4 * h, d, device=DEV, generator=g)).bfloat16() for _ in range(6)]
    st = {
        "chosen": torch.zeros((h, k), dtype=torch.int32, device=DEV),
        "bitmap": torch.zeros((h, K.bitmap_words(nblk + 1)), dtype=torch.int32, device=DEV),
        "block_slot": torch.full((h, nblk), -1, dtype=torch.int32, device=DEV),
        "slot_block": torch.full((h, k), -1, dtype=torch.int32, device=DEV),
        "last_used": torch.full((h, k), -2, dtype=torch.int64, device=DEV),
        "evicted_at": torch.full((h, nblk), NEVER, dtype=torch.int64, device=DEV),
        "pool": torch.zeros((k + 2, h, 2, 16, d), dtype=torch.bfloat16, device=DEV),
        "miss_blk": torch.zeros((h, k), dtype=torch.int32, device=DEV),
        "miss_slot": torch.zeros((h, k), dtype=torch.int32, device=DEV),
        "n_miss": torch.zeros((h,), dtype=torch.int32, device=DEV),
        "slots": torch.zeros((h, k), dtype=torch.int32, device=DEV),
    }
    return kmin, kmax, rec, queries, st


def _compare(a: dict, b: dict) -> None:
    for name in ("chosen", "bitmap", "block_slot", "slot_block", "last_used", "evicted_at", "n_miss", "slots", "pool"):
        assert torch.equal(a[name], b[name]), name
    for j in range(a["n_miss"].shape[0]):
        n = int(a["n_miss"][j])
        assert torch.equal(a["miss_blk"][j, :n], b["miss_blk"][j, :n]) and torch.equal(a["miss_slot"][j, :n], b["miss_slot"][j, :n])


@pytest.mark.parametrize("d", [64, 128])
def test_select_admit_equals_the_two_calls(d: int) -> None:
    from lazykv_b200 import kernels as K

    h, nblk, k = 8, 4096, 1022
    kmin, kmax, rec, queries, a = _state(h, nblk, k, d, seed=d)
    b = {n: t.clone() for n, t in a.items()}
    total_miss = 0
    for step, q in enumerate(queries + queries[:2], start=1):
        K.quest_topk(q, kmin, kmax, 1, nblk - 2, k, out_blocks=a["chosen"], bitmap=a["bitmap"], by_block=True)
        K.tier_admit(a["chosen"], a["block_slot"], a["slot_block"], a["last_used"], a["evicted_at"], step, rec, a["pool"], a["miss_blk"],
                     a["miss_slot"], a["n_miss"], slots_out=a["slots"])
        K.quest_topk_admit(q, kmin, kmax, 1, nblk - 2, k, b["chosen"], b["bitmap"], b["block_slot"], b["slot_block"], b["last_used"],
                           b["evicted_at"], step, rec, b["pool"], b["miss_blk"], b["miss_slot"], b["n_miss"], slots_out=b["slots"])
        torch.cuda.synchronize()
        _compare(a, b)
        total_miss += int(a["n_miss"].sum())
    assert total_miss > h * k  # the first step misses everything, later steps some
    assert K.device_status() == 0


@pytest.mark.parametrize("d", [64, 128])
def test_resident_split_attends_as_the_admit_first_order(d: int) -> None:
    """lkv_quest_topk_resident: the chosen ids equal lkv_quest_topk's; the hot list holds each chosen
    block's slot before the admit (or -1) and the bitmap only the resident ones; the attention over
    them (misses in the exact pass, from their records) equals the attention after the admit, and
    the admit run afterwards (without a hot list) leaves the same tables and pool."""
    from lazykv_b200 import kernels as K

    h, nblk, k = 8, 4096, 1022
    kmin, kmax, rec, queries, a = _state(h, nblk, k, d, seed=d + 1)
    b = {n: t.clone() for n, t in a.items()}
    strides = (h * 2 * 16 * d, 2 * 16 * d, d)
    for step, q in enumerate(queries, start=1):
        # a: admit first, then attend the slots it wrote
        K.quest_topk_admit(q, kmin, kmax, 1, nblk - 2, k, a["chosen"], a["bitmap"], a["block_slot"], a["slot_block"], a["last_used"],
                           a["evicted_at"], step, rec, a["pool"], a["miss_blk"], a["miss_slot"], a["n_miss"], slots_out=a["slots"])
        oa, la = K.exact_attention(q, a["pool"], a["pool"][:, :, 1], strides, a["slots"], 16, rec, 1, nblk - 2, d**-0.5, 16, excluded=a["bitmap"],
                                   out_dtype=torch.float32)
        # b: the resident split, the attention, then the admit
        before = b["block_slot"].clone()
        K.quest_topk_resident(q, kmin, kmax, 1, nblk - 2, k, b["chosen"], b["block_slot"], b["slots"], b["bitmap"])
        ob, lb = K.exact_attention(q, b["pool"], b["pool"][:, :, 1], strides, b["slots"], 16, rec, 1, nblk - 2, d**-0.5, 16, excluded=b["bitmap"],
                                   out_dtype=torch.float32)
        torch.cuda.synchronize()
        want_hot = torch.gather(before, 1, b["chosen"].long())
        want_hot = torch.where(want_hot >= 1, want_hot, torch.full_like(want_hot, -1))
        assert torch.equal(b["slots"], want_hot)
        bits = torch.zeros((h, b["bitmap"].shape[1] * 32), dtype=torch.bool, device=DEV)
        for j in range(h):
            res = b["chosen"][j][want_hot[j] >= 1].long()
            bits[j, res] = True
        words = b["bitmap"].view(torch.int32).cpu().numpy().view("uint32")
        import numpy as np

        got_bits = np.unpackbits(words.view(np.uint8), bitorder="little").reshape(h, -1).astype(bool)
        assert np.array_equal(got_bits, bits.cpu().numpy())
        assert torch.equal(a["chosen"], b["chosen"])
        scale = oa.abs().max()
        assert (ob - oa).abs().max() <= 1e-5 * scale and (lb - la).abs().max() <= 1e-5 * la.abs().max()
        K.tier_admit(b["chosen"], b["block_slot"], b["slot_block"], b["last_used"], b["evicted_at"], step, rec, b["pool"], b["miss_blk"],
                     b["miss_slot"], b["n_miss"])
        torch.cuda.synchronize()
        for name in ("block_slot", "slot_block", "last_used", "evicted_at", "n_miss", "pool"):
            assert torch.equal(a[name], b[name]), name
    assert K.device_status() == 0


def test_large_pool_admit_follows_the_lru_rule() -> None:
    """A pool of 16,384 slots per head with about a quarter of them chosen per step (the global
    selection's ranks at N = 4): the admit that selects only as many victims as there are misses
    (a radix select, then a sort of those) evicts exactly what the reference's rule evicts."""
    import numpy as np

    from lazykv_b200 import kernels as K

    h, cap, n_slots, d = 2, 32768, 16384, 64
    rng = np.random.default_rng(3)
    rec = torch.zeros((cap, h, K.packed_pair_bytes(16, d)), dtype=torch.uint8, device=DEV)
    pool = torch.zeros((n_slots + 2, h, 2, 16, d), dtype=torch.bfloat16, device=DEV)
    dev = {
        "block_slot": torch.full((h, cap), -1, dtype=torch.int32, device=DEV),
        "slot_block": torch.full((h, n_slots), -1, dtype=torch.int32, device=DEV),
        "last_used": torch.full((h, n_slots), -2, dtype=torch.int64, device=DEV),
        "evicted_at": torch.full((h, cap), NEVER, dtype=torch.int64, device=DEV),
    }
    host = {n: t.cpu().numpy().copy() for n, t in dev.items()}
    miss_blk = torch.zeros((h, n_slots), dtype=torch.int32, device=DEV)
    miss_slot = torch.zeros((h, n_slots), dtype=torch.int32, device=DEV)
    n_miss = torch.zeros((h,), dtype=torch.int32, device=DEV)
    base = rng.choice(cap, size=6000, replace=False)
    for step in range(1, 7):
        ch = np.full((h, n_slots), -1, dtype=np.int64)
        for j in range(h):
            pick = np.unique(np.concatenate([rng.choice(base, size=3000, replace=False), rng.choice(cap, size=1200, replace=False)]))
            ch[j, : len(pick)] = np.sort(pick)
        chosen = torch.from_numpy(ch).int().to(DEV)
        K.tier_admit(chosen, dev["block_slot"], dev["slot_block"], dev["last_used"], dev["evicted_at"], step, rec, pool, miss_blk, miss_slot, n_miss)
        misses = lru_admit(ch, host["block_slot"], host["slot_block"], host["last_used"], host["evicted_at"], step)
        torch.cuda.synchronize()
        for name in ("block_slot", "slot_block", "last_used", "evicted_at"):
            assert np.array_equal(dev[name].cpu().numpy(), host[name]), (step, name)
        nm = n_miss.cpu().numpy()
        for j in range(h):
            assert nm[j] == len(misses[j])
            assert np.array_equal(miss_blk[j, : nm[j]].cpu().numpy(), misses[j])
    assert K.device_status() == 0
