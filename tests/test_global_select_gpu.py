"""The global top-K of a context-sharded layer (lkv_quest_bounds on every shard, the bounds
gathered, lkv_topk_gathered on every rank), emulated on one GPU: every rank's part, mapped back to
global block ids and concatenated in rank order, is the selection lkv_quest_topk makes over the
unsharded candidates, and the parts' bitmaps are its bitmap; ties at the threshold that straddle
rank boundaries go to the lower ids. The reference selects on one device (lazykv/selection.py:56-62,
top_blocks), which is the single-call selection these parts must add up to."""

from __future__ import annotations

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _metadata(h: int, n: int, d: int, seed: int, ties: str) -> tuple[torch.Tensor, torch.Tensor]:
    gen = torch.Generator(device=DEV).manual_seed(seed)
    a = torch.randn((h, n, d), generator=gen, device=DEV)
    b = a + torch.rand((h, n, d), generator=gen, device=DEV)
    if ties == "all":  # every block the same: the lowest K ids win
        a[:] = a[:, :1]
        b[:] = b[:, :1]
    elif ties == "runs":  # runs of 97 identical blocks: many ties, some at the threshold
        idx = (torch.arange(n, device=DEV) // 97) * 97
        a, b = a[:, idx], b[:, idx]
    return a.bfloat16().contiguous(), b.bfloat16().contiguous()


def _bits(bm: torch.Tensor) -> np.ndarray:
    h = bm.shape[0]
    return np.unpackbits(bm.cpu().numpy().view(np.uint8), bitorder="little").reshape(h, -1)


@pytest.mark.parametrize("world", [1, 2, 3, 8])
@pytest.mark.parametrize("d,h,g", [(64, 8, 4), (128, 64, 4)])
@pytest.mark.parametrize("ties", ["none", "runs", "all"])
@pytest.mark.parametrize("mode", [torch.bfloat16, torch.float32])
def test_gathered_parts_add_up_to_the_single_gpu_selection(world: int, d: int, h: int, g: int, ties: str, mode: torch.dtype) -> None:
    from lazykv_b200 import kernels as K
    from lazykv_b200.sharded import shard_plan

    n_sealed, k_total = 4097, 1024
    kmin, kmax = _metadata(h, n_sealed, d, seed=world * 7 + d, ties=ties)
    q = torch.randn((h * g, d), generator=torch.Generator(device=DEV).manual_seed(3), device=DEV).bfloat16()
    words = K.bitmap_words(n_sealed)
    want_bm = torch.zeros((h, words), dtype=torch.int32, device=DEV)
    want, _ = K.quest_topk(q, kmin, kmax, 1, n_sealed - 1, k_total, mode, bitmap=want_bm, by_block=True)
    plans = [shard_plan(n_sealed, k_total, world, r) for r in range(world)]
    seg_n = [p.n_cand for p in plans]
    ld = max(seg_n) + 5  # a padded row stride
    gathered = torch.full((world, h, ld), float("nan"), dtype=mode, device=DEV)
    for r, p in enumerate(plans):
        K.quest_bounds(q, kmin[:, p.lo : p.hi].contiguous(), kmax[:, p.lo : p.hi].contiguous(), p.cand_first - p.lo, p.n_cand, gathered[r], mode)
    parts, bits = [], []
    for r, p in enumerate(plans):
        cols = min(k_total, p.n_cand)
        out = torch.full((h, cols + 3), -7, dtype=torch.int32, device=DEV)
        bm = torch.full((h, K.bitmap_words(p.hi - p.lo + 1)), -1, dtype=torch.int32, device=DEV)
        K.topk_gathered(gathered, seg_n, k_total, r, p.cand_first - p.lo, out, bm, out_cols=cols)
        o = out.cpu().numpy()
        assert (o[:, cols:] == -7).all(), "columns past out_cols are not written"
        parts.append((o[:, :cols], p))
        bits.append((_bits(bm), p))
    w = want.cpu().numpy()
    wb = _bits(want_bm)
    for j in range(h):
        got = []
        for o, p in parts:
            row = o[j]
            n_sel = int((row >= 0).sum())
            assert (row[:n_sel] >= 0).all() and (row[n_sel:] == -1).all(), "chosen ids first, then -1"
            got.extend((row[:n_sel] + p.lo).tolist())
        assert got == w[j].tolist()
        for b, p in bits:
            local = np.nonzero(b[j])[0]
            assert np.array_equal(local + p.lo, np.nonzero(wb[j][p.lo : p.hi])[0] + p.lo)


def test_bounds_equal_the_selection_bounds() -> None:
    """lkv_quest_bounds gives the bounds lkv_quest_topk reports (float32), in bf16 exactly."""
    from lazykv_b200 import kernels as K

    h, n, d = 8, 3000, 128
    kmin, kmax = _metadata(h, n, d, seed=11, ties="none")
    q = torch.randn((32, d), generator=torch.Generator(device=DEV).manual_seed(4), device=DEV).bfloat16()
    _, want = K.quest_topk(q, kmin, kmax, 5, n - 5, 100, torch.bfloat16, want_bound=True)
    got16 = torch.empty((h, n), dtype=torch.bfloat16, device=DEV)
    K.quest_bounds(q, kmin, kmax, 5, n - 5, got16, torch.bfloat16)
    assert torch.equal(got16[:, : n - 5].float(), want)
    got32 = torch.empty((h, n - 5), dtype=torch.float32, device=DEV)
    K.quest_bounds(q, kmin, kmax, 5, n - 5, got32, torch.bfloat16)
    assert torch.equal(got32, want)


def test_bad_arguments_raise() -> None:
    from lazykv_b200 import kernels as K
    from lazykv_b200._lib import LkvError

    h, d = 4, 64
    kmin, kmax = _metadata(h, 100, d, seed=1, ties="none")
    q = torch.randn((16, d), device=DEV).bfloat16()
    with pytest.raises(LkvError):  # float32 bounds cannot be stored as bf16
        K.quest_bounds(q, kmin, kmax, 0, 100, torch.empty((h, 100), dtype=torch.bfloat16, device=DEV), torch.float32)
    gathered = torch.zeros((2, h, 60), dtype=torch.bfloat16, device=DEV)
    with pytest.raises(LkvError):  # a rank cannot hold more candidates than the row stride
        K.topk_gathered(gathered, [61, 30], 10, 0, 0, torch.empty((h, 10), dtype=torch.int32, device=DEV))
    with pytest.raises(LkvError):  # too few output columns for min(k, n_rank)
        K.topk_gathered(gathered, [50, 30], 20, 1, 0, torch.empty((h, 10), dtype=torch.int32, device=DEV))


def test_global_selection_of_one_rank_is_the_plain_selection() -> None:
    """sharded.GlobalSelection with a single rank (no process group): its chosen ids and bitmap are
    lkv_quest_topk's over the rank's candidates, -1 past K."""
    from lazykv_b200 import kernels as K
    from lazykv_b200.sharded import GlobalSelection, shard_plan

    h, d, n_sealed, k_total = 8, 64, 2049, 300
    kmin, kmax = _metadata(h, n_sealed, d, seed=21, ties="runs")
    q = torch.randn((h * 4, d), generator=torch.Generator(device=DEV).manual_seed(5), device=DEV).bfloat16()
    plan = shard_plan(n_sealed, k_total, 1, 0)
    sel = GlobalSelection([plan], 0, h, k_total, torch.device(DEV))
    chosen = torch.full((h, sel.cols + 2), -7, dtype=torch.int32, device=DEV)
    bm = torch.full((h, K.bitmap_words(n_sealed + 1)), -1, dtype=torch.int32, device=DEV)
    sel.select(q, kmin, kmax, chosen, bm)
    want_bm = torch.zeros_like(bm)
    want, _ = K.quest_topk(q, kmin, kmax, plan.cand_first - plan.lo, plan.n_cand, k_total, out_blocks=None, bitmap=want_bm, by_block=True)
    torch.cuda.synchronize()
    got = chosen.cpu().numpy()
    assert np.array_equal(got[:, :k_total], want.cpu().numpy())
    assert (got[:, k_total : sel.cols] == -1).all() and (got[:, sel.cols :] == -7).all()
    assert torch.equal(bm, want_bm)


def test_gathered_resident_split_lists_the_resident_slots() -> None:
    """lkv_topk_gathered_resident: the same chosen ids; hot holds each chosen block's slot from
    block_slot or -1 (and -1 in the padding); the bitmap marks only the resident chosen blocks."""
    from lazykv_b200 import kernels as K
    from lazykv_b200.sharded import shard_plan

    h, d, n_sealed, k_total, world = 8, 64, 3001, 500, 2
    kmin, kmax = _metadata(h, n_sealed, d, seed=9, ties="runs")
    q = torch.randn((h * 4, d), generator=torch.Generator(device=DEV).manual_seed(6), device=DEV).bfloat16()
    plans = [shard_plan(n_sealed, k_total, world, r) for r in range(world)]
    seg_n = [p.n_cand for p in plans]
    gathered = torch.zeros((world, h, max(seg_n)), dtype=torch.bfloat16, device=DEV)
    for r, p in enumerate(plans):
        K.quest_bounds(q, kmin[:, p.lo : p.hi].contiguous(), kmax[:, p.lo : p.hi].contiguous(), p.cand_first - p.lo, p.n_cand, gathered[r])
    gen = torch.Generator(device=DEV).manual_seed(12)
    for r, p in enumerate(plans):
        cols = min(k_total, p.n_cand)
        nb = p.hi - p.lo
        block_slot = torch.where(torch.rand((h, nb), generator=gen, device=DEV) < 0.5,
                                 torch.randint(1, 4000, (h, nb), generator=gen, device=DEV), torch.full((h, nb), -1, device=DEV)).int().contiguous()
        plain = torch.empty((h, cols), dtype=torch.int32, device=DEV)
        bm_plain = torch.zeros((h, K.bitmap_words(nb + 1)), dtype=torch.int32, device=DEV)
        K.topk_gathered(gathered, seg_n, k_total, r, p.cand_first - p.lo, plain, bm_plain, out_cols=cols)
        out = torch.empty((h, cols), dtype=torch.int32, device=DEV)
        hot = torch.full((h, cols), -7, dtype=torch.int32, device=DEV)
        bm = torch.full((h, K.bitmap_words(nb + 1)), -1, dtype=torch.int32, device=DEV)
        K.topk_gathered(gathered, seg_n, k_total, r, p.cand_first - p.lo, out, bm, out_cols=cols, block_slot=block_slot, hot=hot)
        torch.cuda.synchronize()
        assert torch.equal(out, plain)
        ids = out.long().clamp(min=0)
        want_hot = torch.where(out >= 0, torch.gather(block_slot, 1, ids), torch.full_like(out, -1))
        want_hot = torch.where(want_hot >= 1, want_hot, torch.full_like(want_hot, -1))
        assert torch.equal(hot, want_hot)
        for j in range(h):
            res = out[j][(out[j] >= 0) & (want_hot[j] >= 1)].cpu().numpy()
            assert np.array_equal(np.nonzero(_bits(bm)[j])[0], np.sort(res))
