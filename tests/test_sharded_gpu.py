"""Context sharding on one GPU: shards emulated in sequence, their partials merged as the
all-gather would deliver them; the global selection merge kernel; -1 padding in hot lists."""

from __future__ import annotations

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _k():
    from lazykv_b200 import kernels

    return kernels


@pytest.mark.parametrize("n,k", [(7, 3), (300, 37), (4096, 1000), (16000, 4000)])
@pytest.mark.parametrize("mode", [torch.bfloat16, torch.float32])
def test_topk_merge_matches_the_host_rule(n: int, k: int, mode: torch.dtype) -> None:
    from lazykv_b200.sharded import host_reference_global_topk, topk_merge

    h = 8
    gen = torch.Generator(device=DEV).manual_seed(n + k)
    ids = torch.sort(torch.randperm(4 * n, generator=gen, device=DEV)[:n]).values.int().repeat(h, 1).contiguous()
    b = torch.randn((h, n), generator=gen, device=DEV)
    b = (b * 4).round() / 4 if mode == torch.bfloat16 else b  # many ties
    b = b.to(mode).float()
    words = (4 * n + 31) // 32
    bm = torch.full((h, words), -1, dtype=torch.int32, device=DEV)
    got = topk_merge(ids, b, k, mode, bitmap=bm)
    want = host_reference_global_topk(ids.cpu().numpy(), b.cpu().numpy(), k)
    assert np.array_equal(got.cpu().numpy(), want)
    bits = np.unpackbits(bm.cpu().numpy().view(np.uint8), bitorder="little").reshape(h, -1)
    for j in range(h):
        assert np.array_equal(np.nonzero(bits[j])[0], want[j])


@pytest.mark.parametrize("d,bs,dt", [(64, 16, torch.bfloat16), (16, 8, torch.bfloat16), (64, 16, torch.float32), (128, 16, torch.bfloat16)])
def test_padding_in_a_hot_list_attends_nothing(d: int, bs: int, dt: torch.dtype) -> None:
    """A hot list with -1 entries (a different count per head) equals the compact lists, per head."""
    K = _k()
    h, g, n = 4, 4, 60
    gen = torch.Generator(device=DEV).manual_seed(d + bs)
    kv = torch.randn((n, h, 2, bs, d), generator=gen, device=DEV).to(dt)
    q = torch.randn((h * g, d), generator=gen, device=DEV).to(dt)
    strides = (h * 2 * bs * d, 2 * bs * d, d)
    counts = [5, 9, 2, 7]
    width = 12
    padded = torch.full((h, width), -1, dtype=torch.int32)
    for j, c in enumerate(counts):
        ids = torch.sort(torch.randperm(n - 1, generator=torch.Generator().manual_seed(j))[:c]).values
        pos = torch.sort(torch.randperm(width - 1, generator=torch.Generator().manual_seed(10 + j))[:c]).values
        padded[j, pos] = ids.int()
    padded[:, -1] = n - 1  # the current block, last
    padded = padded.to(DEV)
    out, lse = K.hot_attention(q, kv, kv[:, :, 1], strides, padded, 5, d**-0.5, bs)
    for j in range(h):
        row = padded[j][padded[j] >= 0].view(1, -1).contiguous()
        qo, ql = K.hot_attention(q[j * g : (j + 1) * g].contiguous(), kv[:, j : j + 1], kv[:, j : j + 1, 1], strides, row, 5, d**-0.5, bs)
        assert torch.allclose(out[j * g : (j + 1) * g], qo, rtol=1e-5, atol=1e-6)
        assert torch.allclose(lse[j * g : (j + 1) * g], ql, rtol=1e-6, atol=1e-6)
    assert K.device_status() == 0


def _layer(n_sealed: int, h: int = 8, g: int = 4, d: int = 64, bs: int = 16, fill: int = 11, seed: int = 0):  # noqa: ANN202
    K = _k()
    gen = torch.Generator(device=DEV).manual_seed(seed)
    kv = torch.randn((n_sealed, h, 2, bs, d), generator=gen, device=DEV)
    kv[:, :, 0] += torch.randn((1, h, 1, d), generator=gen, device=DEV) * 0.7
    kv = kv.bfloat16()
    cur = torch.randn((h, 2, bs, d), generator=gen, device=DEV).bfloat16()
    q = torch.randn((h * g, d), generator=gen, device=DEV).bfloat16()
    kmin = torch.empty((h, n_sealed, d), dtype=torch.bfloat16, device=DEV)
    kmax = torch.empty_like(kmin)
    deq = torch.empty_like(kv)
    rec = K.pack_int8(kv, kmin=kmin, kmax=kmax, deq=deq)
    deq[0] = kv[0]  # the sink stays exact
    return dict(kv=kv, cur=cur, q=q, kmin=kmin, kmax=kmax, deq=deq, rec=rec, fill=fill, h=h, d=d, bs=bs, n=n_sealed)


def _shard_step(L: dict, plan, hot_ids_local: torch.Tensor):  # noqa: ANN001, ANN202
    """A ShardedExactStep over [lo, hi): every local block resident (pool row = local id), the
    current block as local id n_local on the last rank."""
    from lazykv_b200.sharded import ShardedExactStep

    h, d, bs = L["h"], L["d"], L["bs"]
    pool = L["deq"][plan.lo : plan.hi]
    if plan.has_current:
        pool = torch.cat([pool, L["cur"][None]], dim=0)
    pool = pool.contiguous()
    cols = []
    if plan.has_sink:
        cols.append(torch.zeros((h, 1), dtype=torch.int32, device=DEV))
    cols.append(hot_ids_local)
    if plan.has_current:
        cols.append(torch.full((h, 1), plan.hi - plan.lo, dtype=torch.int32, device=DEV))
    hot = torch.cat(cols, dim=1).contiguous()
    words = (plan.hi - plan.lo + 32) // 32 + 1
    bitmap = torch.zeros((h, words), dtype=torch.int32, device=DEV)
    st = ShardedExactStep(plan, bs, L["kmin"][:, plan.lo : plan.hi].contiguous(), L["kmax"][:, plan.lo : plan.hi].contiguous(),
                          L["rec"][plan.lo : plan.hi].contiguous(), pool, None, hot, bitmap, L["fill"], d**-0.5)
    return st


@pytest.mark.parametrize("world", [2, 3, 4])
@pytest.mark.parametrize("selection", ["local", "global"])
def test_sharded_exact_step_equals_the_single_gpu_step(world: int, selection: str) -> None:
    """Shards with local budgets, or with the global selection (candidates merged by
    lkv_topk_merge, hot lists padded per head), merged by lkv_lse_merge: the single-GPU exact
    output within float32 rounding (the exact int8 tier does not depend on the selection)."""
    from lazykv_b200.sharded import local_candidates, merge_partials, shard_hot_list, shard_plan, topk_merge

    K = _k()
    L = _layer(600)
    h, d, bs, n = L["h"], L["d"], L["bs"], L["n"]
    k_total = 150
    # single GPU: global selection over candidates 1..n-1, pool = all blocks dequantised
    pool = torch.cat([L["deq"], L["cur"][None]], dim=0).contiguous()
    sel, _ = K.quest_topk(L["q"], L["kmin"], L["kmax"], 1, n - 1, k_total, by_block=True)
    hot = torch.cat([torch.zeros((h, 1), dtype=torch.int32, device=DEV), sel, torch.full((h, 1), n, dtype=torch.int32, device=DEV)], 1).contiguous()
    bm = torch.zeros((h, (n + 32) // 32 + 1), dtype=torch.int32, device=DEV)
    K.quest_topk(L["q"], L["kmin"], L["kmax"], 1, n - 1, k_total, bitmap=bm, by_block=True)
    strides = (h * 2 * bs * d, 2 * bs * d, d)
    want, want_lse = K.exact_attention(L["q"], pool, pool[:, :, 1], strides, hot, L["fill"], L["rec"], 1, n - 1, d**-0.5, bs, excluded=bm,
                                       out_dtype=torch.float32)
    plans = [shard_plan(n, k_total, world, r) for r in range(world)]
    if selection == "global":
        cands = [local_candidates(L["q"], L["kmin"][:, p.lo : p.hi], L["kmax"][:, p.lo : p.hi], p.cand_first - p.lo, p.n_cand, k_total)
                 for p in plans]
        ids = torch.cat([c[0] + p.lo for c, p in zip(cands, plans)], dim=1).contiguous()  # rank order: ascending global ids
        bounds = torch.cat([c[1] for c in cands], dim=1).contiguous()
        glob = topk_merge(ids, bounds, k_total)
        assert torch.equal(glob, sel)  # the single-GPU selection
    outs, lses = [], []
    for p in plans:
        if selection == "global":
            mine = shard_hot_list(glob, p)
            local = torch.where(mine >= 0, mine - p.lo, mine).int()
            st = _shard_step(L, p, local)
            # the shard's bitmap marks its selected blocks (local ids): the cold pass skips them
            bmn = np.zeros(tuple(st.bitmap.shape), dtype=np.uint32)
            for j, row in enumerate(local.cpu().numpy()):
                for b in row[row >= 0]:
                    bmn[j, b // 32] |= np.uint32(1 << (b % 32))
            st.bitmap.copy_(torch.from_numpy(bmn.view(np.int32)))
        else:
            st = _shard_step(L, p, torch.zeros((h, p.k_local), dtype=torch.int32, device=DEV))
            st.select_local(L["q"])
        o, l = st.attend(L["q"])
        outs.append(o)
        lses.append(l)
    got, got_lse = merge_partials(torch.stack(outs), torch.stack(lses))
    scale = want.abs().max().item()
    assert (got - want).abs().max().item() < 1e-5 * scale
    assert (got_lse - want_lse).abs().max().item() < 1e-5 * want_lse.abs().max().item()
    assert K.device_status() == 0
