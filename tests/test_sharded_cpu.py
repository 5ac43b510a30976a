"""Context sharding on the host: the shard plan, and the cross-rank exchange of partials and of
selection candidates run as two gloo ranks on the CPU, checked with the oracle.

The per-shard partials and candidates are the oracle's (float64 attention, the canonical bound
and tie order); what runs for real is the plan (C ABI, host code) and the collectives of
lazykv_b200.sharded in a two-process group."""

from __future__ import annotations

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import oracle as O
from lazykv_b200.sharded import (gather_candidates, gather_partials, gathered_layout, host_reference_gathered_topk, host_reference_global_topk,
                                 shard_plan)


@pytest.mark.parametrize("n_sealed", [2, 3, 17, 1000, 8191])
@pytest.mark.parametrize("world", [1, 2, 3, 4, 8])
def test_shard_plan_partitions_the_blocks_and_the_budget(n_sealed: int, world: int) -> None:
    n_cand = n_sealed - 1
    for k in sorted({1, max(1, n_cand // 4), n_cand}):
        plans = [shard_plan(n_sealed, k, world, r) for r in range(world)]
        covered = np.zeros(n_sealed, dtype=int)
        for p in plans:
            covered[p.lo : p.hi] += 1
            assert p.cand_first == max(p.lo, 1) and p.n_cand == max(0, p.hi - p.cand_first)
            assert 0 <= p.k_local <= p.n_cand
        assert (covered == 1).all()  # every sealed block on exactly one rank
        assert plans[0].has_sink and not any(p.has_sink for p in plans[1:])
        assert plans[-1].has_current and not any(p.has_current for p in plans[:-1])
        assert sum(p.k_local for p in plans) == k


def test_shard_plan_refuses_a_budget_above_the_candidates() -> None:
    from lazykv_b200._lib import LkvError

    with pytest.raises(LkvError, match="budget"):
        shard_plan(10, 10, 2, 0)


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _layer(seed: int = 3, h: int = 2, g: int = 4, n: int = 41, bs: int = 16, d: int = 32, fill: int = 7):  # noqa: ANN202
    rng = np.random.default_rng(seed)
    k = rng.standard_normal((h, n * bs, d)) + rng.standard_normal((h, 1, d))
    v = rng.standard_normal((h, n * bs, d))
    q = rng.standard_normal((h * g, d))
    cur_k = rng.standard_normal((h, bs, d))
    cur_v = rng.standard_normal((h, bs, d))
    return q, k, v, cur_k, cur_v, fill


def _rank_partials(rank: int, world: int, port: int, results: dict) -> None:  # noqa: ANN001
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        q, k, v, cur_k, cur_v, fill = _layer()
        h, t, d = k.shape
        bs = cur_k.shape[1]
        n = t // bs
        g = q.shape[0] // h
        plan = shard_plan(n, max(1, (n - 1) // 4), world, rank)
        outs, lses = np.zeros((h, g, d)), np.zeros((h, g))
        for j in range(h):
            kk = k[j, plan.lo * bs : plan.hi * bs]
            vv = v[j, plan.lo * bs : plan.hi * bs]
            valid = np.ones(len(kk), dtype=bool)
            if plan.has_current:  # the current block (fill live tokens) belongs to the last rank
                kk = np.concatenate([kk, cur_k[j]])
                vv = np.concatenate([vv, cur_v[j]])
                valid = np.concatenate([valid, np.arange(bs) < fill])
            outs[j], lses[j] = O.attend_tokens(q.reshape(h, g, d)[j], kk, vv, d**-0.5, valid)
        go, gl = gather_partials(torch.from_numpy(outs.reshape(h * g, d)).float(), torch.from_numpy(lses.reshape(-1)).float())
        results[rank] = (go.numpy(), gl.numpy())
    finally:
        dist.destroy_process_group()


def _rank_candidates(rank: int, world: int, port: int, results: dict) -> None:  # noqa: ANN001
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        q, k, _, _, _, _ = _layer(seed=5)
        h, t, d = k.shape
        bs, n = 16, t // 16
        k = (np.round(k * 2) / 2).astype(np.float32)  # coarse keys: tied bounds across the shards
        kmin, kmax = O.block_minmax(k, bs)
        bound = O.quest_bound(q.astype(np.float32), kmin[:, 1:], kmax[:, 1:], "float32")  # candidates 1..n-1
        k_total = 9
        plan = shard_plan(n, k_total, world, rank)
        lo, hi = plan.cand_first - 1, plan.cand_first - 1 + plan.n_cand  # candidate indices of the shard
        kk = min(k_total, plan.n_cand)
        local = O.top_blocks(bound[:, lo:hi], kk) + lo  # shard's best candidates (indices)
        local = np.sort(local, axis=1)
        lb = np.take_along_axis(bound, local, axis=1)
        ids, bounds = gather_candidates(torch.from_numpy(local + 1).int(), torch.from_numpy(lb).float())
        results[rank] = (ids.numpy(), bounds.numpy(), bound, k_total)
    finally:
        dist.destroy_process_group()


def _spawn(fn, world: int) -> dict:  # noqa: ANN001
    ctx = mp.get_context("spawn")
    with ctx.Manager() as m:
        results = m.dict()
        port = _free_port()
        procs = [ctx.Process(target=fn, args=(r, world, port, results)) for r in range(world)]
        for p in procs:
            p.start()
        for p in procs:
            p.join(180)
        codes = [p.exitcode for p in procs]
        for p in procs:
            if p.is_alive():
                p.kill()
        assert codes == [0] * world, codes
        return dict(results)


def test_gathered_partials_merge_to_attention_over_the_whole_context() -> None:
    """Two gloo ranks each attend their range (sink on rank 0, current block on rank 1), exchange
    (out, lse) with gather_partials, and the merge of the gathered partials is dense attention."""
    res = _spawn(_rank_partials, 2)
    q, k, v, cur_k, cur_v, fill = _layer()
    h, t, d = k.shape
    g = q.shape[0] // h
    kk = np.concatenate([k, cur_k[:, :fill]], axis=1)
    vv = np.concatenate([v, cur_v[:, :fill]], axis=1)
    want, _ = O.dense_attention(q, kk, vv, d**-0.5)
    for rank in (0, 1):
        outs, lses = res[rank]
        assert outs.shape == (2, h * g, d) and lses.shape == (2, h * g)
        o, l = O.merge_lse(outs[0].astype(np.float64), lses[0].astype(np.float64), outs[1].astype(np.float64), lses[1].astype(np.float64))
        assert np.abs(o - want).max() < 1e-5 * np.abs(want).max()
    assert np.array_equal(res[0][0], res[1][0])  # every rank holds the same gathered partials


def test_gathered_candidates_give_the_single_gpu_selection() -> None:
    """Two gloo ranks exchange their best min(K, n_local) candidates (ascending ids, with bounds);
    the top-K over the gathered lists, ties to the lower id, is the unsharded selection."""
    res = _spawn(_rank_candidates, 2)
    ids, bounds, bound, k_total = res[0]
    assert np.array_equal(ids, res[1][0]) and np.array_equal(bounds, res[1][1])
    assert (np.diff(ids, axis=1) > 0).all()  # rank order = ascending ids
    got = host_reference_global_topk(ids, bounds, k_total)
    want = np.sort(O.top_blocks(bound, k_total) + 1, axis=1)
    assert np.array_equal(got, want)


def _rank_gathered_bounds(rank: int, world: int, port: int, results: dict) -> None:  # noqa: ANN001
    """GlobalSelection's protocol with the oracle's bounds in place of the kernel's: each rank scores
    its own candidates into a [h, ld] buffer (bf16-rounded, as the kernel stores them), one
    all-gather, then every rank's part of the global selection (host reference of
    lkv_topk_gathered)."""
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        q, k, _, _, _, _ = _layer(seed=7, n=61)
        h, t, d = k.shape
        bs, n = 16, t // 16
        k = (np.round(k * 2) / 2).astype(np.float32)  # coarse keys: ties at the threshold across ranks
        kmin, kmax = O.block_minmax(k, bs)
        k_total = 13
        plans = [shard_plan(n, k_total, world, r) for r in range(world)]
        seg_n, ld = gathered_layout(plans)
        p = plans[rank]
        bound = O.quest_bound(q.astype(np.float32), kmin[:, p.cand_first : p.cand_first + p.n_cand], kmax[:, p.cand_first : p.cand_first + p.n_cand],
                              "bfloat16")
        send = torch.zeros((h, ld), dtype=torch.float32)
        send[:, : p.n_cand] = torch.from_numpy(np.asarray(bound, dtype=np.float32))
        gathered = torch.zeros((world * h, ld), dtype=torch.float32)
        dist.all_gather_into_tensor(gathered, send)
        mine = host_reference_gathered_topk(gathered.view(world, h, ld).numpy(), seg_n, k_total, rank, p.cand_first - p.lo)
        parts = [None] * world
        dist.all_gather_object(parts, (mine, p.lo))
        results[rank] = (parts, k_total, q, kmin, kmax)
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 3])
def test_gathered_bounds_give_the_single_gpu_selection(world: int) -> None:
    """The ranks' parts of the global selection over all-gathered bounds, mapped back to block ids
    and concatenated in rank order, are the unsharded top-K (ties to the lower block ids)."""
    res = _spawn(_rank_gathered_bounds, world)
    parts, k_total, q, kmin, kmax = res[0]
    got = np.concatenate([np.where(m >= 0, m + lo, -1) for m, lo in parts], axis=1)
    bound = O.quest_bound(q.astype(np.float32), kmin[:, 1:], kmax[:, 1:], "bfloat16")
    want = np.sort(O.top_blocks(bound, k_total) + 1, axis=1)
    for j in range(got.shape[0]):
        row = got[j][got[j] >= 0]
        assert np.array_equal(row, want[j])
    assert all(np.array_equal(a[0], b[0]) for a, b in zip(parts, res[1][0]))  # every rank computed the same parts


def test_gathered_reference_edge_cases() -> None:
    """host_reference_gathered_topk: k at or above the candidates takes everything; all-equal bounds
    take the lowest ids across ranks; a rank with no candidates gets an empty, all -1 part."""
    g = np.zeros((3, 2, 5), dtype=np.float32)
    seg_n = [4, 0, 5]
    everything = [host_reference_gathered_topk(g, seg_n, 99, r, 0) for r in range(3)]
    assert everything[0].shape == (2, 4) and (everything[0] == np.arange(4)).all()
    assert everything[1].shape == (2, 0)
    assert (everything[2] == np.arange(5)).all()
    low = [host_reference_gathered_topk(g, seg_n, 6, r, 10) for r in range(3)]
    assert (low[0] == np.arange(10, 14)).all()  # the 4 lowest ids are rank 0's
    assert (low[2][:, :2] == [10, 11]).all() and (low[2][:, 2:] == -1).all()  # then rank 2's first 2
    g[2, 1, 4] = 1.0  # one higher bound on rank 2, head 1: it is taken first, a tie at the end drops
    part = host_reference_gathered_topk(g, seg_n, 6, 2, 0)
    assert part[1].tolist() == [0, 4, -1, -1, -1]
