"""Context sharding over NCCL on two GPUs (skipped with fewer): each rank holds one shard of a
layer, runs ShardedExactStep.step (local selection, hot + cold passes, one all-gather of the packed
partials, lkv_lse_merge_packed), and every rank's output equals the single-GPU exact step."""

from __future__ import annotations

import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank(rank: int, world: int, port: int, results: dict) -> None:  # noqa: ANN001
    import torch.distributed as dist
    from datetime import timedelta

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev, timeout=timedelta(seconds=60))
    try:
        from tests.test_sharded_gpu import _layer, _shard_step
        from lazykv_b200 import kernels as K
        from lazykv_b200.sharded import shard_plan

        torch.cuda.set_device(dev)
        L = _layer(900, seed=11)  # the same seeded layer on every rank
        h, d, bs, n = L["h"], L["d"], L["bs"], L["n"]
        k_total = 200
        plan = shard_plan(n, k_total, world, rank)
        st = _shard_step(L, plan, torch.zeros((h, plan.k_local), dtype=torch.int32, device=dev))
        got = st.step(L["q"], torch.float32)
        torch.cuda.synchronize()
        # the single-GPU exact step on this rank's copy of the whole layer
        pool = torch.cat([L["deq"], L["cur"][None]], dim=0).contiguous()
        sel, _ = K.quest_topk(L["q"], L["kmin"], L["kmax"], 1, n - 1, k_total, by_block=True)
        hot = torch.cat([torch.zeros((h, 1), dtype=torch.int32, device=dev), sel, torch.full((h, 1), n, dtype=torch.int32, device=dev)], 1).contiguous()
        bm = torch.zeros((h, (n + 32) // 32 + 1), dtype=torch.int32, device=dev)
        K.quest_topk(L["q"], L["kmin"], L["kmax"], 1, n - 1, k_total, bitmap=bm, by_block=True)
        want, _ = K.exact_attention(L["q"], pool, pool[:, :, 1], (h * 2 * bs * d, 2 * bs * d, d), hot, L["fill"], L["rec"], 1, n - 1, d**-0.5, bs,
                                    excluded=bm, out_dtype=torch.float32)
        err = ((got - want).abs().max() / want.abs().max()).item()
        results[rank] = err
    finally:
        dist.destroy_process_group()


def test_two_gpu_sharded_step_equals_the_single_gpu_step() -> None:
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    world = 2
    ctx = mp.get_context("spawn")
    with ctx.Manager() as m:
        results = m.dict()
        port = _free_port()
        procs = [ctx.Process(target=_rank, args=(r, world, port, results)) for r in range(world)]
        for p in procs:
            p.start()
        for p in procs:
            p.join(240)
        codes = [p.exitcode for p in procs]
        for p in procs:
            if p.is_alive():
                p.kill()
        assert codes == [0] * world, codes
        for r in range(world):
            assert results[r] < 1e-5, dict(results)
