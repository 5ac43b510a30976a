"""The exchange of partials by peer stores (lkv_exchange_merge): the n-way log-sum-exp merge of
lazykv/exact.py:69-85 over what every rank pushed. On one GPU: a one-rank exchange returns its own
partial; a two-rank exchange whose peer never runs times out into the status word and its own
partial; the peer then arriving finds both ranks' rows and merges them (sequential launches, none
waits for the other). On two GPUs (skipped with fewer): two ranks exchanging every step, eagerly
and from a CUDA graph, against the merge of the all-gathered partials."""

from __future__ import annotations

import ctypes
import os
import socket

import pytest
import torch

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _ref_merge(outs: torch.Tensor, lses: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """[n, rows, d], [n, rows] float32 -> merged (float64)."""
    lse = torch.logsumexp(lses.double(), dim=0)
    w = torch.exp(lses.double() - lse)
    return (w[..., None] * outs.double()).sum(0), lse


def _partial(rows: int, d: int, seed: int) -> tuple[torch.Tensor, torch.Tensor]:
    g = torch.Generator(device=DEV).manual_seed(seed)
    return torch.randn((rows, d), device=DEV, generator=g), torch.randn((rows,), device=DEV, generator=g) * 3


def test_one_rank_returns_its_own_partial() -> None:
    from lazykv_b200 import kernels as K
    from lazykv_b200.sharded import PeerExchange

    x = PeerExchange(32, 64)
    for step in range(5):  # both inbox halves, twice
        o, l = _partial(32, 64, step)
        x.out.copy_(o)
        x.lse.copy_(l)
        merged = torch.empty((32, 64), dtype=torch.float32, device=DEV)
        mlse = torch.empty((32,), dtype=torch.float32, device=DEV)
        x.exchange(merged, mlse)
        torch.cuda.synchronize()
        assert torch.allclose(merged, o, rtol=1e-6, atol=1e-6) and torch.allclose(mlse, l, rtol=1e-6, atol=1e-6)
    assert K.device_status(clear=True) == 0
    x.close()


def test_absent_peer_times_out_then_its_late_rows_merge() -> None:
    from lazykv_b200 import _lib as L
    from lazykv_b200 import kernels as K

    rows, d = 12, 64
    bases = []
    for _ in range(2):
        b = ctypes.c_void_p()
        L.call("lkv_exchange_alloc", rows, d, 2, ctypes.byref(b), (ctypes.c_char * 64)())
        bases.append(b.value)
    arr = (ctypes.c_void_p * 2)(*bases)
    parts = [_partial(rows, d, 10 + r) for r in range(2)]
    outs = [torch.empty((rows, d), dtype=torch.float32, device=DEV) for _ in range(2)]
    lses = [torch.empty((rows,), dtype=torch.float32, device=DEV) for _ in range(2)]
    K.device_status(clear=True)
    try:
        K.debug_set(L.LKV_DEBUG_EXCHANGE_WAIT_ITERS, 2000)  # about a millisecond
        # Rank 0 alone: its wait for rank 1 runs out; its output is its own partial.
        L.call("lkv_exchange_merge", L.ptr(parts[0][0]), L.ptr(parts[0][1]), rows, d, 2, 0, arr, L.ptr(outs[0]), L.dtype_code(torch.float32),
               L.ptr(lses[0]), L.stream_handle())
        torch.cuda.synchronize()
        assert K.device_status(clear=True) == 1
        K.status_attach(torch.device(DEV, torch.cuda.current_device()))
        K.status_poll(clear=True)  # the host mirror too, so that no later caller sees this planned timeout
        assert torch.equal(outs[0], parts[0][0]) and torch.equal(lses[0], parts[0][1])
        # Rank 1 arrives late: rank 0's rows are already in its inbox, so it merges both at once.
        L.call("lkv_exchange_merge", L.ptr(parts[1][0]), L.ptr(parts[1][1]), rows, d, 2, 1, arr, L.ptr(outs[1]), L.dtype_code(torch.float32),
               L.ptr(lses[1]), L.stream_handle())
        torch.cuda.synchronize()
        assert K.device_status(clear=True) == 0
        want_o, want_l = _ref_merge(torch.stack([p[0] for p in parts]), torch.stack([p[1] for p in parts]))
        assert torch.allclose(outs[1].double(), want_o, rtol=1e-5, atol=1e-5) and torch.allclose(lses[1].double(), want_l, rtol=1e-5, atol=1e-5)
    finally:
        K.debug_set(L.LKV_DEBUG_EXCHANGE_WAIT_ITERS, 1 << 22)
        torch.cuda.synchronize()
        for b in bases:
            L.call("lkv_exchange_free", ctypes.c_void_p(b))


def test_bad_arguments_raise() -> None:
    from lazykv_b200 import _lib as L

    b = ctypes.c_void_p()
    with pytest.raises(L.LkvError):  # d not a multiple of 4
        L.call("lkv_exchange_alloc", 4, 6, 2, ctypes.byref(b), (ctypes.c_char * 64)())
    with pytest.raises(L.LkvError):  # world above 64
        L.call("lkv_exchange_alloc", 4, 64, 65, ctypes.byref(b), (ctypes.c_char * 64)())


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _two_rank_worker(rank: int, port: int, rows: int, d: int, steps: int) -> None:
    import datetime

    import torch.distributed as dist

    from lazykv_b200 import kernels as K
    from lazykv_b200.sharded import PeerExchange

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=2, device_id=dev, timeout=datetime.timedelta(seconds=60))
    try:
        x = PeerExchange(rows, d, device=dev)
        merged = torch.empty((rows, d), dtype=torch.bfloat16, device=dev)
        mlse = torch.empty((rows,), dtype=torch.float32, device=dev)
        gen = torch.Generator(device=dev).manual_seed(100 + rank)

        def check() -> None:
            allp = torch.empty((2, rows * (d + 1)), dtype=torch.float32, device=dev)
            dist.all_gather_into_tensor(allp, x.buf)
            want_o, want_l = _ref_merge(allp[:, : rows * d].view(2, rows, d), allp[:, rows * d :])
            err = (merged.double() - want_o).abs().max().item()
            assert err <= 2.0**-8 * want_o.abs().max().item() + 1e-6, err
            assert torch.allclose(mlse.double(), want_l, rtol=1e-5, atol=1e-5)

        for _ in range(steps):  # eager
            x.out.copy_(torch.randn((rows, d), device=dev, generator=gen))
            x.lse.copy_(torch.randn((rows,), device=dev, generator=gen))
            x.exchange(merged, mlse)
            torch.cuda.synchronize()
            check()
        graph = torch.cuda.CUDAGraph()
        side = torch.cuda.Stream()
        with torch.cuda.stream(side), torch.cuda.graph(graph, stream=side):
            x.exchange(merged, mlse)
        for _ in range(steps):  # the same launch, replayed
            x.out.copy_(torch.randn((rows, d), device=dev, generator=gen))
            x.lse.copy_(torch.randn((rows,), device=dev, generator=gen))
            torch.cuda.synchronize()
            graph.replay()
            torch.cuda.synchronize()
            check()
        del graph
        assert K.device_status(clear=True) == 0
        dist.barrier()
        x.close()
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_two_ranks_exchange_every_step() -> None:
    import torch.multiprocessing as mp

    mp.spawn(_two_rank_worker, args=(_free_port(), 256, 128, 6), nprocs=2, join=True)
