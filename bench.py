"""Benchmark of the tiered decode-attention hot path at BASELINE's metric configuration.

Workload (BASELINE config 2 shapes at the metric's context): Llama-3.2-1B attention (32 query heads,
8 KV heads, head_dim 64), 131,072-token context in 16-token blocks, 25% budget
(K = blocks_for_budget = 2,046 selected of 8,190 candidates), 14 selecting layers (16 layers, the
first 2 dense). One step = one decode token through the hot path of the 14 selecting layers:
Quest scoring + device top-K -> split decode over the HBM-resident hot blocks -> exact pass over the
int8 cold blocks -> log-sum-exp merge. Data are seeded synthetic K/V (N(0,1), keys with a
per-(head, channel) offset of variance 0.5) with random queries, bf16; every layer has its own
buffers, so one step reads ~2.8 GB, far above the 126 MB L2 (no flush needed).

Residency: the hot slot pool holds exactly the blocks the step selects (the steady state in which
every selected block is already resident); the cold records live in HBM (`--cold device`, the
headline) or in pinned host memory read through zero-copy loads (`--cold host`, also reported).

Multi-GPU (torchrun): the context is sharded by block range across ranks (strong scaling of the
same 128K sequence); each rank selects K/N of its own candidates, runs both passes on its shard,
merges locally, and the per-rank (out, lse) partials are all-gathered with NCCL and merged.

`--impl reference` times the reference's algorithm on the host cores instead (the oracle port of
lazykv's CPU path: selection, the float32 partial attentions and the merge) on a bounded sample.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "decode tokens/s and us per layer-step at 128K ctx, 25% budget; % HBM roofline"
HQ, HKV, D, BS = 32, 8, 64, 16
N_LAYERS, DENSE = 16, 2


def parse() -> argparse.Namespace:
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=20)
    p.add_argument("--warmup", type=int, default=5)
    p.add_argument("--impl", choices=["ours", "reference"], default="ours")
    p.add_argument("--ctx", type=int, default=131072)
    p.add_argument("--budget", type=float, default=0.25)
    p.add_argument("--cold", choices=["device", "host"], default="device")
    p.add_argument("--no-host-leg", action="store_true", help="skip the zero-copy (host cold tier) measurement")
    p.add_argument("--no-cpu-baseline", action="store_true")
    p.add_argument("--layers", type=int, default=N_LAYERS - DENSE, help="selecting layers (the metric runs all 14; fewer for profiling)")
    p.add_argument("--workload", choices=["metric", "ragged"], default="metric",
                   help="ragged: BASELINE config 3 instead of the metric (64 sequences of 4K-128K tokens, 6.25%% budget, one layer)")
    p.add_argument("--profile-calls", action="store_true",
                   help="profiling target: build the layers, then call, twice each and eagerly on the first layer, the selection, the hot "
                        "pass alone, the cold pass alone and the fused attention; print nothing else")
    return p.parse_args()


def attention_traffic() -> int | None:
    """DRAM bytes (read + write) of one attention launch at this workload, from the committed ncu
    summary of that launch (null when the summary is absent)."""
    import re

    f = ROOT / "profiles" / "attn_stream_ctx128k.md"
    if not f.exists():
        return None
    m = re.search(r"traffic_bytes_per_launch\s*=\s*(\d+)", f.read_text())
    return int(m.group(1)) if m else None


def load_peaks() -> dict:
    f = ROOT / "MEASURED_PEAKS.json"
    if f.exists():
        d = json.loads(f.read_text())
        return {"hbm_gbs": float(d["hbm_gbs"]), "source": "measured"}
    return {"hbm_gbs": 6650.0, "source": "fallback"}


class Clocks:
    """nvidia-smi sampling during the timed region (clocks and throttle reasons)."""

    FIELDS = "index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap"

    def __init__(self, index: int) -> None:
        self.index = index
        self.proc: subprocess.Popen | None = None
        self.lines: list[str] = []

    def __enter__(self) -> "Clocks":
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits", "-lms", "100"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self._t = threading.Thread(target=self._read, daemon=True)
            self._t.start()
        except FileNotFoundError:
            self.proc = None
        return self

    def wait_first_sample(self, timeout: float) -> None:
        t0 = time.perf_counter()
        while self.proc is not None and not self.lines and time.perf_counter() - t0 < timeout:
            time.sleep(0.01)

    def _read(self) -> None:
        assert self.proc is not None and self.proc.stdout is not None
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *a: object) -> None:
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self) -> dict:
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in self.lines:
            f = [x.strip() for x in line.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx = float(f[2])
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx, "reasons": sorted(reasons), "samples": len(sm)}


# ---------------------------------------------------------------------------------------------
# our arm
# ---------------------------------------------------------------------------------------------


class Layer:
    """One selecting layer's device state for one rank's shard of the context."""


def build_layers(args: argparse.Namespace, rank: int, world: int, dev) -> tuple[list, dict]:
    import torch

    from lazykv_b200 import kernels as K
    from lazykv_b200.selection import blocks_for_budget

    nb = args.ctx // BS  # blocks in the context; the last one is the (full) current block
    n_sealed = nb - 1
    k_total = blocks_for_budget(args.budget, args.ctx, BS)
    # Shard the sealed blocks 0..n_sealed-1 by contiguous range (lkv_shard_plan): the sink on rank 0,
    # the current block on the last rank, the budget shared in proportion to the candidates.
    from lazykv_b200.sharded import shard_plan

    plan = shard_plan(n_sealed, k_total, world, rank)
    lo, hi, has_sink, has_cur = plan.lo, plan.hi, plan.has_sink, plan.has_current
    cand_lo, n_cand, k_local = plan.cand_first, plan.n_cand, plan.k_local
    if n_cand <= k_local:
        raise SystemExit(f"shard of {n_cand} candidates cannot select {k_local}")
    n_list = k_local + int(has_sink) + int(has_cur)
    n_slots = n_list
    scale = D**-0.5
    g = torch.Generator(device=dev).manual_seed(1234 + rank)
    layers = []
    torch.cuda.synchronize(dev)
    for li in range(args.layers):
        L = Layer()
        nblk = hi - lo
        off = torch.randn(HKV, 1, D, device=dev, generator=g) * 0.5**0.5
        kv = torch.randn(nblk, HKV, 2, BS, D, device=dev, generator=g)
        kv[:, :, 0] += off.view(1, HKV, 1, D)
        kv = kv.bfloat16()
        L.kmin = torch.empty((HKV, nblk, D), dtype=torch.bfloat16, device=dev)
        L.kmax = torch.empty_like(L.kmin)
        L.deq = torch.empty_like(kv)
        L.records = K.pack_int8(kv, kmin=L.kmin, kmax=L.kmax, deq=L.deq)  # [nblk, h, W], local block ids
        L.q = torch.randn(HQ, D, device=dev, generator=g).bfloat16()
        # Hot list [sink?, selected..., current?] (local block ids) and the bitmap of the cold pass.
        L.list = torch.zeros((HKV, n_list), dtype=torch.int32, device=dev)
        L.words = K.bitmap_words(nblk + 1)
        L.bitmap = torch.zeros((HKV, L.words), dtype=torch.int32, device=dev)
        sel_off = int(has_sink)
        if has_cur:
            L.list[:, -1] = nblk  # local id of the current block
        K.quest_topk(L.q, L.kmin, L.kmax, cand_lo - lo, n_cand, k_local, out_blocks=L.list[:, sel_off : sel_off + k_local], bitmap=L.bitmap,
                     by_block=True)
        # Steady-state residency: slot s holds the s-th listed block of each head.
        L.pool = torch.zeros((n_slots, HKV, 2, BS, D), dtype=torch.bfloat16, device=dev)
        L.slot_of = torch.zeros((HKV, nblk + 1), dtype=torch.int32, device=dev)
        heads = torch.arange(HKV, device=dev)[:, None].expand(HKV, n_list)
        slots = torch.arange(n_list, device=dev, dtype=torch.int32)[None].expand(HKV, n_list)
        L.slot_of[heads, L.list.long()] = slots
        ids = L.list.long().clamp(max=nblk - 1)
        L.pool.view(n_slots, HKV, -1)[slots.long(), heads] = L.deq.view(nblk, HKV, -1)[ids, heads]
        if has_sink:
            L.pool[0] = kv[0]  # the sink stays exact
        if has_cur:
            L.pool[n_slots - 1] = torch.randn(HKV, 2, BS, D, device=dev, generator=g).bfloat16()
        del kv
        L.deq = None
        if world == 1:
            L.out = torch.empty((HQ, D), dtype=torch.bfloat16, device=dev)
            L.lse = torch.empty((HQ,), dtype=torch.float32, device=dev)
            L.packed = None
        else:
            # One buffer per layer, out then lse: one all-gather per layer, merged in place.
            from lazykv_b200.sharded import PackedPartial

            L.packed = PackedPartial(HQ, D, world, dev)
            L.out, L.lse = L.packed.out, L.packed.lse
        L.records_host = None
        layers.append(L)
    torch.cuda.synchronize(dev)
    geo = dict(nb=nb, n_sealed=n_sealed, k_total=k_total, k_local=k_local, lo=lo, hi=hi, cand_lo=cand_lo, n_cand=n_cand, n_list=n_list,
               sel_off=int(has_sink), scale=scale, has_cur=has_cur)
    return layers, geo


def layer_step(L, geo: dict, cold_store=None, events: list | None = None) -> None:
    """One layer-step of the hot path (all launches on the current stream): score + top-K, then
    the hot and cold passes and their merge in one attention launch plus its combine."""
    from lazykv_b200 import kernels as K

    def mark() -> None:
        if events is not None:
            import torch

            e = torch.cuda.Event(enable_timing=True)
            e.record()
            events.append(e)

    mark()
    K.quest_topk(L.q, L.kmin, L.kmax, geo["cand_lo"] - geo["lo"], geo["n_cand"], geo["k_local"],
                 out_blocks=L.list[:, geo["sel_off"] : geo["sel_off"] + geo["k_local"]], bitmap=L.bitmap, by_block=True)
    mark()
    K.exact_attention(L.q, L.pool, L.pool[:, :, 1], (HKV * 2 * BS * D, 2 * BS * D, D), L.list, BS, L.records if cold_store is None else cold_store,
                      geo["cand_lo"] - geo["lo"], geo["n_cand"], geo["scale"], BS, excluded=L.bitmap, slot_of=L.slot_of, out=L.out, lse=L.lse)
    mark()


LAUNCHES_PER_LAYER_STEP = 2  # the single-launch selection (scores and radix select) and the attention (both passes; the head's last CTA folds)


def profile_calls(args: argparse.Namespace) -> None:
    """The kernel calls of one layer-step, each twice and eagerly, for a profiler to capture."""
    import torch

    from lazykv_b200 import kernels as K
    from lazykv_b200.build import build

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    build()
    layers, geo = build_layers(args, 0, 1, dev)
    L = layers[0]
    strides = (HKV * 2 * BS * D, 2 * BS * D, D)
    out = torch.empty((HQ, D), dtype=torch.float32, device=dev)
    lse = torch.empty((HQ,), dtype=torch.float32, device=dev)
    first = geo["cand_lo"] - geo["lo"]
    for _ in range(2):
        K.quest_topk(L.q, L.kmin, L.kmax, first, geo["n_cand"], geo["k_local"],
                     out_blocks=L.list[:, geo["sel_off"] : geo["sel_off"] + geo["k_local"]], bitmap=L.bitmap, by_block=True)
    for _ in range(2):
        K.hot_attention(L.q, L.pool, L.pool[:, :, 1], strides, L.list, BS, geo["scale"], BS, slot_of=L.slot_of, out=out, lse=lse)
    for _ in range(2):
        K.cold_attention(L.q, L.records, BS, first, geo["n_cand"], geo["scale"], excluded=L.bitmap, out=out, lse=lse)
    for _ in range(2):
        K.exact_attention(L.q, L.pool, L.pool[:, :, 1], strides, L.list, BS, L.records, first, geo["n_cand"], geo["scale"], BS,
                          excluded=L.bitmap, slot_of=L.slot_of, out=L.out, lse=L.lse)
    torch.cuda.synchronize()


def run_ours(args: argparse.Namespace) -> None:
    import torch
    import torch.distributed as dist

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    if world > 1:
        from datetime import timedelta

        dist.init_process_group("nccl", device_id=dev, timeout=timedelta(seconds=120))
    from lazykv_b200.build import build

    if rank == 0 or world == 1:
        build()
    if world > 1:
        dist.barrier()
    layers, geo = build_layers(args, rank, world, dev)
    n_steps, n_warm = args.steps, args.warmup
    finals = [torch.empty((HQ, D), dtype=torch.bfloat16, device=dev) for _ in layers]

    from lazykv_b200 import kernels as K

    def step(cold: str = "device") -> None:
        for i, L in enumerate(layers):
            layer_step(L, geo, None if cold == "device" else L.records_host)
            if world > 1:
                L.packed.exchange()
                L.packed.merge(torch.bfloat16, out=finals[i])

    # Warm-up (also compiles nothing: the library is prebuilt) and graph capture of one step (the
    # NCCL all-gathers are captured too at N > 1; the graph is released before the process group).
    for _ in range(n_warm):
        step()
    torch.cuda.synchronize()
    graph = None
    if True:
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            step()
        torch.cuda.current_stream().wait_stream(s)
        torch.cuda.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            step()
        for _ in range(n_warm):
            graph.replay()
        torch.cuda.synchronize()

    def soak(fn, seconds: float) -> None:
        # About `seconds` of back-to-back replays; the count is fixed from a short calibration and
        # agreed across ranks (the graph holds collectives at N > 1, so every rank replays alike).
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        for _ in range(5):
            fn()
        torch.cuda.synchronize()
        per = max((time.perf_counter() - t0) / 5, 1e-5)
        n = torch.tensor([min(100000, int(seconds / per) + 1)], device=dev)
        if world > 1:
            dist.all_reduce(n, op=dist.ReduceOp.MAX)
        for _ in range(int(n.item())):
            fn()
        torch.cuda.synchronize()

    def timed(fn, steps: int) -> float:
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        for _ in range(steps):
            fn()
        b.record()
        b.synchronize()
        ms = a.elapsed_time(b)
        if world > 1:
            t = torch.tensor([ms], device=dev)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            ms = float(t.item())
        return ms

    # Clocks: nvidia-smi samples every 100 ms, so the sampler runs over a window of back-to-back
    # replays (about half a second on either side) that contains the timed region.
    run = graph.replay if graph is not None else step
    with Clocks(local) as clocks:
        clocks.wait_first_sample(2.0)
        soak(run, 0.5)
        ms = timed(run, n_steps)
        soak(run, 0.5)
    ms_step = ms / n_steps
    n_sel = args.layers
    us_layer = ms_step * 1e3 / n_sel
    tokens_per_s = 1e3 / ms_step

    # Per-kernel durations: each kernel group (selection: score + select; attention) captured alone
    # over every layer in its own CUDA graph and replayed back to back, timed with CUDA events on
    # the replaying stream, per layer-step (the local part at N > 1: no exchange).
    names = ["select", "attention"]

    def sel_only() -> None:
        for L in layers:
            K.quest_topk(L.q, L.kmin, L.kmax, geo["cand_lo"] - geo["lo"], geo["n_cand"], geo["k_local"],
                         out_blocks=L.list[:, geo["sel_off"] : geo["sel_off"] + geo["k_local"]], bitmap=L.bitmap, by_block=True)

    def attn_only() -> None:
        for L in layers:
            K.exact_attention(L.q, L.pool, L.pool[:, :, 1], (HKV * 2 * BS * D, 2 * BS * D, D), L.list, BS, L.records, geo["cand_lo"] - geo["lo"],
                              geo["n_cand"], geo["scale"], BS, excluded=L.bitmap, slot_of=L.slot_of, out=L.out, lse=L.lse)

    kernel_us = {}
    for n, fn in zip(names, (sel_only, attn_only)):
        fn()
        torch.cuda.synchronize()
        g_k = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g_k):
            fn()
        for _ in range(3):
            g_k.replay()
        reps = max(5, n_steps)
        kernel_us[n] = timed(g_k.replay, reps) / reps * 1e3 / len(layers)  # max over ranks at N > 1
        del g_k

    peaks = load_peaks()
    k_local = geo["k_local"]
    hot_blocks = geo["n_list"]
    cold_blocks = geo["n_cand"] - k_local
    bytes_meta = HKV * geo["n_cand"] * D * 2 * 2
    bytes_hot = hot_blocks * HKV * 2 * BS * D * 2
    rec_w = K.packed_pair_bytes(BS, D)
    bytes_cold = cold_blocks * HKV * rec_w
    algo = {"select": bytes_meta, "attention": bytes_hot + bytes_cold}
    dominant = max(("select", "attention"), key=lambda n: kernel_us[n])
    achieved = algo[dominant] / (kernel_us[dominant] * 1e-6) / 1e9
    layer_bytes = bytes_meta + bytes_hot + bytes_cold

    # End to end through the public API with host buffers: per step, every layer's query comes
    # from pinned host memory and its output goes back to pinned host memory.
    q_host = [torch.empty((HQ, D), dtype=torch.bfloat16).pin_memory() for _ in layers]
    o_host = [torch.empty((HQ, D), dtype=torch.bfloat16).pin_memory() for _ in layers]
    for qh, L in zip(q_host, layers):
        qh.copy_(L.q.cpu())

    def e2e_step() -> None:
        for i, L in enumerate(layers):
            L.q.copy_(q_host[i], non_blocking=True)
            layer_step(L, geo)
            src = L.out if world == 1 else finals[i]
            if world > 1:
                L.packed.exchange()
                L.packed.merge(torch.bfloat16, out=finals[i])
            o_host[i].copy_(src, non_blocking=True)

    for _ in range(2):
        e2e_step()
    e2e_ms = timed(e2e_step, max(3, n_steps // 2)) / max(3, n_steps // 2)

    result = {
        "metric": METRIC,
        "value": round(tokens_per_s * (1 if world == 1 else 1), 3),
        "unit": "tokens/s",
        "n_gpus": world,
        "steps": n_steps,
        "warmup": n_warm,
        "ms_per_step": round(ms_step, 4),
        "us_per_layer_step": round(us_layer, 3),
        "higher_is_better": True,
        "scaling": "strong",
        "vs_baseline": None,
        "dtype": "bf16",
        "data": "synthetic (seeded N(0,1) K/V with key offsets, random queries; no weights involved)",
        "config": {"workload": "tiered decode hot path, Llama-3.2-1B attention (32q/8kv/d64), 131072-token context, bs 16, 25% budget (K=2046), 14 selecting layers, int8 cold tier in HBM",
                   "ctx": args.ctx, "block_size": BS, "k_blocks": geo["k_total"], "selecting_layers": n_sel, "batch": 1,
                   "cold_placement": "device", "l2": "inputs larger than L2 (~2.8 GB read per step)", "parallelism": f"context-sharded x{world}",
                   "timing": "CUDA graph of one step (NCCL all-gathers captured at N > 1), CUDA events, max over ranks"},
        "kernel_us": {k: round(v, 3) for k, v in kernel_us.items()},
        "roofline": {"bound": "hbm", "kernel": dominant, "achieved": round(achieved, 1), "peak": peaks["hbm_gbs"], "unit": "GB/s",
                     "frac": round(achieved / peaks["hbm_gbs"], 4),
                     "traffic": attention_traffic() if dominant == "attention" and args.ctx == 131072 and world == 1 else None,
                     "traffic_source": "ncu dram__bytes_read.sum + dram__bytes_write.sum of one attention launch at this workload",
                     "peak_source": peaks["source"],
                     "algorithmic_bytes": algo[dominant]},
        "layer_step_roofline": {"algorithmic_bytes": layer_bytes, "us": round(us_layer, 3),
                                "achieved_gbs": round(layer_bytes / (us_layer * 1e-6) / 1e9, 1),
                                "frac": round(layer_bytes / (us_layer * 1e-6) / 1e9 / peaks["hbm_gbs"], 4)},
        "e2e": {"value": round(1e3 / e2e_ms, 3), "unit": "tokens/s", "h2d_bytes_per_step": n_sel * HQ * D * 2,
                "d2h_bytes_per_step": n_sel * HQ * D * 2, "path": "lazykv_b200.kernels (C ABI) per layer, eager, host q in / host out"},
        "gpu_launches": n_steps * n_sel * (LAUNCHES_PER_LAYER_STEP + (1 if world > 1 else 0)),  # + the merge kernel at N > 1 (NCCL's own kernels not counted)
        "clocks": clocks.summary(),
    }

    # Zero-copy leg: the same step with the cold records in pinned host memory.
    if world == 1 and not args.no_host_leg:
        from lazykv_b200.pinned import device_view, pinned_empty

        for L in layers:
            h = pinned_empty(tuple(L.records.shape), torch.uint8)
            h.copy_(L.records.cpu())
            L.records_host_cpu = h
            L.records_host = device_view(h)
        torch.cuda.synchronize()
        for _ in range(2):
            step("host")
        hs = max(2, n_steps // 4)
        hms = timed(lambda: step("host"), hs) / hs
        cold_us = []
        for L in layers[:4]:
            ev: list = []
            layer_step(L, geo, L.records_host, ev)
            torch.cuda.synchronize()
            cold_us.append(ev[1].elapsed_time(ev[2]) * 1e3)
        cu = statistics.median(cold_us)
        result["host_cold_tier"] = {"value": round(1e3 / hms, 3), "unit": "tokens/s", "us_per_layer_step": round(hms * 1e3 / n_sel, 1),
                                    "attention_us": round(cu, 1), "link_gbs": round(bytes_cold / (cu * 1e-6) / 1e9, 2),
                                    "link_peak_gbs": 55.5, "link_peak_source": "pinned H2D copy measured on this pool's B200 hosts (PCIe 5 x16)"}

    if rank == 0 and not args.no_cpu_baseline:
        result["cpu_baseline"] = cpu_baseline(args, budget_s=12.0)
    if rank == 0:
        print(json.dumps(result), flush=True)
    if world > 1:
        # The graph holds NCCL work: every reference to it (the graph and its bound replay) goes
        # before the process group does, or the group's destruction waits for it for good.
        import gc

        del run, graph
        gc.collect()
        torch.cuda.synchronize()
        dist.barrier()
        dist.destroy_process_group()


# ---------------------------------------------------------------------------------------------
# reference arm: the reference's algorithm on the host cores (the oracle port)
# ---------------------------------------------------------------------------------------------


def cpu_layer_inputs(args: argparse.Namespace, seed: int = 7) -> dict:
    rng = np.random.default_rng(seed)
    t = args.ctx
    off = rng.standard_normal((HKV, 1, D), dtype=np.float32) * np.float32(0.5**0.5)
    k = (rng.standard_normal((HKV, t, D), dtype=np.float32) + off)
    v = rng.standard_normal((HKV, t, D), dtype=np.float32)
    # bf16 values, float32 mirror (lazykv/exact.py:130-152 keeps a float32 copy of the bf16 tier)
    import oracle as O

    k, v = O.bf16_round(k), O.bf16_round(v)
    q = O.bf16_round(rng.standard_normal((HQ, D), dtype=np.float32))
    nb = t // BS
    kmin, kmax = O.block_minmax(k, BS)
    return {"k": k, "v": v, "q": q, "kmin": kmin, "kmax": kmax, "nb": nb}


def cpu_layer_step(x: dict, k_blocks: int) -> np.ndarray:
    """One layer-step of the reference's algorithm on CPU: lazykv/selection.py:38-62 (bound + top-K),
    lazykv/exact.py:88-127 twice (the hot set and every other sealed block, masked), :69-85 merge."""
    import oracle as O

    nb = x["nb"]
    n_full = nb - 1
    bound = O.quest_bound(x["q"], x["kmin"][:, 1:n_full], x["kmax"][:, 1:n_full], "bfloat16")
    sel = O.top_blocks(bound, k_blocks) + 1
    qg = x["q"].reshape(HKV, HQ // HKV, D)
    hot = np.concatenate([np.zeros((HKV, 1), np.int64), sel, np.full((HKV, 1), n_full)], axis=1)
    scale = D**-0.5
    allb = np.arange(nb)
    rest = np.stack([np.setdiff1d(allb, hot[j]) for j in range(HKV)])
    ho, hl = O.cpu_partial_attention(x["k"], x["v"], qg, scale, BS, rest)
    co, cl = O.cpu_partial_attention(x["k"][:, : n_full * BS], x["v"][:, : n_full * BS], qg, scale, BS, hot[:, :-1])
    out, _ = O.merge_lse(ho, hl, co, cl)
    return out


def cpu_baseline(args: argparse.Namespace, budget_s: float = 12.0) -> dict:
    from lazykv_b200.selection import blocks_for_budget

    x = cpu_layer_inputs(args)
    k = blocks_for_budget(args.budget, args.ctx, BS)
    cpu_layer_step(x, k)  # warm
    times = []
    t_end = time.perf_counter() + budget_s
    while time.perf_counter() < t_end or not times:
        t0 = time.perf_counter()
        cpu_layer_step(x, k)
        times.append(time.perf_counter() - t0)
    per_layer = statistics.median(times)
    n_sel = args.layers
    return {"value": round(1.0 / (per_layer * n_sel), 4), "unit": "tokens/s", "cores": os.cpu_count(), "kind": "port",
            "sample": f"{len(times)} layer-steps of one selecting layer at {args.ctx} tokens (numpy port of the reference's CPU path: bf16 bound + top-K, two float32 partial attentions over the full mirror, LSE merge); tokens/s = 1 / (14 x median layer-step); BLAS multithreaded, elementwise single-threaded",
            "us_per_layer_step": round(per_layer * 1e6, 1)}


def run_reference(args: argparse.Namespace) -> None:
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    n_steps, n_warm = max(1, args.steps), max(0, args.warmup)
    x = cpu_layer_inputs(args)
    from lazykv_b200.selection import blocks_for_budget

    k = blocks_for_budget(args.budget, args.ctx, BS)
    for _ in range(min(n_warm, 1)):
        cpu_layer_step(x, k)
    # Each step is a bounded sample of the workload: one selecting layer's layer-step, scaled to a
    # token by the 14 selecting layers.
    times = []
    for _ in range(min(n_steps, 20)):
        t0 = time.perf_counter()
        cpu_layer_step(x, k)
        times.append(time.perf_counter() - t0)
    per_layer = statistics.median(times)
    n_sel = args.layers
    value = 1.0 / (per_layer * n_sel)
    print(json.dumps({
        "impl": "reference", "metric": METRIC, "value": round(value, 4), "unit": "tokens/s", "n_gpus": int(os.environ.get("WORLD_SIZE", "1")),
        "steps": len(times), "warmup": n_warm, "ms_per_step": round(per_layer * n_sel * 1e3, 2), "us_per_layer_step": round(per_layer * 1e6, 1),
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded)",
        "config": {"workload": "tiered decode hot path at 131072 tokens, 25% budget, on the host cores", "ctx": args.ctx, "k_blocks": k},
        "cpu_baseline": {"value": round(value, 4), "unit": "tokens/s", "cores": os.cpu_count(), "kind": "port",
                         "sample": f"{len(times)} layer-steps of one selecting layer (numpy port of lazykv's CPU exact path), scaled x14 layers"},
        "e2e": {"value": round(value, 4), "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }))


def run_ragged(args: argparse.Namespace) -> None:
    """ragged continuous batching. 64 sequences with lengths uniform in [4,096,
    131,072] (seeded), Llama-3.2-1B attention shapes, 6.25% budget, the int8 store in HBM, one
    selecting layer. A step is one decode token of every sequence through that layer (selection and
    the exact attention, the kept blocks read in place from the store), timed with CUDA events; between
    timed steps each sequence appends its token and, at random, a sequence finishes and a new one of
    random length takes its slot (untimed, as a prefill would be). Prints one JSON line."""
    import torch

    from lazykv_b200.ragged import RaggedTier

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    n_seqs, lo, hi, budget = 64, 4096, 131072, 0.0625
    rng = np.random.default_rng(3)
    gen = torch.Generator(device=dev).manual_seed(3)
    steps = args.steps + args.warmup
    max_tokens = hi + steps + 16
    store = n_seqs * (-(-max_tokens // BS) + 1)
    tier = RaggedTier(HKV, HQ // HKV, D, BS, max_seqs=n_seqs, max_tokens=max_tokens, store_blocks=store, budget=budget, device=dev)

    def new_seq() -> int:
        n = int(rng.integers(lo, hi + 1))
        off = torch.randn((HKV, 1, D), generator=gen, device=dev) * 0.5 ** 0.5
        keys = (torch.randn((HKV, n, D), generator=gen, device=dev) + off).bfloat16()
        values = torch.randn((HKV, n, D), generator=gen, device=dev).bfloat16()
        return tier.add(keys, values)

    ids = [new_seq() for _ in range(n_seqs)]
    scale = D ** -0.5
    times, toks, nbytes = [], [], []
    with Clocks(0) as clocks:
        for step in range(steps):
            ids.sort()
            q = torch.randn((len(ids) * HQ, D), generator=gen, device=dev).bfloat16()
            # algorithmic bytes of the step: every candidate's bounds and record (kept blocks are
            # attended in place from the store), the sink and the current block
            b = 0
            for s in ids:
                nc = tier.seqs[s].n_sealed - 1
                b += HKV * (nc * (2 * D * 2 + tier.W) + 2 * 2 * BS * D * 2)
            torch.cuda.synchronize()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            tier.decode(ids, q, scale)
            e1.record()
            torch.cuda.synchronize()
            if step >= args.warmup:
                times.append(e0.elapsed_time(e1) / 1e3)
                toks.append(len(ids))
                nbytes.append(b)
            kv = torch.randn((len(ids), 2, HKV, D), generator=gen, device=dev).bfloat16()
            for i, s in enumerate(ids):
                tier.append(s, kv[i, 0], kv[i, 1])
            if rng.random() < 1 / 8:  # a sequence finishes; a new one takes its slot
                gone = ids.pop(int(rng.integers(len(ids))))
                tier.drop(gone)
                ids.append(new_seq())
    total_s = sum(times)
    value = sum(toks) / total_s
    achieved = sum(nbytes) / total_s / 1e9
    peak = json.loads((ROOT / "MEASURED_PEAKS.json").read_text()).get("hbm_gbs") if (ROOT / "MEASURED_PEAKS.json").exists() else None
    peak_src = "measured" if peak else "fallback"
    peak = peak or 6650.0
    print(json.dumps({
        "metric": "ragged decode tokens/s per selecting layer (config 3: 64 sequences, ctx U[4096, 131072], 6.25% budget)",
        "value": round(value, 1), "unit": "tokens/s", "n_gpus": 1, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(1e3 * total_s / len(times), 4), "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "bf16", "data": "synthetic (seeded N(0,1) K/V with per-head key offsets, random queries)",
        "config": {"workload": "ragged continuous batching, Llama-3.2-1B attention (32q/8kv/d64), 64 sequences, lengths U[4096, 131072], "
                               "bs 16, 6.25% budget, int8 store in HBM (kept blocks attended in place), one selecting layer",
                   "l2": "inputs larger than L2 (~GBs per step)", "timing": "CUDA events around each decode step (host-built schedule included)"},
        "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s", "frac": round(achieved / peak, 4),
                     "traffic": None, "peak_source": peak_src, "algorithmic_bytes_per_step": int(statistics.mean(nbytes))},
        "gpu_launches": 3 * len(times),
        "clocks": clocks.summary(),
    }))


def main() -> None:
    args = parse()
    if args.impl == "reference":
        run_reference(args)
    elif args.workload == "ragged":
        run_ragged(args)
    elif args.profile_calls:
        profile_calls(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
