"""Benchmark of the tiered decode-attention hot path at BASELINE's metric configuration.

Workload (BASELINE config 2 shapes at the metric's context): Llama-3.2-1B attention (32 query heads,
8 KV heads, head_dim 64), 131,072-token context in 16-token blocks, 25% budget
(K = blocks_for_budget = 2,046 selected of 8,190 candidates), 14 selecting layers (16 layers, the
first 2 dense). One step = one decode token through the hot path of the 14 selecting layers:
Quest scoring + device top-K -> device LRU admit and the fetch of the missed blocks into HBM slots
-> split decode over the hot blocks -> exact pass over the int8 cold blocks -> log-sum-exp merge.
Data are seeded synthetic K/V (N(0,1), keys with a per-(head, channel) offset of variance 0.5),
bf16; every layer has its own buffers, so one step reads ~2.8 GB, far above the 126 MB L2 (no
flush needed).

Residency churn: each layer holds a ring of queries (a base query plus a drift of N(0,1) noise),
decode token s uses query s mod the ring, and the admit runs in every layer-step, so each step
fetches the blocks its selection newly wants (a hit rate near 0.84 at the default drift; the
reference measured 0.79-1.0 with real models). The cold records live in HBM (`--cold device`, the
headline) or, in a second leg, in pinned host memory read through zero-copy loads.

Multi-GPU (torchrun): the context is sharded by block range across ranks (strong scaling of the
same 128K sequence); each rank selects K/N of its own candidates, runs both passes on its shard,
and one launch per layer pushes its (out, lse) partial to every peer over NVLink and merges what
arrived (lkv_exchange_merge: peer stores, no collective in the step).

Further legs in the same JSON line: `long_ctx` (8 sequences of 1,048,576 tokens at head_dim 128,
a global top-K across the shards, at every N), and at N = 1 `model_decode` (the random-init
16-layer model through the attention hook: 32,768-token prefill, 128 greedy steps) and
`capacity_sweep` (130,048-token layer-major prefill, four budgets).

`--impl reference` times the reference's own CPU implementation of the path on the host cores instead:
the unmodified reference installed under baseline/_ref (lazykv.selection.top_blocks, two
lazykv.exact.cpu_partial_attention passes and merge_lse per selecting layer, torch on every core).
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
    p.add_argument("--queries", type=int, default=8, help="queries in each layer's ring: decode token s uses query s mod this")
    p.add_argument("--drift", type=float, default=0.15, help="a ring query is a base query + drift x N(0,1) (0.15: a hit rate near 0.84, inside the 0.79-1.0 the reference measured with real models)")
    p.add_argument("--admit-first", action="store_true",
                   help="admit and fetch before the attention on one stream (default: the resident selection, the attention, and the admit "
                        "beside it on a side stream)")
    p.add_argument("--no-model", action="store_true", help="skip the model legs (32K-token greedy decode; the 130,048-token capacity sweep)")
    p.add_argument("--no-long-ctx", action="store_true", help="skip the 1,048,576-token leg (8 sequences, head_dim 128, global top-K)")
    p.add_argument("--long-layers", type=int, default=4, help="layers of the long-context leg held and timed (each 30 GB at N = 1)")
    p.add_argument("--long-steps", type=int, default=32, help="timed decode steps of the long-context leg")
    p.add_argument("--workload", choices=["metric", "ragged"], default="metric",
                   help="ragged: BASELINE config 3 instead of the metric (64 sequences of 4K-128K tokens, 6.25%% budget, one layer)")
    p.add_argument("--ragged-cold", choices=["host", "device"], default="host",
                   help="ragged: the int8 cold tier in pinned host memory read over the link (config 3), or in HBM")
    p.add_argument("--profile-long", action="store_true",
                   help="with --profile-calls: the long-context geometry (64 rows, d 128) at --ctx tokens, its selection, global select, "
                        "admit, attention and exchange kernels")
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


NEVER = -(2**40)  # "evicted at" of a block never evicted (the tier's convention)


def metric_shape(args: argparse.Namespace) -> dict:
    """The metric's geometry: Llama-3.2-1B attention at the bench's context, budget and layer count."""
    return dict(ctx=args.ctx, h=HKV, hq=HQ, d=D, layers=args.layers, budget=args.budget, queries=max(1, getattr(args, "queries", 1)),
                drift=getattr(args, "drift", 0.15), seed=1234)


def build_layers(args: argparse.Namespace, rank: int, world: int, dev, keep_source: bool = False, shape: dict | None = None,
                 global_select: bool = False) -> tuple[list, dict]:
    """Every selecting layer's device state for this rank's shard, laid out as the tier keeps it:
    int8 records of the sealed blocks (local ids) in HBM, the bf16 min/max key metadata, a slot pool
    [K + 2, h, 2, bs, d] (slot 0 the exact sink on rank 0, slots 1..K the admitted blocks, slot K + 1
    the current block on the last rank), the residency tables of the device admit, and a ring of
    `queries` queries (a base query plus `drift` x N(0, 1), rounded to bf16: the queries of
    successive decode steps, which select overlapping but different blocks). `shape` gives the
    geometry (context, KV rows h, query rows hq, head_dim d, layers, budget; the metric's by
    default); rows may be several sequences' KV heads, which every kernel takes as more heads. The
    blocks are generated and packed in chunks. With `keep_source`, a layer also keeps its sealed
    blocks (L.kv, bf16 [blocks, h, 2, bs, d]) and its current block (L.cur). With `global_select`
    the rank holds whatever part of one global top-K falls in its range (sharded.GlobalSelection):
    its slots, chosen ids and hot list take min(K, candidates) entries per row instead of its
    proportional share."""
    import torch

    from lazykv_b200 import kernels as K
    from lazykv_b200.selection import blocks_for_budget

    sh = shape or metric_shape(args)
    h, hq, d = sh["h"], sh["hq"], sh["d"]
    nb = sh["ctx"] // BS  # blocks in the context; the last one is the (full) current block
    n_sealed = nb - 1
    k_total = blocks_for_budget(sh["budget"], sh["ctx"], BS)
    # Shard the sealed blocks 0..n_sealed-1 by contiguous range (lkv_shard_plan): the sink on rank 0,
    # the current block on the last rank, the budget shared in proportion to the candidates.
    from lazykv_b200.sharded import shard_plan

    plan = shard_plan(n_sealed, k_total, world, rank)
    lo, hi, has_sink, has_cur = plan.lo, plan.hi, plan.has_sink, plan.has_current
    cand_lo, n_cand, k_local = plan.cand_first, plan.n_cand, plan.k_local
    if global_select:
        k_local = min(k_total, n_cand)
    elif n_cand <= k_local:
        raise SystemExit(f"shard of {n_cand} candidates cannot select {k_local}")
    n_list = k_local + int(has_sink) + int(has_cur)
    sel_off = int(has_sink)
    scale = d**-0.5
    n_q, drift = sh["queries"], sh["drift"]
    g = torch.Generator(device=dev).manual_seed(sh["seed"] + rank)
    nblk = hi - lo
    chunk = max(1, (1 << 31) // (h * 2 * BS * d * 2))  # blocks generated at once: 2 GiB of bf16 pairs
    layers = []
    torch.cuda.synchronize(dev)
    for li in range(sh["layers"]):
        L = Layer()
        off = torch.randn(h, 1, d, device=dev, generator=g) * 0.5**0.5
        L.kmin = torch.empty((h, nblk, d), dtype=torch.bfloat16, device=dev)
        L.kmax = torch.empty_like(L.kmin)
        L.records = torch.empty((nblk, h, K.packed_pair_bytes(BS, d)), dtype=torch.uint8, device=dev)  # local block ids
        kv_all = []
        sink = None
        for c0 in range(0, nblk, chunk):
            c1 = min(nblk, c0 + chunk)
            kv = torch.randn(c1 - c0, h, 2, BS, d, device=dev, generator=g)
            kv[:, :, 0] += off.view(1, h, 1, d)
            kv = kv.bfloat16()
            K.pack_int8(kv, records=L.records[c0:c1], kmin=L.kmin, kmax=L.kmax, first_block=c0)
            if c0 == 0:
                sink = kv[0].clone()
            if keep_source:
                kv_all.append(kv)
            del kv
        q_base = torch.randn(hq, d, device=dev, generator=g)
        L.q_ring = (q_base[None] + drift * torch.randn(n_q, hq, d, device=dev, generator=g)).bfloat16()
        L.q = L.q_ring[0]
        # Hot list [sink slot?, admitted slots..., current slot?] and the bitmap of the cold pass.
        L.list = torch.zeros((h, n_list), dtype=torch.int32, device=dev)
        if has_cur:
            L.list[:, -1] = k_local + 1
        L.chosen = torch.zeros((h, k_local), dtype=torch.int32, device=dev)  # the selection, local block ids ascending
        L.words = K.bitmap_words(nblk + 1)
        L.bitmap = torch.zeros((h, L.words), dtype=torch.int32, device=dev)
        L.pool = torch.zeros((k_local + 2, h, 2, BS, d), dtype=torch.bfloat16, device=dev)
        if has_sink:
            L.pool[0] = sink  # the sink stays exact
        if has_cur:
            L.pool[k_local + 1] = torch.randn(h, 2, BS, d, device=dev, generator=g).bfloat16()
        # Residency tables (lazykv/tiered.py:281-288): nothing resident yet; the first step admits.
        L.block_slot = torch.full((h, nblk), -1, dtype=torch.int32, device=dev)
        L.slot_block = torch.full((h, k_local), -1, dtype=torch.int32, device=dev)
        L.last_used = torch.full((h, k_local), -2, dtype=torch.int64, device=dev)
        L.evicted_at = torch.full((h, nblk), NEVER, dtype=torch.int64, device=dev)
        L.miss_blk = torch.zeros((h, k_local), dtype=torch.int32, device=dev)
        L.miss_slot = torch.zeros((h, k_local), dtype=torch.int32, device=dev)
        L.n_miss = torch.zeros((h,), dtype=torch.int32, device=dev)
        L.kv = torch.cat(kv_all) if keep_source else None
        L.cur = L.pool[k_local + 1].clone() if keep_source and has_cur else None
        del kv_all, sink
        if world == 1:
            L.out = torch.empty((hq, d), dtype=torch.bfloat16, device=dev)
            L.lse = torch.empty((hq,), dtype=torch.float32, device=dev)
            L.xchg = None
        else:
            # The rank's partial lives in its exchange buffer; one launch per layer pushes it to
            # every peer over NVLink and merges what arrived (lkv_exchange_merge).
            from lazykv_b200.sharded import PeerExchange

            L.xchg = PeerExchange(hq, d, device=dev)
            L.out, L.lse = L.xchg.out, L.xchg.lse
        L.records_host = None
        layers.append(L)
    torch.cuda.synchronize(dev)
    geo = dict(nb=nb, n_sealed=n_sealed, k_total=k_total, k_local=k_local, lo=lo, hi=hi, cand_lo=cand_lo, n_cand=n_cand, n_list=n_list,
               sel_off=sel_off, scale=scale, has_cur=has_cur, n_q=n_q, h=h, hq=hq, d=d, global_select=global_select)
    return layers, geo


def select_call(L, geo: dict, r: int = 0) -> None:  # noqa: ANN001
    """Quest bound + device top-K of query r (block order) into L.chosen, and the bitmap."""
    from lazykv_b200 import kernels as K

    K.quest_topk(L.q_ring[r], L.kmin, L.kmax, geo["cand_lo"] - geo["lo"], geo["n_cand"], geo["k_local"], out_blocks=L.chosen, bitmap=L.bitmap,
                 by_block=True)


def admit_call(L, geo: dict, step: int, cold_store=None, hot: bool = True) -> None:  # noqa: ANN001
    """The device admit of L.chosen (lazykv/tiered.py:389-463: LRU victims, the misses fetched from
    the store and dequantised into their slots); with `hot`, the admitted slots go to the hot list."""
    from lazykv_b200 import kernels as K

    so = geo["sel_off"]
    K.tier_admit(L.chosen, L.block_slot, L.slot_block, L.last_used, L.evicted_at, step, L.records if cold_store is None else cold_store, L.pool,
                 L.miss_blk, L.miss_slot, L.n_miss, slots_out=L.list[:, so : so + geo["k_local"]] if hot else None)


def resident_select_call(L, geo: dict, r: int = 0) -> None:  # noqa: ANN001
    """The selection of query r for an attention before the admit (lkv_quest_topk_resident): the
    hot list gets the chosen blocks' current slots (-1 for those not resident), the bitmap only the
    resident ones, so the exact pass covers the misses from their records."""
    from lazykv_b200 import kernels as K

    so = geo["sel_off"]
    K.quest_topk_resident(L.q_ring[r], L.kmin, L.kmax, geo["cand_lo"] - geo["lo"], geo["n_cand"], geo["k_local"], L.chosen, L.block_slot,
                          L.list[:, so : so + geo["k_local"]], L.bitmap)


def attention_call(L, geo: dict, r: int = 0, cold_store=None) -> None:  # noqa: ANN001
    """Hot pass over the listed slots, cold pass over the bitmap's complement, merge: one launch."""
    from lazykv_b200 import kernels as K

    h, d = geo["h"], geo["d"]
    K.exact_attention(L.q_ring[r], L.pool, L.pool[:, :, 1], (h * 2 * BS * d, 2 * BS * d, d), L.list, BS, L.records if cold_store is None else cold_store,
                      geo["cand_lo"] - geo["lo"], geo["n_cand"], geo["scale"], BS, excluded=L.bitmap, out=L.out, lse=L.lse)


def select_admit_call(L, geo: dict, r: int, step: int, cold_store=None) -> None:  # noqa: ANN001
    """The selection of query r and its admit in one call (lkv_quest_topk_admit)."""
    from lazykv_b200 import kernels as K

    so = geo["sel_off"]
    K.quest_topk_admit(L.q_ring[r], L.kmin, L.kmax, geo["cand_lo"] - geo["lo"], geo["n_cand"], geo["k_local"], L.chosen, L.bitmap, L.block_slot,
                       L.slot_block, L.last_used, L.evicted_at, step, L.records if cold_store is None else cold_store, L.pool, L.miss_blk,
                       L.miss_slot, L.n_miss, slots_out=L.list[:, so : so + geo["k_local"]])


def layer_step(L, geo: dict, r: int = 0, step: int = 1, cold_store=None, events: list | None = None, side=None) -> None:  # noqa: ANN001
    """One layer-step of the hot path with query r. Without `side` (all launches on the current
    stream): score + top-K, then the device admit and the fetch of misses (one call), then the hot
    and cold passes and their merge in one attention launch. With a side stream: the resident
    selection, then the attention on the current stream while the admit and the fetch run on
    `side` (forked after the selection; the caller joins `side` before the layer's next step)."""
    if side is not None:
        import torch

        resident_select_call(L, geo, r)
        side.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(side):
            admit_call(L, geo, step, cold_store, hot=False)
        attention_call(L, geo, r, cold_store)
        return


    def mark() -> None:
        if events is not None:
            import torch

            e = torch.cuda.Event(enable_timing=True)
            e.record()
            events.append(e)

    mark()
    select_admit_call(L, geo, r, step, cold_store)
    mark()
    attention_call(L, geo, r, cold_store)
    mark()


LAUNCHES_PER_LAYER_STEP = 5  # the selection (TMA scoring, a cluster select per head), the admit and the fetch of misses, the attention (both passes and their merge)


def dequant_records(records, dtype, d: int = D):  # noqa: ANN001, ANN201
    """[n, h, W] int8 records -> [n, h, 2, bs, d] in `dtype`, restated in torch from the record
    layout (kq | vq | k scale | k zero | v scale | v zero; lazykv/quant.py:90-105): (code + 128) *
    scale + zero in float32, then rounded to the model dtype. Used only to check the kernels' output."""
    import torch

    n, h, _ = records.shape
    r = records.reshape(n * h, -1)
    nk = BS * d
    kq = r[:, :nk].contiguous().view(torch.int8).view(-1, BS, d).float()
    vq = r[:, nk : 2 * nk].contiguous().view(torch.int8).view(-1, BS, d).float()
    o = 2 * nk
    ks = r[:, o : o + 2 * d].contiguous().view(torch.float16).float()
    kz = r[:, o + 2 * d : o + 4 * d].contiguous().view(torch.float16).float()
    vs = r[:, o + 4 * d : o + 4 * d + 2 * BS].contiguous().view(torch.float16).float()
    vz = r[:, o + 4 * d + 2 * BS : o + 4 * d + 4 * BS].contiguous().view(torch.float16).float()
    k = (kq + 128.0) * ks[:, None, :] + kz[:, None, :]
    v = (vq + 128.0) * vs[:, :, None] + vz[:, :, None]
    return torch.stack([k, v], dim=1).to(dtype).view(n, h, 2, BS, d)


def shard_reference(L, geo: dict, r: int = 0, rows: list | None = None):  # noqa: ANN001, ANN201
    """float64 (out [rows * G, d], lse [rows * G]) of this rank's shard of one layer for query r, for
    the KV rows `rows` (all by default), from the layer's stores with torch on the device: the sink
    (exact, in the pool) on rank 0, every candidate block as its record dequantised to bf16 (what the
    hot slots and the cold pass both hold), and the current block (exact) on the last rank; softmax
    attention in float64. Independent of the kernels."""
    import torch

    h, hq, d = geo["h"], geo["hq"], geo["d"]
    g = hq // h
    rows = list(range(h)) if rows is None else list(rows)
    ri = torch.tensor(rows, device=L.records.device)
    c0 = geo["cand_lo"] - geo["lo"]
    deq = dequant_records(L.records[c0 : c0 + geo["n_cand"]].index_select(1, ri), torch.bfloat16, d)  # [n, rows, 2, bs, d]
    parts = []
    if geo["sel_off"]:
        parts.append(L.pool[0].index_select(0, ri).unsqueeze(0))
    parts.append(deq)
    if geo["has_cur"]:
        parts.append(L.pool[geo["k_local"] + 1].index_select(0, ri).unsqueeze(0))
    blocks = torch.cat(parts, dim=0).double()  # [m, rows, 2, bs, d]
    del deq, parts
    nr = len(rows)
    keys = blocks[:, :, 0].permute(1, 0, 2, 3).reshape(nr, -1, d)
    vals = blocks[:, :, 1].permute(1, 0, 2, 3).reshape(nr, -1, d)
    del blocks
    q = L.q_ring[r].view(h, g, d).index_select(0, ri).double()
    s_ = torch.einsum("hgd,htd->hgt", q, keys) * geo["scale"]
    m = s_.amax(dim=-1, keepdim=True)
    p = torch.exp(s_ - m)
    l = p.sum(dim=-1, keepdim=True)
    out = torch.einsum("hgt,htd->hgd", p / l, vals).reshape(nr * g, d)
    lse = (m + torch.log(l)).reshape(nr * g)
    return out, lse


def parity_check(got, parts: list) -> dict:  # noqa: ANN001
    """Merges the float64 shard partials [(out, lse)] and holds the bf16 output `got` to them: each
    element the bf16 rounding of a value within 2e-5 of max|ref| (|got - ref| <= 2^-8 |ref| + 2e-5
    max|ref|)."""
    import torch

    outs = torch.stack([o for o, _ in parts])
    lses = torch.stack([l for _, l in parts])
    lse = torch.logsumexp(lses, dim=0)
    ref = (torch.exp(lses - lse)[..., None] * outs).sum(0)
    g = got.double()
    err = (g - ref).abs()
    bound = 2.0**-8 * ref.abs() + 2e-5 * ref.abs().max()
    return {"layer": 0, "max_rel": float(err.max() / ref.abs().max()), "ok": bool((err <= bound).all()),
            "rule": "bf16 output within half a bf16 unit + 2e-5 max|ref| of a float64 torch restatement over the layer's stores"}


def profile_long_calls(args: argparse.Namespace) -> None:
    """The long-context layer-step's kernels at --ctx tokens (64 rows, head_dim 128, one layer),
    each twice and eagerly, for a profiler: the selection with its admit (misses, then hits), the
    bounds alone, the gathered select (one rank), the attention, and the peer-store exchange of
    one rank (its own partial only)."""
    import torch

    from lazykv_b200 import kernels as K
    from lazykv_b200.build import build
    from lazykv_b200.sharded import PeerExchange

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    build()
    shape = dict(LONG_SHAPE, ctx=args.ctx, layers=1, queries=2)
    layers, geo = build_layers(args, 0, 1, dev, shape=shape)
    L = layers[0]
    first = geo["cand_lo"] - geo["lo"]
    layer_step(L, geo, 0, 1)
    for st in range(2):
        select_admit_call(L, geo, 1, 2 + st)  # query 1's misses, then all hits
    bounds = torch.empty((geo["h"], geo["n_cand"]), dtype=torch.bfloat16, device=dev)
    for _ in range(2):
        K.quest_bounds(L.q_ring[1], L.kmin, L.kmax, first, geo["n_cand"], bounds, torch.bfloat16)
    gathered = bounds.view(1, geo["h"], geo["n_cand"])
    chosen = torch.empty((geo["h"], geo["k_local"]), dtype=torch.int32, device=dev)
    for _ in range(2):
        K.topk_gathered(gathered, [geo["n_cand"]], geo["k_total"], 0, first, chosen, L.bitmap)
    for _ in range(2):
        attention_call(L, geo, 1)
    x = PeerExchange(geo["hq"], geo["d"], device=dev)
    merged = torch.empty((geo["hq"], geo["d"]), dtype=torch.bfloat16, device=dev)
    for _ in range(2):
        x.exchange(merged)
    torch.cuda.synchronize()
    x.close()


def profile_calls(args: argparse.Namespace) -> None:
    """The kernel calls of one layer-step, each twice and eagerly, for a profiler to capture: the
    selection, the admit (the first with misses), the hot pass alone, the cold pass alone and the
    fused attention; the resident split (a third query's selection, the fused attention twice with
    its misses in the exact pass, the admit); then the codec and merge kernels at sizes above L2:
    pack and unpack of 4,096 blocks x 8 heads, block min/max over them, and an 8-part LSE merge."""
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
    r1 = 1 % geo["n_q"]
    layer_step(L, geo, 0, 1)  # residency of query 0
    for _ in range(2):
        select_call(L, geo, r1)
    for st in range(2):
        admit_call(L, geo, 2 + st)  # query 1's misses, then all hits
    for _ in range(2):
        K.hot_attention(L.q_ring[r1], L.pool, L.pool[:, :, 1], strides, L.list, BS, geo["scale"], BS, out=out, lse=lse)
    for _ in range(2):
        K.cold_attention(L.q_ring[r1], L.records, BS, first, geo["n_cand"], geo["scale"], excluded=L.bitmap, out=out, lse=lse)
    for _ in range(2):
        attention_call(L, geo, r1)
    # The bench's order (the resident split): another query's selection, the attention with its
    # misses in the exact pass, then the admit.
    r2 = 2 % geo["n_q"]
    resident_select_call(L, geo, r2)
    for _ in range(2):
        attention_call(L, geo, r2)
    admit_call(L, geo, 4, hot=False)
    torch.cuda.synchronize()
    n = 4096
    g = torch.Generator(device=dev).manual_seed(5)
    pairs = torch.randn((n, HKV, 2, BS, D), device=dev, generator=g).bfloat16()
    kmin = torch.empty((HKV, n, D), dtype=torch.bfloat16, device=dev)
    kmax = torch.empty_like(kmin)
    for _ in range(2):
        rec = K.pack_int8(pairs, kmin=kmin, kmax=kmax)
    for _ in range(2):
        K.unpack_int8(rec.view(-1, rec.shape[-1]), BS, D, torch.bfloat16)
    for _ in range(2):
        K.block_minmax(pairs[:, :, 0].transpose(0, 1), BS, kmin, kmax)
    outs = torch.randn((8, 4096, D), device=dev, generator=g)
    lses = torch.randn((8, 4096), device=dev, generator=g)
    for _ in range(2):
        K.lse_merge(outs, lses, torch.bfloat16)
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
    from lazykv_b200 import kernels as K

    K.status_attach(dev)
    layers, geo = build_layers(args, rank, world, dev)
    n_steps, n_warm = args.steps, args.warmup
    R = geo["n_q"]
    finals = [torch.empty((HQ, D), dtype=torch.bfloat16, device=dev) for _ in layers]

    admit_side = None if args.admit_first else torch.cuda.Stream()

    def token(r: int, step_no: int, cold_of=None) -> None:
        """One decode token with query r of the ring: every selecting layer's hot path (and, at N > 1,
        the exchange of the layer's partials over NVLink and their merge on every rank); the
        admits run beside the attentions on a side stream, joined at the token's end."""
        for i, L in enumerate(layers):
            layer_step(L, geo, r, step_no, None if cold_of is None else cold_of(L), side=admit_side)
            if world > 1:
                L.xchg.exchange(finals[i])
        if admit_side is not None:
            torch.cuda.current_stream().wait_stream(admit_side)

    # Warm-up: the first token admits every selected block of query 0; then the ring of queries.
    step_no = 0
    for w in range(max(n_warm, R)):
        step_no += 1
        token(w % R, step_no)
    torch.cuda.synchronize()

    # One CUDA graph per query of the ring, each a whole decode token (the exchanges are
    # captured too at N > 1; the graphs are released before the process group). A graph's admit step
    # number is fixed at capture, so the LRU clock cycles with the ring.
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        token(0, step_no + 1)
    torch.cuda.current_stream().wait_stream(side)
    torch.cuda.synchronize()
    graphs = []
    for r in range(R):
        gph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(gph):
            token(r, step_no + 1 + r)
        graphs.append(gph)
    del gph  # the graphs hold cross-rank work at N > 1: only `graphs` may keep them, so that dropping it frees them
    ring_pos = [0]

    def run() -> None:
        graphs[ring_pos[0] % R].replay()
        ring_pos[0] += 1

    for _ in range(max(n_warm, R)):
        run()
    torch.cuda.synchronize()

    def soak(fn, seconds: float) -> None:
        # About `seconds` of back-to-back replays; the count is fixed from a short calibration and
        # agreed across ranks (the graphs hold collectives at N > 1, so every rank replays alike).
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
    with Clocks(local) as clocks:
        clocks.wait_first_sample(2.0)
        soak(run, 0.5)
        ms = timed(run, n_steps)
        soak(run, 0.5)
    ms_step = ms / n_steps
    n_sel = args.layers
    us_layer = ms_step * 1e3 / n_sel
    tokens_per_s = 1e3 / ms_step

    # Per-kernel durations: each kernel group captured alone over every layer, one graph per query of
    # the ring, replayed in turn and timed with CUDA events on the replaying stream, per layer-step
    # (the local part at N > 1: no exchange). The admit is the difference between selection + admit
    # and the selection alone.
    def group_us(body) -> float:
        gs = []
        for r in range(R):
            body(r, step_no + 1 + r)
            torch.cuda.synchronize()
            gk = torch.cuda.CUDAGraph()
            with torch.cuda.graph(gk):
                body(r, step_no + 1 + r)
            gs.append(gk)
        pos = [0]

        def rep() -> None:
            gs[pos[0] % R].replay()
            pos[0] += 1

        for _ in range(R):
            rep()
        reps = max(5 * R, n_steps)
        us = timed(rep, reps) / reps * 1e3 / len(layers)  # max over ranks at N > 1
        del gs
        return us

    if args.admit_first:
        sel_us = group_us(lambda r, st: [select_call(L, geo, r) for L in layers])
        sel_admit_us = group_us(lambda r, st: [select_admit_call(L, geo, r, st) for L in layers])
    else:  # the resident selection, and the admit (with the fetch) after it on the same stream
        sel_us = group_us(lambda r, st: [resident_select_call(L, geo, r) for L in layers])
        sel_admit_us = group_us(lambda r, st: [(resident_select_call(L, geo, r), admit_call(L, geo, st, hot=False)) for L in layers])
    attn_us = group_us(lambda r, st: [attention_call(L, geo, r) for L in layers])
    kernel_us = {"select": sel_us, "admit": max(0.0, sel_admit_us - sel_us), "attention": attn_us}

    # Residency churn over the ring (eager, after the timing): the share of selected (block, head)
    # pairs already resident, and the bytes the admit's fetch moves per layer-step.
    misses = torch.zeros((), dtype=torch.int64, device=dev)
    for r in range(R):
        step_no += 1
        for L in layers:
            select_admit_call(L, geo, r, step_no)
            misses += L.n_miss.sum()
    torch.cuda.synchronize()
    miss_pairs = float(misses.item()) / (R * len(layers))
    hit_rate = 1.0 - miss_pairs / (geo["h"] * geo["k_local"])

    # Correctness of what was timed: a fresh token (query 0), layer 0's merged output against a
    # float64 restatement over every rank's shard, gathered to every rank; and the status word of the
    # kernels' bounded waits (host mirror, then the device word).
    step_no += 1
    token(0, step_no)
    torch.cuda.synchronize()
    ref_o, ref_l = shard_reference(layers[0], geo, 0)
    if world > 1:
        packed = torch.cat([ref_o, ref_l[:, None]], dim=1).contiguous()
        allp = torch.empty((world, *packed.shape), dtype=packed.dtype, device=dev)
        dist.all_gather_into_tensor(allp, packed)
        parts = [(allp[r, :, :D], allp[r, :, D]) for r in range(world)]
        got0 = finals[0]
    else:
        parts = [(ref_o, ref_l)]
        got0 = layers[0].out
    parity = parity_check(got0, parts)
    status = max(K.status_poll(clear=True), K.device_status(clear=True))
    if world > 1:
        st_t = torch.tensor([status, int(not parity["ok"])], device=dev)
        dist.all_reduce(st_t, op=dist.ReduceOp.MAX)
        status, bad = int(st_t[0].item()), int(st_t[1].item())
        parity["ok"] = parity["ok"] and not bad
    parity["device_status"] = status
    parity["ok"] = parity["ok"] and status == 0
    parity["query"] = 0
    del ref_o, ref_l, parts

    peaks = load_peaks()
    k_local = geo["k_local"]
    # The attention's blocks per head: the listed slots and the range's records. In the resident
    # split the misses are attended from their records (the fetch fills their slots beside it).
    moved = 0.0 if args.admit_first else miss_pairs / HKV
    hot_blocks = geo["n_list"] - moved
    cold_blocks = geo["n_cand"] - k_local + moved
    bytes_meta = HKV * geo["n_cand"] * D * 2 * 2
    bytes_hot = int(hot_blocks * HKV * 2 * BS * D * 2)
    rec_w = K.packed_pair_bytes(BS, D)
    bytes_cold = int(cold_blocks * HKV * rec_w)
    bytes_fetch = int(miss_pairs * (rec_w + 2 * BS * D * 2))  # a miss: its record read, its slot written
    algo = {"select": bytes_meta, "attention": bytes_hot + bytes_cold}
    dominant = max(("select", "attention"), key=lambda n: kernel_us[n])
    achieved = algo[dominant] / (kernel_us[dominant] * 1e-6) / 1e9
    layer_bytes = bytes_meta + bytes_hot + bytes_cold + bytes_fetch

    # End to end. At N = 1 through the drop-in API, as a model calls it each decode step: for every
    # layer the new token's KV goes to ExactTieredCache.update (the tier appends it; a full block is
    # sealed, packed and its metadata written), and for every selecting layer ExactTieredCache.decode
    # runs the hot path (selection, admit, exact attention) on a query copied from pinned host memory,
    # whose output is copied back to pinned host memory. At N > 1, the sharded kernels' path above,
    # eager, with the same host copies.
    if world == 1:
        e2e = run_e2e_api(args, geo, layers, dev, timed)
    else:
        q_host = torch.stack([L.q_ring for L in layers], dim=1).cpu().pin_memory()  # [R, layers, HQ, D]
        o_host = torch.empty((len(layers), HQ, D), dtype=torch.bfloat16).pin_memory()
        e_pos = [0]

        def e2e_step() -> None:
            r = e_pos[0] % R
            e_pos[0] += 1
            for i, L in enumerate(layers):
                L.q_ring[r].copy_(q_host[r, i], non_blocking=True)
                layer_step(L, geo, r, 10**9 + e_pos[0], side=admit_side)
                L.xchg.exchange(finals[i])
                o_host[i].copy_(finals[i], non_blocking=True)
            if admit_side is not None:
                torch.cuda.current_stream().wait_stream(admit_side)

        for _ in range(2):
            e2e_step()
        n_e = max(3, n_steps // 2)
        e2e_ms = timed(e2e_step, n_e) / n_e
        e2e = {"value": round(1e3 / e2e_ms, 3), "unit": "tokens/s", "h2d_bytes_per_step": n_sel * HQ * D * 2,
               "d2h_bytes_per_step": n_sel * HQ * D * 2,
               "path": "lazykv_b200.kernels (C ABI) per layer with the peer-store exchange and merge, eager, host q in / host out"}

    result = {
        "metric": METRIC,
        "value": round(tokens_per_s, 3),
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
        "data": f"synthetic (seeded N(0,1) K/V with key offsets; per layer a ring of {R} queries, base + {args.drift} x N(0,1); no weights involved)",
        "config": {"workload": "tiered decode hot path, Llama-3.2-1B attention (32q/8kv/d64), 131072-token context, bs 16, 25% budget (K=2046), 14 selecting layers, int8 cold tier in HBM, device admit with a fresh query every step"
                               + (" (admit first)" if args.admit_first else " (resident split: the admit beside the attention)"),
                   "ctx": args.ctx, "block_size": BS, "k_blocks": geo["k_total"], "selecting_layers": n_sel, "batch": 1, "queries_in_ring": R,
                   "cold_placement": "device", "l2": "inputs larger than L2 (~2.8 GB read per step)", "parallelism": f"context-sharded x{world}",
                   "timing": "one CUDA graph per decode token (select, admit, attention per layer; the exchange launch at N > 1), CUDA events, max over ranks"},
        "kernel_us": {k: round(v, 3) for k, v in kernel_us.items()},
        "residency": {"hit_rate": round(hit_rate, 4), "fetched_pairs_per_layer_step": round(miss_pairs, 1), "fetch_bytes_per_layer_step": bytes_fetch},
        "roofline": {"bound": "hbm", "kernel": dominant, "achieved": round(achieved, 1), "peak": peaks["hbm_gbs"], "unit": "GB/s",
                     "frac": round(achieved / peaks["hbm_gbs"], 4),
                     "traffic": attention_traffic() if dominant == "attention" and args.ctx == 131072 and world == 1 else None,
                     "traffic_source": "not measured by this run: dram__bytes_read.sum + dram__bytes_write.sum of one attention launch at this workload from the ncu capture committed in profiles/attn_stream_ctx128k.md (the build profiled there)",
                     "peak_source": peaks["source"],
                     "algorithmic_bytes": algo[dominant]},
        "layer_step_roofline": {"algorithmic_bytes": layer_bytes, "of_which_fetch": bytes_fetch, "us": round(us_layer, 3),
                                "achieved_gbs": round(layer_bytes / (us_layer * 1e-6) / 1e9, 1),
                                "frac": round(layer_bytes / (us_layer * 1e-6) / 1e9 / peaks["hbm_gbs"], 4)},
        "e2e": e2e,
        "gpu_launches": n_steps * n_sel * (LAUNCHES_PER_LAYER_STEP + (1 if world > 1 else 0)),  # + the exchange-and-merge kernel at N > 1
        "clocks": clocks.summary(),
        "parity": parity,
    }

    # Zero-copy leg: the same step with the cold records in pinned host memory (the admit's fetch
    # and the cold pass read them over the link).
    if world == 1 and not args.no_host_leg:
        from lazykv_b200.pinned import device_view, pinned_empty

        for L in layers:
            h = pinned_empty(tuple(L.records.shape), torch.uint8)
            h.copy_(L.records.cpu())
            L.records_host_cpu = h
            L.records_host = device_view(h)
        torch.cuda.synchronize()
        host_of = lambda L: L.records_host  # noqa: E731
        for r in range(2):
            step_no += 1
            token(r % R, step_no, host_of)
        hs = max(2, n_steps // 4)
        h_pos = [0]

        def host_token() -> None:
            h_pos[0] += 1
            token(h_pos[0] % R, step_no + h_pos[0], host_of)

        hms = timed(host_token, hs) / hs
        cold_us = []
        for L in layers[:4]:
            ev: list = []
            layer_step(L, geo, 0, step_no + 10**6, L.records_host, ev)
            torch.cuda.synchronize()
            cold_us.append(ev[1].elapsed_time(ev[2]) * 1e3)
        cu = statistics.median(cold_us)
        link = measure_link_gbs(dev)
        result["host_cold_tier"] = {"value": round(1e3 / hms, 3), "unit": "tokens/s", "us_per_layer_step": round(hms * 1e3 / n_sel, 1),
                                    "attention_us": round(cu, 1), "link_gbs": round(bytes_cold / (cu * 1e-6) / 1e9, 2),
                                    "link_peak_gbs": link, "link_peak_source": "measured by this run: pinned host -> device copy of 1 GiB, best of 5, CUDA events"}

    if not args.no_long_ctx:
        result["long_ctx"] = run_long_ctx(args, rank, world, dev, timed)
    if world == 1 and not args.no_model:
        cfg, model = random_llama(dev)
        result["model_decode"] = run_model_decode(dev, cfg, model)
        result["capacity_sweep"] = run_capacity_sweep(dev, cfg, model)
        del model
        torch.cuda.empty_cache()
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        result["cpu_baseline"] = cpu_baseline(args, budget_s=12.0)
    if rank == 0:
        print(json.dumps(result), flush=True)
    if world > 1:
        # The graphs hold cross-rank work: every reference to them (the graphs and the replay
        # closure) goes first; each rank's exchange region is released only after every rank has
        # finished its last exchange (the barrier), then the process group goes.
        import gc

        del run, graphs
        gc.collect()
        torch.cuda.synchronize()
        dist.barrier()
        for L in layers:
            L.xchg.close()
        dist.destroy_process_group()


# The long-context leg: 8 sequences of 1,048,576 tokens with Llama-3.1-8B attention shapes (32 query
# heads, 8 KV heads, head_dim 128) in 16-token blocks, 25% of each (sequence, KV head)'s blocks hot.
# The 8 sequences' KV heads are the kernels' 64 rows (rows are independent in the selection, the
# admit and the attention), their query heads the 256 query rows.
LONG_SEQS, LONG_CTX = 8, 1 << 20
LONG_SHAPE = dict(ctx=LONG_CTX, h=8 * LONG_SEQS, hq=32 * LONG_SEQS, d=128, budget=0.25, queries=4, drift=0.15, seed=4321)
LONG_MODEL_LAYERS = 32


def run_long_ctx(args: argparse.Namespace, rank: int, world: int, dev, timed) -> dict:  # noqa: ANN001
    """The long-context leg at this world size: `--long-layers` layers sharded by block range over
    the ranks, the top-K chosen globally across shards at N > 1 (every rank's bounds all-gathered,
    the same select on every rank, each admitting and attending its part), the int8 cold tier in
    HBM, a fresh query of the ring each step, the partials exchanged over NVLink and merged per layer. Each
    layer holds its own stores (about 30 GB at N = 1), so no layer-step reads another's data from
    L2. Reported per layer-step and as decode tokens/s of the 32-layer model (8 sequences per step,
    32 layer-steps each at the measured time)."""
    import torch
    import torch.distributed as dist

    from lazykv_b200 import kernels as K
    from lazykv_b200.sharded import GlobalSelection, shard_plan

    shape = dict(LONG_SHAPE, layers=args.long_layers)
    glob = world > 1
    t_build = time.perf_counter()
    layers, geo = build_layers(args, rank, world, dev, shape=shape, global_select=glob)
    build_s = time.perf_counter() - t_build
    h, hq, d = geo["h"], geo["hq"], geo["d"]
    R = geo["n_q"]
    gsel = None
    if glob:
        plans = [shard_plan(geo["n_sealed"], geo["k_total"], world, r) for r in range(world)]
        gsel = GlobalSelection(plans, rank, h, geo["k_total"], dev)
    finals = [torch.empty((hq, d), dtype=torch.bfloat16, device=dev) for _ in layers]

    def select_admit(L, r: int, step: int) -> None:  # noqa: ANN001
        """The selection then the admit, admit first (also the residency pass below)."""
        if gsel is None:
            select_admit_call(L, geo, r, step)
        else:
            gsel.select(L.q_ring[r], L.kmin, L.kmax, L.chosen, L.bitmap)
            admit_call(L, geo, step)

    so, kl = geo["sel_off"], geo["k_local"]
    admit_side = None if args.admit_first else torch.cuda.Stream()

    def layer(L, r: int, step: int) -> None:  # noqa: ANN001
        """One layer-step in the main leg's order: the resident selection (local or global), the
        attention, the admit and fetch beside it on the side stream; or admit first."""
        if admit_side is None:
            select_admit(L, r, step)
            attention_call(L, geo, r)
            return
        if gsel is None:
            resident_select_call(L, geo, r)
        else:
            gsel.select(L.q_ring[r], L.kmin, L.kmax, L.chosen, L.bitmap, block_slot=L.block_slot, hot=L.list[:, so : so + kl])
        admit_side.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(admit_side):
            admit_call(L, geo, step, hot=False)
        attention_call(L, geo, r)

    def token(r: int, step_no: int) -> None:
        for i, L in enumerate(layers):
            layer(L, r, step_no)
            if world > 1:
                L.xchg.exchange(finals[i])
        if admit_side is not None:
            torch.cuda.current_stream().wait_stream(admit_side)

    step_no = 0
    for w in range(max(args.warmup, R)):
        step_no += 1
        token(w % R, step_no)
    torch.cuda.synchronize()
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        token(0, step_no + 1)
    torch.cuda.current_stream().wait_stream(side)
    torch.cuda.synchronize()
    graphs = []
    for r in range(R):
        gph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(gph):
            token(r, step_no + 1 + r)
        graphs.append(gph)
    del gph  # the graphs hold cross-rank work at N > 1: only `graphs` may keep them, so that dropping it frees them
    pos = [0]

    def run() -> None:
        graphs[pos[0] % R].replay()
        pos[0] += 1

    for _ in range(max(args.warmup, R)):
        run()
    torch.cuda.synchronize()
    n_steps = args.long_steps
    with Clocks(dev.index) as clocks:
        clocks.wait_first_sample(2.0)
        for _ in range(2 * R):
            run()
        ms = timed(run, n_steps)
        for _ in range(2 * R):
            run()
        torch.cuda.synchronize()
    ms_step = ms / n_steps
    us_layer = ms_step * 1e3 / len(layers)

    # Per kernel group, eager, layer 0 (the device-side split of one layer-step; max over ranks).
    def ev_pair():
        return torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)

    sel_ms, att_ms = [], []
    for r in range(R):
        step_no += 1
        (a, b), (c, e) = ev_pair(), ev_pair()
        a.record()
        select_admit(layers[0], r, step_no)
        b.record()
        c.record()
        attention_call(layers[0], geo, r)
        e.record()
        e.synchronize()
        sel_ms.append(a.elapsed_time(b))
        att_ms.append(c.elapsed_time(e))
    k_us = torch.tensor([statistics.median(sel_ms) * 1e3, statistics.median(att_ms) * 1e3], device=dev)
    if world > 1:
        dist.all_reduce(k_us, op=dist.ReduceOp.MAX)

    # Residency over the ring, and how many blocks each row selected on this rank.
    misses = torch.zeros((), dtype=torch.int64, device=dev)
    chosen = torch.zeros((), dtype=torch.int64, device=dev)
    for r in range(R):
        step_no += 1
        for L in layers:
            select_admit(L, r, step_no)
            misses += L.n_miss.sum()
            chosen += (L.chosen >= 0).sum()
    # The rows' selections add up to K on every row (global), or are the local budget.
    per_row = (layers[0].chosen >= 0).sum(dim=1).to(torch.int64)
    tot = torch.stack([misses, chosen]).to(torch.float64)
    if world > 1:
        dist.all_reduce(per_row)
        dist.all_reduce(tot)
    k_ok = bool((per_row == geo["k_total"]).all()) if glob else True
    miss_pairs = float(tot[0].item()) / (R * len(layers))  # all ranks
    sel_pairs = float(tot[1].item()) / (R * len(layers))
    hit_rate = 1.0 - miss_pairs / max(1.0, sel_pairs)

    # Parity of what was timed: a fresh token with query 0, layer 0's merged output on KV rows 0 and
    # h - 1 (the first and the last sequence) against the float64 restatement over every shard.
    step_no += 1
    token(0, step_no)
    torch.cuda.synchronize()
    rows = [0, h - 1]
    g = hq // h
    qrows = torch.tensor([r * g + i for r in rows for i in range(g)], device=dev)
    ref_o, ref_l = shard_reference(layers[0], geo, 0, rows=rows)
    got = (finals[0] if world > 1 else layers[0].out).index_select(0, qrows)
    if world > 1:
        packed = torch.cat([ref_o, ref_l[:, None]], dim=1).contiguous()
        allp = torch.empty((world, *packed.shape), dtype=packed.dtype, device=dev)
        dist.all_gather_into_tensor(allp, packed)
        parts = [(allp[r, :, :d], allp[r, :, d]) for r in range(world)]
    else:
        parts = [(ref_o, ref_l)]
    parity = parity_check(got, parts)
    status = max(K.status_poll(clear=True), K.device_status(clear=True))
    flags = torch.tensor([status, int(not parity["ok"]), int(not k_ok)], device=dev)
    if world > 1:
        dist.all_reduce(flags, op=dist.ReduceOp.MAX)
    parity.update(kv_rows=rows, device_status=int(flags[0].item()), global_k_ok=not bool(flags[2].item()))
    parity["ok"] = not bool(flags[1].item()) and int(flags[0].item()) == 0 and parity["global_k_ok"]
    del ref_o, ref_l, parts

    # Algorithmic bytes of one layer-step, summed over the ranks: the metadata, the selected blocks
    # (bf16 slots) and the sink/current blocks, the other candidates' int8 records, the fetch of
    # misses. In the resident split the misses are attended from their records.
    rec_w = K.packed_pair_bytes(BS, d)
    pair_b = 2 * BS * d * 2
    n_cand_all = geo["n_sealed"] - 1
    hot_rows = sel_pairs - (0.0 if args.admit_first else miss_pairs)  # (block, row) pairs read from slots, all ranks
    bytes_layer = (h * n_cand_all * d * 2 * 2 + (hot_rows + 2 * h) * pair_b + (h * n_cand_all - hot_rows) * rec_w
                   + miss_pairs * (rec_w + pair_b))
    peaks = load_peaks()
    achieved = bytes_layer / (us_layer * 1e-6) / 1e9
    mem_gb = torch.cuda.max_memory_allocated(dev) / 1e9
    out = {
        "workload": f"{LONG_SEQS} sequences x {LONG_CTX} tokens, Llama-3.1-8B attention (32q/8kv/d128; the 8 sequences' KV heads as 64 rows), "
                    f"bs 16, 25% budget (K={geo['k_total']} blocks per row), int8 cold tier in HBM, device admit, a fresh query each step",
        "selection": "global top-K: every rank's bounds all-gathered (bf16), the same select on every rank (lkv_topk_gathered)" if glob
                     else "single GPU (lkv_quest_topk_admit)",
        "value": round(LONG_SEQS / (LONG_MODEL_LAYERS * us_layer * 1e-6), 3),
        "unit": "tokens/s",
        "value_rule": f"decode tokens/s of the {LONG_MODEL_LAYERS}-layer model: {LONG_SEQS} tokens per step, {LONG_MODEL_LAYERS} layer-steps "
                      f"at the measured layer-step time ({len(layers)} layers held and timed, each with its own stores)",
        "us_per_layer_step": round(us_layer, 2),
        "layers_timed": len(layers),
        "steps": n_steps,
        "ms_per_step_timed_layers": round(ms_step, 3),
        "kernel_us": {"select_admit": round(float(k_us[0].item()), 1), "attention": round(float(k_us[1].item()), 1)},
        "residency": {"hit_rate": round(hit_rate, 4), "fetched_pairs_per_layer_step": round(miss_pairs, 1)},
        "layer_step_roofline": {"algorithmic_bytes": int(bytes_layer), "achieved_gbs": round(achieved, 1), "peak": peaks["hbm_gbs"] * world,
                                "frac": round(achieved / (peaks["hbm_gbs"] * world), 4), "peak_rule": "measured HBM copy GB/s x GPUs"},
        "parity": parity,
        "clocks": clocks.summary(),
        "build_s": round(build_s, 1),
        "max_memory_gb_rank0": round(mem_gb, 1),
        "timing": "one CUDA graph per query of the ring (per layer the resident selection, the attention, and the admit with the fetch beside it "
                  "on a side stream, unless --admit-first; at N > 1 the NCCL all-gather of the bounds and the peer-store exchange of the "
                  "partials captured too), CUDA events over the timed steps, max over ranks; kernel_us: eager, admit first",
    }
    del graphs, run
    import gc

    gc.collect()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    return out


# The model legs: the random-init Llama-3.2-1B architecture through the drop-in API (the attention
# hook, layer-major prefill into the tier, greedy decode), as a user of the reference runs it.
LLAMA_1B = dict(hidden_size=2048, intermediate_size=8192, num_hidden_layers=16, num_attention_heads=32, num_key_value_heads=8, head_dim=64,
                vocab_size=128256, max_position_embeddings=131072, tie_word_embeddings=True, rms_norm_eps=1e-5,
                rope_parameters={"rope_type": "llama3", "rope_theta": 500000.0, "factor": 32.0, "low_freq_factor": 1.0, "high_freq_factor": 4.0,
                                 "original_max_position_embeddings": 8192})


def random_llama(dev):  # noqa: ANN001, ANN201
    """Llama-3.2-1B's architecture with seeded random weights in bf16 (no checkpoint), its attention
    routed through lazykv_b200's hook (tiered decode on the selecting layers, SDPA elsewhere)."""
    import torch
    from transformers import LlamaConfig, LlamaForCausalLM

    from lazykv_b200.attention import IMPLEMENTATION_NAME, install

    cfg = LlamaConfig(**LLAMA_1B)
    install(None, cfg.num_attention_heads, cfg.num_key_value_heads, cfg.head_dim)
    torch.manual_seed(1234)
    with torch.device(dev):
        model = LlamaForCausalLM(cfg)
    model = model.to(torch.bfloat16).eval()
    model.set_attn_implementation(IMPLEMENTATION_NAME)
    return cfg, model


def _decode_timed(model, cache, first_logits, n_new: int, warm: int = 4):  # noqa: ANN001, ANN202
    """warm + n_new greedy decode steps through the model (the loop of generate.greedy_decode); the
    time of the last n_new, from CUDA events (every step syncs on its argmax)."""
    import torch

    from lazykv_b200.generate import cache_model_kwargs

    tok = int(torch.argmax(first_logits).item())
    toks = [tok]
    ids = torch.empty((1, 1), dtype=torch.long, device=model.device)
    extra = cache_model_kwargs(cache)
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.inference_mode():
        for i in range(warm + n_new):
            if i == warm:
                a.record()
            ids.fill_(tok)
            out = model(input_ids=ids, past_key_values=cache, use_cache=True, logits_to_keep=1, **extra)
            tok = int(torch.argmax(out.logits[0, -1]).item())
            toks.append(tok)
    b.record()
    b.synchronize()
    return toks, a.elapsed_time(b)


def run_model_decode(dev, cfg, model, prompt: int = 32768, n_new: int = 128, budget: float = 0.25, chunk: int = 4096) -> dict:  # noqa: ANN001
    """The 16-layer model at a 32,768-token random prompt: layer-major prefill straight into int8
    tiers (cold blocks in pinned host memory, 25% hot), then 128 greedy decode steps through the
    hook (selection, admit, exact attention over the cold blocks and the merge on every selecting
    layer and step); beside it the same prompt and steps with every token in HBM (FullGPUCache,
    SDPA decode), and how many greedy tokens the two agree on."""
    import torch

    from lazykv_b200.cache import FullGPUCache
    from lazykv_b200.exact import ExactTieredCache
    from lazykv_b200.generate import prefill
    from lazykv_b200.selection import blocks_for_budget
    from lazykv_b200.tiered_prefill import tiered_prefill

    gen = torch.Generator(device=dev).manual_seed(99)
    ids = torch.randint(0, cfg.vocab_size, (1, prompt), device=dev, generator=gen)
    k_blocks = blocks_for_budget(budget, prompt, BS)
    cap = prompt + n_new + 128
    out = {"workload": f"Llama-3.2-1B architecture (16 layers, 32q/8kv/d64, vocab 128256), random bf16 weights, {prompt}-token random prompt, "
                       f"{n_new} greedy decode steps, int8 tiers with {int(budget * 100)}% of the blocks hot (K={k_blocks}), exact merge every step",
           "path": "lazykv_b200.tiered_prefill(cache_cls=ExactTieredCache), then greedy decode through the transformers attention hook "
                   "(4 warm-up steps, then the timed ones)"}
    for placement in ("device", "host"):
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        res = tiered_prefill(model, ids, chunk, k_blocks, BS, cap, quant="int8", cache_cls=ExactTieredCache, cold_placement=placement, fetch="gather")
        torch.cuda.synchronize()
        pre_s = time.perf_counter() - t0
        toks, ms = _decode_timed(model, res.cache, res.last_logits, n_new)
        st = res.cache.stats()
        out[f"cold_{placement}"] = {"decode_tokens_per_s": round(n_new * 1e3 / ms, 2), "prefill_s": round(pre_s, 2),
                                    "gpu_resident_kv_bytes": st.gpu_resident_kv_bytes, "host_kv_bytes": st.host_kv_bytes}
        if placement == "device":
            lazy_toks, lazy_first = toks, res.last_logits.clone()
        res.cache.close()
        del res
        torch.cuda.empty_cache()
    full = FullGPUCache(cfg.num_hidden_layers, cap)
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    pre = prefill(model, full, ids, chunk)
    torch.cuda.synchronize()
    pre_s = time.perf_counter() - t0
    toks, ms = _decode_timed(model, full, pre.last_logits, n_new)
    diverge = next((i for i, (a, b) in enumerate(zip(lazy_toks, toks)) if a != b), len(toks))
    out["full_gpu_cache"] = {"decode_tokens_per_s": round(n_new * 1e3 / ms, 2), "prefill_s": round(pre_s, 2),
                             "gpu_resident_kv_bytes": full.stats().gpu_resident_kv_bytes}
    # The prefill is exact in both (the tier is written from the same prompt KV), so the first
    # logits agree; decode then differs by the int8 rounding of the cold blocks, and a random
    # model's nearly flat logits let greedy choices part soon after.
    out["agreement_with_full_cache"] = {"prefill_logits_max_abs_diff": float((lazy_first - pre.last_logits).abs().max().item()),
                                        "first_differing_greedy_token": diverge, "tokens": len(toks)}
    del full, pre
    torch.cuda.empty_cache()
    return out


def run_capacity_sweep(dev, cfg, model, prompt: int = 130048, n_new: int = 64, budgets=(0.0625, 0.25, 0.5, 0.75), chunk: int = 4096) -> dict:  # noqa: ANN001
    """The capacity sweep: a 130,048-token random prompt prefilled layer by layer straight into int8
    tiers whose cold blocks live in pinned host memory (the full KV is never resident), then 64
    greedy decode steps with the exact merge, at each budget."""
    import torch

    from lazykv_b200.exact import ExactTieredCache
    from lazykv_b200.selection import blocks_for_budget
    from lazykv_b200.tiered_prefill import tiered_prefill

    gen = torch.Generator(device=dev).manual_seed(98)
    ids = torch.randint(0, cfg.vocab_size, (1, prompt), device=dev, generator=gen)
    cap = prompt + n_new + 128
    rows = []
    for b in budgets:
        k_blocks = blocks_for_budget(b, prompt, BS)
        torch.cuda.reset_peak_memory_stats(dev)
        base = torch.cuda.memory_allocated(dev)
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        res = tiered_prefill(model, ids, chunk, k_blocks, BS, cap, quant="int8", cache_cls=ExactTieredCache, cold_placement="host", fetch="gather")
        torch.cuda.synchronize()
        pre_s = time.perf_counter() - t0
        toks, ms = _decode_timed(model, res.cache, res.last_logits, n_new)
        st = res.cache.stats()
        rows.append({"budget": b, "k_blocks": k_blocks, "decode_tokens_per_s": round(n_new * 1e3 / ms, 2), "prefill_s": round(pre_s, 2),
                     "gpu_resident_kv_bytes": st.gpu_resident_kv_bytes, "host_kv_bytes": st.host_kv_bytes,
                     "peak_device_bytes_above_weights": int(torch.cuda.max_memory_allocated(dev) - base)})
        res.cache.close()
        del res
        torch.cuda.empty_cache()
    full_kv = cfg.num_hidden_layers * 2 * cfg.num_key_value_heads * prompt * cfg.head_dim * 2
    return {"workload": f"Llama-3.2-1B architecture, random bf16 weights, {prompt}-token random prompt prefilled layer by layer into int8 tiers "
                        f"(cold blocks in pinned host memory), {n_new} greedy decode steps with the exact merge, per budget",
            "full_kv_bytes_bf16": full_kv, "budgets": rows}


def measure_link_gbs(dev) -> float:  # noqa: ANN001
    """Host-link bandwidth of this box: a 1 GiB copy from pinned host memory to the device, best of 5."""
    import torch

    src = torch.empty(1 << 30, dtype=torch.uint8).pin_memory()
    dst = torch.empty(1 << 30, dtype=torch.uint8, device=dev)
    best = 0.0
    for _ in range(5):
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        dst.copy_(src, non_blocking=True)
        b.record()
        b.synchronize()
        best = max(best, (1 << 30) / (a.elapsed_time(b) * 1e-3) / 1e9)
    del src, dst
    return round(best, 2)


def run_e2e_api(args: argparse.Namespace, geo: dict, layers: list, dev, timed) -> dict:  # noqa: ANN001
    """End to end through the drop-in API at N = 1: an ExactTieredCache over 14 int8 tiers of a
    131,071-token prompt (seeded like the bench's layers), stepped one decode token at a time with
    the calls a model makes: update() for every layer's new KV, decode() for every selecting layer,
    with the queries from pinned host memory and the outputs copied back to it."""
    import torch

    from lazykv_b200.cache import FullGPUCache
    from lazykv_b200.exact import ExactTieredCache
    from lazykv_b200.tiered import TieredLayer

    R = geo["n_q"]
    n_sel = len(layers)
    n_e = max(3, args.steps // 2)
    prompt = args.ctx - 1  # the first decode token completes the current block: the metric geometry
    cap = args.ctx + 4 * (n_e + 8) + 64
    g = torch.Generator(device=dev).manual_seed(4321)
    tiers = {}
    for i in range(n_sel):
        off = torch.randn(1, HKV, 1, D, device=dev, generator=g) * 0.5**0.5
        keys = (torch.randn(1, HKV, prompt, D, device=dev, generator=g) + off).bfloat16()
        values = torch.randn(1, HKV, prompt, D, device=dev, generator=g).bfloat16()
        tiers[DENSE + i] = TieredLayer(keys, values, geo["k_total"], BS, cap, quant="int8", cold_placement="device")
        del keys, values
    full = FullGPUCache(DENSE + n_sel, cap)
    split = not args.admit_first  # the order of the device-timed step: the attention does not wait for the admit
    cache = ExactTieredCache(full, geo["k_total"], BS, cap, dense_layers=DENSE, quant="int8", fetch="gather", tiers=tiers, resident_split=split)
    q_host = torch.stack([L.q_ring for L in layers], dim=1).cpu().pin_memory()  # [R, layers, HQ, D]
    kv_host = torch.randn((R, DENSE + n_sel, 2, 1, HKV, 1, D), generator=torch.Generator().manual_seed(7)).bfloat16().pin_memory()
    o_host = torch.empty((n_sel, HQ, D), dtype=torch.bfloat16).pin_memory()
    q_dev = torch.empty((n_sel, HQ, D), dtype=torch.bfloat16, device=dev)
    kv_dev = torch.empty((DENSE + n_sel, 2, 1, HKV, 1, D), dtype=torch.bfloat16, device=dev)
    scale = D**-0.5
    pos = [0]

    def e2e_step() -> None:
        # One copy in of the step's queries and new KV (every layer), one copy out of the outputs.
        r = pos[0] % R
        pos[0] += 1
        kv_dev.copy_(kv_host[r], non_blocking=True)
        q_dev.copy_(q_host[r], non_blocking=True)
        outs = []
        for layer in range(DENSE + n_sel):
            cache.update(kv_dev[layer, 0], kv_dev[layer, 1], layer)
            if layer >= DENSE:
                outs.append(cache.decode(layer, q_dev[layer - DENSE].view(1, HQ, 1, D), kv_dev[layer, 0], kv_dev[layer, 1], scale))
        o_host.copy_(torch.stack(outs).view(n_sel, HQ, D), non_blocking=True)

    for _ in range(2 + R):
        e2e_step()
    e2e_ms = timed(e2e_step, n_e) / n_e
    cache.close()
    h2d = (DENSE + n_sel) * 2 * HKV * D * 2 + n_sel * HQ * D * 2
    d2h = n_sel * HQ * D * 2
    value = round(1e3 / e2e_ms, 3)
    del cache, tiers, full
    torch.cuda.empty_cache()
    return {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
            "path": "ExactTieredCache.update (every layer) + ExactTieredCache.decode (every selecting layer): the drop-in API a model's "
                    "attention hook calls, eager; each step one copy in of every layer's query and new KV from pinned host memory and one "
                    "copy out of every layer's output; int8 tier with the cold store in HBM; "
                    + ("admit first (--admit-first)" if args.admit_first else
                       "ExactTieredCache(resident_split=True): the attention before the admit, which runs beside it on a second stream, "
                       "as in the device-timed step")}


# ---------------------------------------------------------------------------------------------
# reference arm: the reference's own CPU implementation of the path, on the host cores
# ---------------------------------------------------------------------------------------------


def reference_modules():  # noqa: ANN201
    """lazykv.selection and lazykv.exact of the unmodified reference, from its install under
    baseline/_ref (pip install --target; the install travels with the repository snapshot).
    Raises ImportError when it is not installed."""
    ref = ROOT / "baseline" / "_ref"
    if not (ref / "lazykv" / "__init__.py").exists():
        raise ImportError("the reference is not installed under baseline/_ref")
    if str(ref) not in sys.path:
        sys.path.insert(0, str(ref))
    import lazykv.exact as ex
    import lazykv.selection as sel

    return sel, ex


def reference_threads() -> int:
    """Every host core for the reference's torch CPU kernels (torchrun sets OMP_NUM_THREADS=1,
    which would otherwise starve it); returns the thread count in use."""
    import torch

    torch.set_num_threads(os.cpu_count() or 1)
    return torch.get_num_threads()


def reference_inputs(ctx: int, seed: int = 7) -> dict:
    """One selecting layer as the reference's exact tier holds it: bf16 keys/values (N(0,1), keys
    with a per-(head, channel) offset of variance 0.5) mirrored in float32 ([h, T, d], contiguous per
    head, lazykv/exact.py:130-152), bf16 block min/max metadata [1, h, n, d]
    (lazykv/selection.py:142-144) and a bf16 query [1, Hq, 1, d]."""
    import torch

    g = torch.Generator().manual_seed(seed)
    off = torch.randn(HKV, 1, D, generator=g) * 0.5**0.5
    k = (torch.randn(HKV, ctx, D, generator=g) + off).bfloat16()
    v = torch.randn(HKV, ctx, D, generator=g).bfloat16()
    q = torch.randn(1, HQ, 1, D, generator=g).bfloat16()
    kb = k.view(HKV, ctx // BS, BS, D)
    return {"k": k.float().contiguous(), "v": v.float().contiguous(), "q": q, "kmin": kb.amin(2)[None].contiguous(),
            "kmax": kb.amax(2)[None].contiguous(), "nb": ctx // BS}


def reference_layer_step(sel, ex, x: dict, k_blocks: int):  # noqa: ANN001, ANN201
    """One layer-step through the reference's own functions: top_blocks over the Quest bound
    (lazykv/selection.py:38-62, indices +1 as lazykv/tiered.py:383-387), cpu_partial_attention over
    the hot set [sink, selected, current] and over every other sealed block (lazykv/exact.py:88-127),
    and merge_lse (lazykv/exact.py:69-85)."""
    nb = x["nb"]
    n_full = nb - 1
    top = sel.top_blocks(x["q"], x["kmin"][:, :, 1:n_full], x["kmax"][:, :, 1:n_full], k_blocks)[0].numpy() + 1
    hot = np.concatenate([np.zeros((HKV, 1), np.int64), top, np.full((HKV, 1), n_full, np.int64)], axis=1)
    every = np.arange(nb)
    rest = np.stack([np.setdiff1d(every, hot[j], assume_unique=True) for j in range(HKV)])
    qg = x["q"].float().view(HKV, HQ // HKV, D)
    scale = D**-0.5
    ho, hl = ex.cpu_partial_attention(x["k"], x["v"], qg, scale, BS, rest)
    co, cl = ex.cpu_partial_attention(x["k"][:, : n_full * BS], x["v"][:, : n_full * BS], qg, scale, BS, hot[:, :-1])
    return ex.merge_lse(ho, hl, co, cl)


def reference_step(sel, ex, x: dict, k_blocks: int, n_layers: int) -> float:
    """Seconds for one decode token's hot path through `n_layers` selecting layers (one layer's
    stores serve every layer: at 1.1 GB per layer the data do not stay in any CPU cache)."""
    t0 = time.perf_counter()
    for _ in range(n_layers):
        reference_layer_step(sel, ex, x, k_blocks)
    return time.perf_counter() - t0


def cpu_baseline(args: argparse.Namespace, budget_s: float = 12.0) -> dict:
    """The reference arm's measurement as a bounded sample: whole steps (all selecting layers) for
    about `budget_s` seconds."""
    from lazykv_b200.selection import blocks_for_budget

    try:
        sel, ex = reference_modules()
    except ImportError as e:
        return {"value": None, "unit": "tokens/s", "kind": "reference", "unavailable": str(e)}
    threads = reference_threads()
    x = reference_inputs(args.ctx)
    k = blocks_for_budget(args.budget, args.ctx, BS)
    reference_layer_step(sel, ex, x, k)  # warm
    times = []
    t_end = time.perf_counter() + budget_s
    while time.perf_counter() < t_end or len(times) < 2:
        times.append(reference_step(sel, ex, x, k, args.layers))
    per_step = statistics.median(times)
    return {"value": round(1.0 / per_step, 4), "unit": "tokens/s", "cores": os.cpu_count(), "threads": threads, "kind": "reference",
            "sample": f"{len(times)} decode steps of {args.layers} selecting layers at {args.ctx} tokens through the unmodified reference "
                      f"(baseline/_ref: lazykv.selection.top_blocks, lazykv.exact.cpu_partial_attention x2, merge_lse; torch CPU, "
                      f"{threads} threads); tokens/s = 1 / median step",
            "ms_per_step": round(per_step * 1e3, 1), "us_per_layer_step": round(per_step * 1e6 / args.layers, 1)}


def run_reference(args: argparse.Namespace) -> None:
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if rank != 0:
        return
    try:
        sel, ex = reference_modules()
    except ImportError as e:
        print(json.dumps({"impl": "reference", "unavailable": f"{e}"}))
        return
    from lazykv_b200.selection import blocks_for_budget

    threads = reference_threads()
    n_steps, n_warm = max(1, args.steps), max(0, args.warmup)
    x = reference_inputs(args.ctx)
    k = blocks_for_budget(args.budget, args.ctx, BS)
    t_run = time.perf_counter()
    for _ in range(n_warm):
        reference_step(sel, ex, x, k, args.layers)
    times = [reference_step(sel, ex, x, k, args.layers) for _ in range(n_steps)]
    wall = time.perf_counter() - t_run
    per_step = sum(times) / len(times)
    value = 1.0 / per_step
    sample = (f"{n_steps} decode steps, each the hot path of {args.layers} selecting layers at {args.ctx} tokens through the unmodified "
              f"reference (baseline/_ref: lazykv.selection.top_blocks, lazykv.exact.cpu_partial_attention over the hot and the cold set, "
              f"merge_lse; torch CPU, {threads} threads on {os.cpu_count()} cores); one layer's stores serve every layer")
    print(json.dumps({
        "impl": "reference", "metric": METRIC, "value": round(value, 4), "unit": "tokens/s", "n_gpus": world,
        "steps": n_steps, "warmup": n_warm, "ms_per_step": round(per_step * 1e3, 2), "us_per_layer_step": round(per_step * 1e6 / args.layers, 1),
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded N(0,1) K/V with key offsets, bf16 values in a float32 mirror)",
        "config": {"workload": "tiered decode hot path, Llama-3.2-1B attention (32q/8kv/d64), 131072-token context, bs 16, 25% budget (K=2046), "
                               "14 selecting layers, on the host cores (the reference's exact tier: bf16 values, float32 CPU mirror)",
                   "ctx": args.ctx, "k_blocks": k, "selecting_layers": args.layers},
        "cpu_baseline": {"value": round(value, 4), "unit": "tokens/s", "cores": os.cpu_count(), "threads": threads, "kind": "reference", "sample": sample},
        "e2e": {"value": round(value, 4), "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "timed_s": round(sum(times), 2), "wall_s": round(wall, 2),
    }), flush=True)


def run_ragged(args: argparse.Namespace) -> None:
    """ragged continuous batching. 64 sequences with lengths uniform in [4,096,
    131,072] (seeded), Llama-3.2-1B attention shapes, 6.25% budget, one selecting layer, the int8
    store in pinned host memory (`--ragged-cold host`, the config's zero-copy cold tier: every step
    the records the attention reads cross the host link by mapped loads into an HBM stage) or in
    HBM (`device`). A step is one decode token of every sequence through that layer (selection, the
    staging of the cold records when the store is on the host, and the exact attention, the kept
    blocks read in place from the store), timed with CUDA events; between timed steps each sequence
    appends its token and, at random, a sequence finishes and a new one of random length takes its
    slot (untimed, as a prefill would be). Prints one JSON line."""
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
    host_cold = args.ragged_cold == "host"
    tier = RaggedTier(HKV, HQ // HKV, D, BS, max_seqs=n_seqs, max_tokens=max_tokens, store_blocks=store, budget=budget, device=dev,
                      cold_placement=args.ragged_cold)
    link_peak = measure_link_gbs(dev) if host_cold else None

    def new_seq() -> int:
        n = int(rng.integers(lo, hi + 1))
        off = torch.randn((HKV, 1, D), generator=gen, device=dev) * 0.5 ** 0.5
        keys = (torch.randn((HKV, n, D), generator=gen, device=dev) + off).bfloat16()
        values = torch.randn((HKV, n, D), generator=gen, device=dev).bfloat16()
        return tier.add(keys, values)

    ids = [new_seq() for _ in range(n_seqs)]
    scale = D ** -0.5
    times, toks, nbytes, lbytes = [], [], [], []
    with Clocks(0) as clocks:
        for step in range(steps):
            ids.sort()
            q = torch.randn((len(ids) * HQ, D), generator=gen, device=dev).bfloat16()
            # algorithmic bytes of the step: every candidate's bounds and record (kept blocks are
            # attended in place from the store), the sink and the current block
            b = lb = 0
            for s in ids:
                nc = tier.seqs[s].n_sealed - 1
                b += HKV * (nc * (2 * D * 2 + tier.W) + 2 * 2 * BS * D * 2)
                lb += HKV * nc * tier.W  # host store: every candidate's record crosses the link once
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
                lbytes.append(lb)
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
    if host_cold:
        link = sum(lbytes) / total_s / 1e9
        roofline = {"bound": "host-link", "achieved": round(link, 2), "peak": link_peak, "unit": "GB/s", "frac": round(link / link_peak, 4),
                    "traffic": None, "peak_source": "measured by this run: pinned host -> device copy of 1 GiB, best of 5, CUDA events",
                    "link_bytes_per_step": int(statistics.mean(lbytes)), "hbm_achieved_gbs": round(achieved, 1),
                    "algorithmic_bytes_per_step": int(statistics.mean(nbytes))}
        store_desc = "int8 store in pinned host memory, records staged in HBM over the link each step (zero-copy mapped loads)"
    else:
        roofline = {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s", "frac": round(achieved / peak, 4),
                    "traffic": None, "peak_source": peak_src, "algorithmic_bytes_per_step": int(statistics.mean(nbytes))}
        store_desc = "int8 store in HBM"
    print(json.dumps({
        "metric": "ragged decode tokens/s per selecting layer (config 3: 64 sequences, ctx U[4096, 131072], 6.25% budget)",
        "value": round(value, 1), "unit": "tokens/s", "n_gpus": 1, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(1e3 * total_s / len(times), 4), "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "bf16", "data": "synthetic (seeded N(0,1) K/V with per-head key offsets, random queries)",
        "config": {"workload": "ragged continuous batching, Llama-3.2-1B attention (32q/8kv/d64), 64 sequences, lengths U[4096, 131072], "
                               f"bs 16, 6.25% budget, {store_desc} (kept blocks attended in place), one selecting layer",
                   "l2": "inputs larger than L2 (~GBs per step)", "timing": "CUDA events around each decode step (host-built schedule included)"},
        "roofline": roofline,
        "gpu_launches": (4 if host_cold else 3) * len(times),
        "clocks": clocks.summary(),
    }))


def main() -> None:
    args = parse()
    if args.impl == "reference":
        run_reference(args)
    elif args.workload == "ragged":
        run_ragged(args)
    elif args.profile_calls:
        profile_long_calls(args) if args.profile_long else profile_calls(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
