"""The bench's own launches at the metric geometry, against the oracle.

One selecting layer exactly as `bench.py` builds and runs it (131,072 tokens, 16-token blocks, 8 KV
heads, G = 4, d = 64, 25% budget: K = 2,046 of 8,190 candidates, the int8 cold tier in HBM): the
TMA-scored selection in block order, the device admit that fetches the selected blocks into the slot
pool (dequantised from their records), then the fused attention (hot pass over the listed slots,
cold pass over the complement of the bitmap and their merge in one launch, 18 CTAs per head with
their per-CTA lists, rings and fold at full size).
The same seeded layer goes through `oracle.tiered_decode` (float64 attention over the reference's
pieces: `unpack(pack(block))` in bf16 for the sealed blocks, the exact sink and current block),
which makes its own selection. Held:
  * int8 records and block metadata byte/bit-exact with the oracle's `pack` and min/max;
  * the Quest bounds bit-exact and the selected set equal to the oracle's top-K (ties to the lower ids);
  * every selected block in a slot of the pool, holding its record dequantised to bf16;
  * the float32 merged output within 1e-5 of max|out| (and lse within 1e-5), the bf16 output the
    bf16 rounding of a value within 2e-5 of the oracle (at most half a bf16 unit plus 2e-5 of the max).
"""

from __future__ import annotations

import argparse

import numpy as np
import pytest
import torch

import oracle as O
from tests.parity import bf16_close

pytestmark = pytest.mark.gpu

CTX, HQ, HKV, D, BS = 131072, 32, 8, 64, 16


@pytest.fixture(scope="module")
def metric_layer():
    import bench
    from lazykv_b200 import kernels as K

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    args = argparse.Namespace(ctx=CTX, budget=0.25, layers=1, queries=1, drift=0.5)
    layers, geo = bench.build_layers(args, 0, 1, dev, keep_source=True)
    L = layers[0]
    assert geo["n_cand"] == 8190 and geo["k_local"] == 2046 and geo["n_list"] == 2048
    # Bounds of the same call (the bench's call does not ask for them): the selection's own output.
    bound = torch.empty((HKV, geo["n_cand"]), dtype=torch.float32, device=dev)
    sel = torch.empty((HKV, geo["k_local"]), dtype=torch.int32, device=dev)
    K.quest_topk(L.q, L.kmin, L.kmax, 1, geo["n_cand"], geo["k_local"], out_blocks=sel, want_bound=False, by_block=True)
    _, bound = K.quest_topk(L.q, L.kmin, L.kmax, 1, geo["n_cand"], geo["k_local"], want_bound=True, by_block=True)
    # The bench's layer-step, twice (the second call sees what the first left in the workspaces).
    for _ in range(2):
        bench.layer_step(L, geo)
    out_bf16 = L.out.clone()
    out32 = torch.empty((HQ, D), dtype=torch.float32, device=dev)
    lse32 = torch.empty((HQ,), dtype=torch.float32, device=dev)
    K.exact_attention(L.q, L.pool, L.pool[:, :, 1], (HKV * 2 * BS * D, 2 * BS * D, D), L.list, BS, L.records, 1, geo["n_cand"],
                      geo["scale"], BS, excluded=L.bitmap, out_dtype=torch.float32, out=out32, lse=lse32)
    torch.cuda.synchronize()
    status = K.device_status(clear=True)
    got = {
        "records": L.records.cpu().numpy(),
        "kmin": L.kmin.float().cpu().numpy(),
        "kmax": L.kmax.float().cpu().numpy(),
        "bound": bound.cpu().numpy(),
        "list": L.list.cpu().numpy(),
        "chosen": L.chosen.cpu().numpy(),
        "sel_call": sel.cpu().numpy(),
        "pool": L.pool.cpu(),
        "deq": K.unpack_int8(L.records.view(-1, L.records.shape[-1]), BS, D, torch.bfloat16).view(L.records.shape[0], HKV, 2, BS, D).cpu(),
        "bitmap": L.bitmap.cpu().numpy(),
        "out_bf16": out_bf16.float().cpu().numpy(),
        "out32": out32.cpu().numpy(),
        "lse32": lse32.cpu().numpy(),
        "status": status,
    }
    want = O.tiered_decode(L.q.float().cpu().numpy(), L.kv.float().cpu().numpy(), L.cur.float().cpu().numpy(), BS, geo["k_local"],
                           geo["scale"], "bfloat16", "int8")
    return got, want, geo


def test_records_and_metadata_are_bit_exact_at_full_size(metric_layer) -> None:  # noqa: ANN001
    got, want, _ = metric_layer
    assert np.array_equal(got["records"], want["records"])
    # The candidates' metadata (blocks 1..8190), taken over the dequantised keys. Block 0, the sink,
    # is never a candidate: the oracle takes its min/max over the exact keys it keeps, the pack over
    # its dequantised record, and neither is read.
    n = want["kmin"].shape[1]
    assert np.array_equal(got["kmin"][:, 1:n], want["kmin"][:, 1:])
    assert np.array_equal(got["kmax"][:, 1:n], want["kmax"][:, 1:])


def test_bounds_bit_exact_and_the_selected_set_is_the_oracles(metric_layer) -> None:  # noqa: ANN001
    got, want, geo = metric_layer
    assert np.array_equal(got["bound"], want["bound"].astype(np.float32))
    k = geo["k_local"]
    want_sel = np.sort(want["selected"], axis=1)
    assert np.array_equal(got["chosen"], want_sel)
    assert np.array_equal(got["sel_call"], want_sel)
    # hot list: the sink's slot, the admitted slots, the current block's slot
    assert (got["list"][:, 0] == 0).all() and (got["list"][:, -1] == k + 1).all()
    bits = np.unpackbits(got["bitmap"].view(np.uint8), bitorder="little").reshape(HKV, -1)
    for j in range(HKV):
        assert np.array_equal(np.nonzero(bits[j])[0], want_sel[j])


def test_the_admit_put_every_selected_block_in_a_slot(metric_layer) -> None:  # noqa: ANN001
    got, _, geo = metric_layer
    k = geo["k_local"]
    slots = got["list"][:, 1 : 1 + k]
    for j in range(HKV):
        assert sorted(slots[j].tolist()) == list(range(1, k + 1))  # every slot holds one selected block
        for s_, b in zip(slots[j].tolist(), got["chosen"][j].tolist()):
            assert torch.equal(got["pool"][s_, j], got["deq"][b, j]), (j, s_, b)


def test_fused_attention_matches_the_oracle_at_full_size(metric_layer) -> None:  # noqa: ANN001
    got, want, _ = metric_layer
    ref = want["out"].reshape(HQ, D)
    err = np.abs(got["out32"].astype(np.float64) - ref).max() / np.abs(ref).max()
    assert err < 1e-5, err
    assert np.abs(got["lse32"].astype(np.float64) - want["lse"].reshape(HQ)).max() < 1e-5
    assert bf16_close(got["out_bf16"], ref)
    assert got["status"] == 0
