"""Record and replay of the selection, the reference's tests/test_tiered_int8.py:232-290 and
tests/test_trace.py:105-130 on the device tier: a recorded run replayed through
`replay_selection` repeats its fetches and outputs bit for bit (also with the device stalled, so
the host runs ahead of the queued copies), and the reference's LRU rule run on the host over the
recorded selection fetches exactly what the device admit fetched, step by step."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from tests.parity import lru_admit
from tests.tiny_model import BS, CAP, K, PROMPT, forced, make_tiny, prefilled

pytestmark = pytest.mark.gpu
STEPS = 30  # forced positions; the first comes from the prefill, so 29 decode steps cross several seals
FWD = STEPS - 1


@pytest.fixture(scope="module")
def tiny():  # noqa: ANN201
    return make_tiny()


def _cache(full, kind: str, **kw):  # noqa: ANN001, ANN202
    from lazykv_b200.exact import ExactTieredCache
    from lazykv_b200.tiered import TieredCache

    if kind == "bf16":
        return TieredCache(full, K, BS, capacity_tokens=CAP, dense_layers=1, fetch="gather", **kw)
    if kind == "int8":
        return TieredCache(full, K, BS, capacity_tokens=CAP, dense_layers=1, fetch="gather", quant="int8", **kw)
    return ExactTieredCache(full, K, BS, capacity_tokens=CAP, dense_layers=1, fetch="gather", quant="int8", resident_split=kind == "exact_split", **kw)


@pytest.mark.parametrize("kind", ["bf16", "int8", "exact", "exact_split"])
@pytest.mark.parametrize("stall", [False, True])
def test_replaying_a_recorded_selection_reproduces_the_run_exactly(tiny, kind: str, stall: bool) -> None:  # noqa: ANN001
    cfg, model = tiny
    ids, full, pre = prefilled(model, cfg)
    rec = _cache(full, kind, record_selection=True)
    ref = forced(model, rec, pre, ids, STEPS)
    rec.close()
    selection = rec.recorded_selection()
    rec_counts = rec.counters_dict()
    full.truncate(PROMPT)
    assert len(selection) == FWD * len(rec.tiers)
    for (layer, step), ch in selection.items():
        assert ch.dtype == np.int64 and ch.shape == (cfg.num_key_value_heads, K)
        assert (np.diff(ch, axis=1) > 0).all(), "decode records ascending ids"
        assert layer in rec.tiers and 1 <= step <= FWD

    rep = _cache(full, kind, replay_selection=selection)
    if stall:
        torch.cuda._sleep(200_000_000)  # every copy below queues behind this: the host runs ahead
    got = forced(model, rep, pre, ids, STEPS)
    rep.close()
    rep_counts = rep.counters_dict()
    full.truncate(PROMPT)
    assert torch.equal(got, ref)
    assert rep_counts["fetched_pairs"] == rec_counts["fetched_pairs"] > 0
    assert rep_counts["fetched_pairs_per_step"] == rec_counts["fetched_pairs_per_step"]


def test_a_replayed_foreign_selection_is_what_gets_attended(tiny) -> None:  # noqa: ANN001
    """Replaying a selection the tier would not make (the lowest K candidates every step) changes
    the output, and recording that replay gives the replayed ids back."""
    cfg, model = tiny
    ids, full, pre = prefilled(model, cfg)
    base = _cache(full, "bf16")
    ref = forced(model, base, pre, ids, 8)
    base.close()
    full.truncate(PROMPT)
    h = cfg.num_key_value_heads
    lowest = np.tile(np.arange(1, K + 1, dtype=np.int64), (h, 1))
    foreign = {(layer, s): lowest for layer in base.tiers for s in range(1, 8)}  # 8 positions: 7 decode steps
    rep = _cache(full, "bf16", replay_selection=foreign, record_selection=True)
    got = forced(model, rep, pre, ids, 8)
    again = rep.recorded_selection()
    rep.close()
    full.truncate(PROMPT)
    assert not torch.equal(got, ref)
    assert all(np.array_equal(again[key], lowest) for key in foreign)


def test_simulated_lru_fetches_exactly_what_the_tier_fetched(tiny) -> None:  # noqa: ANN001
    """The reference's LRU rule, run on the host over the recorded selection from the tier's
    initial tables, gives the per-step fetch counts the device admit produced."""
    cfg, model = tiny
    ids, full, pre = prefilled(model, cfg)
    tier = _cache(full, "bf16", n_slots=K + 3, record_selection=True)
    tables = {i: [t.block_slot.copy(), t.slot_block.copy(), t.last_used.copy(), t.evicted_at.copy()] for i, t in tier.tiers.items()}
    forced(model, tier, pre, ids, STEPS)
    tier.close()
    per_step = tier.counters_dict()["fetched_pairs_per_step"]
    rec = tier.recorded_selection()
    full.truncate(PROMPT)
    steps = sorted({s for _, s in rec})
    assert steps == list(range(1, FWD + 1))
    sim = np.zeros(len(steps), dtype=np.int64)
    for layer, (block_slot, slot_block, last_used, evicted_at) in tables.items():
        for i, s in enumerate(steps):
            sim[i] += sum(len(m) for m in lru_admit(rec[(layer, s)], block_slot, slot_block, last_used, evicted_at, s))
    assert sim.sum() > 0
    assert sim.tolist() == per_step


def test_select_protocol_records_and_replays(tiny) -> None:  # noqa: ANN001
    """select() (the gathered-set protocol) records its rank-order selection; replaying it there
    gathers the same sets after the same admits."""
    cfg, model = tiny
    ids, full, pre = prefilled(model, cfg)
    h, hq, d = cfg.num_key_value_heads, cfg.num_attention_heads, cfg.head_dim
    gen = torch.Generator(device="cuda").manual_seed(5)
    queries = [torch.randn((1, hq, 1, d), generator=gen, device="cuda").bfloat16() for _ in range(4)]
    kv = torch.zeros((1, h, 1, d), dtype=torch.bfloat16, device="cuda")

    def run(cache):  # noqa: ANN001, ANN202
        outs = []
        for step, q in enumerate(queries, start=1):
            cache._step = step
            outs.append([t.clone() for t in cache.select(1, q, kv, kv)])
        return outs

    rec = _cache(full, "bf16", record_selection=True)
    want = run(rec)
    selection = rec.recorded_selection()
    rep = _cache(full, "bf16", replay_selection=selection)
    got = run(rep)
    for a, b in zip(want, got):
        for x, y in zip(a, b):
            assert torch.equal(x, y)
    assert sorted(selection) == [(1, s) for s in range(1, 5)]


def test_bad_replays_and_reads_are_refused(tiny) -> None:  # noqa: ANN001
    cfg, model = tiny
    ids, full, pre = prefilled(model, cfg)
    plain = _cache(full, "bf16")
    with pytest.raises(RuntimeError, match="record_selection=True"):
        plain.recorded_selection()
    layer = plain.tiers[1]
    h = cfg.num_key_value_heads
    n_full, _ = layer.candidates()
    with pytest.raises(ValueError, match="block ids, got"):
        layer.load_chosen(np.ones((h, K + 1), dtype=np.int64))
    with pytest.raises(ValueError, match="must lie in"):
        layer.load_chosen(np.full((h, K), n_full, dtype=np.int64))
    with pytest.raises(ValueError, match="must lie in"):
        layer.load_chosen(np.zeros((h, K), dtype=np.int64))  # the sink is not a candidate
    with pytest.raises(ValueError, match="distinct"):
        layer.load_chosen(np.ones((h, K), dtype=np.int64))
    missing = _cache(full, "bf16", replay_selection={})
    with pytest.raises(KeyError):
        forced(model, missing, pre, ids, 2)  # one decode step
    missing.close()
    plain.close()
    full.truncate(PROMPT)


@pytest.mark.parametrize("h,k,words", [(1, 1, 1), (8, 2046, 256), (5, 37, 3)])
def test_mark_blocks_sets_exactly_the_listed_bits(h: int, k: int, words: int) -> None:
    from lazykv_b200 import kernels as K_

    rng = np.random.default_rng(h * 1000 + k)
    ids = np.full((h, k + 3), -1, dtype=np.int32)
    for j in range(h):
        n = min(k, words * 32)
        ids[j, :n] = rng.choice(words * 32, size=n, replace=False)
    ids[0, 0] = words * 32 + 5  # past the bitmap: skipped
    dev_ids = torch.from_numpy(ids).cuda()[:, :k]  # row stride k + 3
    bm = torch.full((h, words), -1, dtype=torch.int32, device="cuda")
    K_.mark_blocks(dev_ids, bm)
    want = np.zeros((h, words * 32), dtype=np.uint8)
    for j in range(h):
        row = ids[j, :k]
        row = row[(row >= 0) & (row < words * 32)]
        want[j, row] = 1
    got = np.unpackbits(bm.cpu().numpy().view(np.uint8), bitorder="little").reshape(h, -1)
    assert np.array_equal(got, want)
