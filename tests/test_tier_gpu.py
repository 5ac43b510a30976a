"""The bf16 tier (TieredCache) on the tiny model: the reference's tier tests (tests/test_tiered.py),
through the device hot path. The tier may move bytes, never change them: same selection, same
block order, same kernel as QuestView over the full cache, so the same log-probs bit for bit."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from tests.tiny_model import BS, CAP, K, PROMPT, check_residency, forced, make_tiny, prefilled

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def tiny():  # noqa: ANN201
    return make_tiny()


@pytest.mark.parametrize("prefetch", [False, True])
@pytest.mark.parametrize(("fetch", "spare"), [("runs", 0), ("gather", 0), ("gather", 2)])
def test_tier_is_bit_identical_to_questview(tiny, fetch: str, spare: int, prefetch: bool) -> None:  # noqa: ANN001
    """tests/test_tiered.py:58: residency moves blocks into slots; the attention reads the same bytes
    (with the layer-ahead prefetch too: it changes where blocks sit and when they arrive, not what
    is attended)."""
    from lazykv_b200.selection import QuestView
    from lazykv_b200.tiered import TieredCache

    cfg, model = tiny
    ids, full, pre = prefilled(model, cfg)
    quest = QuestView(full, k_blocks=K, block_size=BS, dense_layers=1)
    ref = forced(model, quest, pre, ids, 40)  # crosses several seals
    assert quest.counters.selections > 0
    full.truncate(PROMPT)
    tier = TieredCache(full, K, BS, capacity_tokens=CAP, model=model, dense_layers=1, n_slots=K + spare, fetch=fetch, prefetch=prefetch)
    got = forced(model, tier, pre, ids, 40)
    tier.close()
    assert torch.equal(got, ref)
    c = tier.counters_dict()
    if prefetch:
        assert c["prefetched_pairs"] > 0 and 0 <= c["prefetch_used_pairs"] <= c["prefetched_pairs"]
        assert c["prefetch_transfers"] == c["selections"]  # every selecting layer step (layer 1's from the hook on layer 0)
        assert tier.policy_name == "tiered_prefetch"
    assert c["selections"] == quest.counters.selections
    assert c["seals"] == ((PROMPT + 39) // BS - PROMPT // BS) * 3  # 3 tiered layers
    assert c["hit_pairs"] + c["fetched_pairs"] == c["selected_pairs"]
    assert c["fetched_pairs"] > 0  # the recency seed cannot be right for a random model
    assert sum(c["fetched_pairs_per_step"]) == c["fetched_pairs"]
    check_residency(tier)


def test_zerocopy_tier_matches_questview(tiny) -> None:  # noqa: ANN001
    """tests/test_tiered.py:190, with one difference: the selected blocks are read in place from
    the pinned store and the sink + current block from VRAM, as two partials merged by their
    log-sum-exp, so the bar is float32 merge rounding, not bit identity."""
    from lazykv_b200.selection import QuestView
    from lazykv_b200.tiered import TieredCache

    cfg, model = tiny
    ids, full, pre = prefilled(model, cfg)
    quest = QuestView(full, k_blocks=K, block_size=BS, dense_layers=1)
    ref = forced(model, quest, pre, ids, 40)
    full.truncate(PROMPT)
    tier = TieredCache(full, K, BS, capacity_tokens=CAP, model=model, dense_layers=1, fetch="zerocopy")
    got = forced(model, tier, pre, ids, 40)
    tier.close()
    assert (got - ref).abs().max().item() < 0.02
    c = tier.counters_dict()
    assert c["selections"] == quest.counters.selections
    assert c["fetched_pairs"] == 0 and c["hit_pairs"] == 0
    assert c["zerocopy_bytes"] == c["selected_pairs"] * next(iter(tier.tiers.values())).pair_bytes > 0
    for t in tier.tiers.values():
        assert t.n_slots == 0 and t.pool.shape[0] == 2  # VRAM: the sink and the current block


def test_seal_writes_the_exact_block_to_host(tiny) -> None:  # noqa: ANN001
    """tests/test_tiered.py:93: host rows and metadata equal what QuestView appends to the full cache."""
    from lazykv_b200.selection import QuestView
    from lazykv_b200.tiered import TieredCache

    cfg, model = tiny
    ids, full, pre = prefilled(model, cfg)
    tier = TieredCache(full, K, BS, capacity_tokens=CAP, dense_layers=1)
    forced(model, tier, pre, ids, 30)
    tier.close()
    torch.cuda.synchronize()
    full.truncate(PROMPT)
    forced(model, QuestView(full, K, BS, dense_layers=1), pre, ids, 30)
    for i, t in tier.tiers.items():
        layer = full.layers[i]
        assert t.n_sealed == (PROMPT + 29) // BS
        for b in range(t.n_sealed):
            got = t.host[b, :, 0]
            assert torch.equal(got, layer.keys[0, :, b * BS : (b + 1) * BS].cpu())
            assert torch.equal(t.host[b, :, 1], layer.values[0, :, b * BS : (b + 1) * BS].cpu())
            assert torch.equal(t.kmin[0, :, b].cpu(), got.amin(dim=1)) and torch.equal(t.kmax[0, :, b].cpu(), got.amax(dim=1))


def test_admit_coalesces_runs_and_evicts_outside_the_selection(tiny) -> None:  # noqa: ANN001
    """tests/test_tiered.py:119, on the device admit."""
    from lazykv_b200.tiered import TierCounters, TieredCache

    cfg, model = tiny
    _, full, _ = prefilled(model, cfg)
    cache = TieredCache(full, K, BS, capacity_tokens=CAP, dense_layers=1)
    tier = cache.tiers[1]
    assert (tier.slot_block == np.array([9, 10, 11])).all()  # recency seed: blocks 9..11 in slots 1..3
    chosen = np.array([[2, 3, 11], [2, 3, 11]])
    mh, mb, transfers = tier.admit(chosen, step=1, counters=TierCounters(), stream=None)
    assert sorted(zip(mh.tolist(), mb.tolist())) == [(0, 2), (0, 3), (1, 2), (1, 3)]
    assert transfers == 1  # one fetch launch for the step
    bsl, ev = tier.block_slot, tier.evicted_at
    assert bsl[0, 11] == 3 and bsl[0, 9] == -1 and ev[1, 10] == 1
    assert (bsl[:, 2] == 1).all() and (bsl[:, 3] == 2).all()  # victims: the least recent slots, lowest first
    check_residency(cache)
    cache.close()


def test_spare_slots_evict_least_recently_used_and_fill_empty_slots_first(tiny) -> None:  # noqa: ANN001
    """tests/test_tiered.py:164, with the tables edited through set_tables (they live on the device)."""
    from lazykv_b200.tiered import TierCounters, TieredCache

    cfg, model = tiny
    _, full, _ = prefilled(model, cfg, n=40)  # 5 blocks: 4 candidates, seeded into 4 of 6 slots
    cache = TieredCache(full, 2, BS, capacity_tokens=CAP, dense_layers=1, n_slots=6)
    tier = cache.tiers[1]
    assert (tier.slot_block[:, :4] == np.array([1, 2, 3, 4])).all() and (tier.slot_block[:, 4:] == -1).all()
    counters = TierCounters()
    assert tier.admit(np.array([[1, 4], [2, 3]]), step=1, counters=counters)[0].size == 0  # all resident
    lu, bsl, sb = tier.last_used, tier.block_slot, tier.slot_block
    lu[:, :4] = [[5, 1, 7, 3], [5, 1, 7, 3]]
    bsl[:, 4] = -1  # pretend block 4 was evicted, so it must be fetched again
    sb[:, 3] = -1
    lu[:, 3] = -2
    tier.set_tables(slot_block=sb, block_slot=bsl, last_used=lu)
    mh, mb, _ = tier.admit(np.array([[4, 1], [4, 1]]), step=9, counters=counters)
    assert sorted(mb.tolist()) == [4, 4]
    assert (tier.block_slot[:, 4] == 4).all()  # the empty slot (pool index 4) before any occupied one
    assert (tier.last_used[:, 3] == 9).all() and (tier.last_used[:, 0] == 9).all()
    check_residency(cache)
    cache.close()


def test_lru_victim_is_the_least_recently_used_occupied_slot(tiny) -> None:  # noqa: ANN001
    """With no empty slot, the victim is the occupied slot used longest ago, outside the selection."""
    from lazykv_b200.tiered import TierCounters, TieredCache

    cfg, model = tiny
    _, full, _ = prefilled(model, cfg)
    cache = TieredCache(full, K, BS, capacity_tokens=CAP, dense_layers=1, n_slots=K + 1)
    tier = cache.tiers[1]
    sb = tier.slot_block
    assert (sb == np.array([8, 9, 10, 11])).all()
    tier.set_tables(last_used=np.array([[4, 2, 6, 3], [1, 5, 2, 7]]))
    mh, mb, _ = tier.admit(np.array([[1, 10, 11], [1, 9, 11]]), step=8, counters=TierCounters())
    # head 0: free slots (not selected) are 0 (lu 4) and 1 (lu 2) -> slot 1; head 1: slots 0 (lu 1), 2 (lu 2) -> slot 0
    assert mh.tolist() == [0, 1] and mb.tolist() == [1, 1]
    bsl = tier.block_slot
    assert bsl[0, 1] == 2 and bsl[1, 1] == 1
    assert tier.evicted_at[0, 9] == 8 and tier.evicted_at[1, 8] == 8
    check_residency(cache)
    cache.close()


def test_budget_that_covers_every_block_is_refused(tiny) -> None:  # noqa: ANN001
    from lazykv_b200.tiered import TieredCache

    cfg, model = tiny
    _, full, _ = prefilled(model, cfg)
    with pytest.raises(ValueError, match="needs selection"):
        TieredCache(full, 11, BS, capacity_tokens=CAP, dense_layers=1)


def test_refusals(tiny) -> None:  # noqa: ANN001
    """Zero-copy has no residency to prefetch, record or replay: refused loudly."""
    from lazykv_b200.tiered import TieredCache

    cfg, model = tiny
    _, full, _ = prefilled(model, cfg)
    with pytest.raises(ValueError, match="zero-copy"):
        TieredCache(full, K, BS, capacity_tokens=CAP, model=model, dense_layers=1, fetch="zerocopy", prefetch=True)
    with pytest.raises(ValueError, match="zero-copy"):
        TieredCache(full, K, BS, capacity_tokens=CAP, dense_layers=1, fetch="zerocopy", record_selection=True)
    with pytest.raises(ValueError, match="zero-copy"):
        TieredCache(full, K, BS, capacity_tokens=CAP, dense_layers=1, fetch="zerocopy", replay_selection={})


def test_device_cold_placement_is_bit_identical(tiny) -> None:  # noqa: ANN001
    """A device copy of the store (cold_placement='device') feeds the same fetches: same log-probs."""
    from lazykv_b200.tiered import TieredCache

    cfg, model = tiny
    ids, full, pre = prefilled(model, cfg)
    host = TieredCache(full, K, BS, capacity_tokens=CAP, dense_layers=1, fetch="gather")
    a = forced(model, host, pre, ids, 24)
    host.close()
    full.truncate(PROMPT)
    dev = TieredCache(full, K, BS, capacity_tokens=CAP, dense_layers=1, fetch="gather", cold_placement="device")
    b = forced(model, dev, pre, ids, 24)
    dev.close()
    assert torch.equal(a, b)
    for t in dev.tiers.values():
        assert torch.equal(t.dev_store[: t.n_sealed].cpu(), t.host[: t.n_sealed])


def test_select_protocol_matches_decode(tiny) -> None:  # noqa: ANN001
    """The reference's select/attend protocol (gather in rank order, SDPA) against the fused decode."""
    from lazykv_b200.tiered import TieredCache

    cfg, model = tiny
    ids, full, pre = prefilled(model, cfg)
    fused = TieredCache(full, K, BS, capacity_tokens=CAP, dense_layers=1)
    a = forced(model, fused, pre, ids, 24)
    fused.close()
    full.truncate(PROMPT)
    proto = TieredCache(full, K, BS, capacity_tokens=CAP, dense_layers=1)
    proto.decode = lambda *args, **kw: None  # type: ignore[method-assign]
    b = forced(model, proto, pre, ids, 24)
    proto.close()
    assert (a - b).abs().max().item() < 0.02
    check_residency(proto)


def test_close_removes_prefetch_hooks(tiny) -> None:  # noqa: ANN001
    """tests/test_tiered.py:141: one pre-hook per selecting layer after the first, removed by close()."""
    from lazykv_b200.tiered import TieredCache

    cfg, model = tiny
    _, full, _ = prefilled(model, cfg)
    before = [len(layer._forward_pre_hooks) for layer in model.model.layers]
    cache = TieredCache(full, K, BS, capacity_tokens=CAP, model=model, prefetch=True, dense_layers=1)
    assert sum(len(layer._forward_pre_hooks) for layer in model.model.layers) == sum(before) + 3
    cache.close()
    assert [len(layer._forward_pre_hooks) for layer in model.model.layers] == before


@pytest.mark.parametrize("quant", [None, "int8"])
def test_prefetch_leaves_the_decode_unchanged_and_measures_its_overlap(tiny, quant: str | None) -> None:  # noqa: ANN001
    """The same log-probs with and without the prefetch (bf16 and int8 tiers, a pool of K + 3 slots
    so that prefetched blocks can stay resident); with instrument=True, overlap() reports one timed
    prefetch per prefetching layer step, each fraction in [0, 1]."""
    from lazykv_b200.tiered import TieredCache

    cfg, model = tiny
    ids, full, pre = prefilled(model, cfg)
    kw = {"fetch": "gather", "quant": quant, "n_slots": K + 3}
    base = TieredCache(full, K, BS, capacity_tokens=CAP, model=model, dense_layers=1, **kw)
    ref = forced(model, base, pre, ids, 30)
    base.close()
    full.truncate(PROMPT)
    pf = TieredCache(full, K, BS, capacity_tokens=CAP, model=model, dense_layers=1, prefetch=True, instrument=True, **kw)
    got = forced(model, pf, pre, ids, 30)
    pf.close()
    full.truncate(PROMPT)
    assert torch.equal(got, ref)
    c, b = pf.counters_dict(), base.counters_dict()
    assert c["selected_pairs"] == b["selected_pairs"] and c["hit_pairs"] + c["fetched_pairs"] == c["selected_pairs"]
    assert c["prefetched_pairs"] > 0 and c["prefetch_used_pairs"] > 0
    ov = pf.overlap()
    assert ov["prefetches_timed"] == 29 * 3  # every selecting layer, every decode step
    assert all(0.0 <= f <= 1.0 for f in ov["overlap_fraction"]) and all(s >= 0.0 for s in ov["stall_ms"])
    check_residency(pf)


def test_zerocopy_select_gathers_what_the_slot_tier_gathers(tiny) -> None:  # noqa: ANN001
    """tests/test_tiered.py:190 through select(): gather_zerocopy reads the selected pairs through
    the pinned store's device view; the gathered keys and values (up to the current block's fill)
    and the mask equal those of the slot tier's select(), which admits and gathers from slots."""
    from lazykv_b200.tiered import TieredCache, allocate_stages

    cfg, model = tiny
    _, full, _ = prefilled(model, cfg)
    zc = TieredCache(full, K, BS, capacity_tokens=CAP, dense_layers=1, fetch="zerocopy")
    slots = TieredCache(full, K, BS, capacity_tokens=CAP, dense_layers=1, fetch="gather", stages=allocate_stages(64, 2, cfg.head_dim, BS))
    h, hq, d = cfg.num_key_value_heads, cfg.num_attention_heads, cfg.head_dim
    gen = torch.Generator(device="cuda").manual_seed(9)
    kv = torch.zeros((1, h, 1, d), dtype=torch.bfloat16, device="cuda")
    for step in range(1, 4):
        q = torch.randn((1, hq, 1, d), generator=gen, device="cuda").bfloat16()
        for cache in (zc, slots):
            cache._step = step
        for layer in zc.tiers:
            a, b = zc.select(layer, q, kv, kv), slots.select(layer, q, kv, kv)
            valid = (K + 1) * BS + zc.tiers[layer].fill
            assert torch.equal(a[0][:, :, :valid], b[0][:, :, :valid]) and torch.equal(a[1][:, :, :valid], b[1][:, :, :valid])
            assert torch.equal(a[2], b[2])
    c = zc.counters_dict()
    assert c["zerocopy_bytes"] == c["selected_pairs"] * next(iter(zc.tiers.values())).pair_bytes > 0
