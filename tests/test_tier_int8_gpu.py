"""The int8 tier: the reference's rung-8 tests (tests/test_tiered_int8.py) on the device tier."""

from __future__ import annotations

import pytest
import torch

from tests.tiny_model import BS, CAP, K, PROMPT, forced, make_tiny, prefilled

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def tiny():  # noqa: ANN201
    return make_tiny()


def _dequantized(tier, block: int) -> torch.Tensor:  # noqa: ANN001
    """What a fetch of `block` puts in a slot: [h, 2, bs, d] in the model dtype."""
    from lazykv_b200.quant import unpack

    return unpack(tier.host[block].cuda(), tier.bs, tier.d, tier.pool.dtype)


def _build(model, full, **kw):  # noqa: ANN001, ANN202
    from lazykv_b200.tiered import TieredCache

    return TieredCache(full, K, BS, capacity_tokens=CAP, model=model, dense_layers=1, fetch="gather", quant="int8", **kw)


def test_the_host_pool_narrows_by_exactly_the_record_width(tiny) -> None:  # noqa: ANN001
    from lazykv_b200.quant import packed_pair_bytes

    cfg, model = tiny
    _, full, _ = prefilled(model, cfg)
    tier = _build(model, full)
    logical, stored = tier.host_logical_bytes(), tier.stats().host_kv_bytes
    assert stored / logical == packed_pair_bytes(BS, cfg.head_dim) / (2 * BS * cfg.head_dim * 2)
    assert tier.quant == "int8" and tier.policy_name == "tiered_int8"


@pytest.mark.parametrize("placement", ["host", "device"])
def test_every_resident_slot_holds_exactly_what_a_fetch_would_produce(tiny, placement: str) -> None:  # noqa: ANN001
    cfg, model = tiny
    ids, full, pre = prefilled(model, cfg)
    tier = _build(model, full, cold_placement=placement)
    forced(model, tier, pre, ids, 40)
    torch.cuda.synchronize()
    checked = 0
    for layer in tier.tiers.values():
        sb = layer.slot_block
        for j in range(layer.h):
            for s in range(layer.n_slots):
                b = int(sb[j, s])
                if b < 0:
                    continue
                assert torch.equal(layer.pool[s + 1, j], _dequantized(layer, b)[j])
                checked += 1
    assert checked > 0
    assert tier.counters_dict()["fetched_pairs"] > 0


def test_refetching_an_evicted_block_returns_the_same_bytes(tiny) -> None:  # noqa: ANN001
    import numpy as np

    cfg, model = tiny
    _, full, _ = prefilled(model, cfg)
    tier = _build(model, full)
    layer = next(iter(tier.tiers.values()))
    chosen = layer.slot_block[:, :1].copy()  # resident right now, in slot 1
    before = {j: layer.pool[1, j].clone() for j in range(layer.h)}
    layer.set_tables(slot_block=np.full_like(layer.slot_block, -1), block_slot=np.full_like(layer.block_slot, -1),
                     last_used=np.full_like(layer.last_used, -2))
    layer.pool[1:].zero_()
    layer.admit(chosen, step=1, counters=tier.counters)
    bsl = layer.block_slot
    for j in range(layer.h):
        slot = int(bsl[j, chosen[j, 0]])
        assert torch.equal(layer.pool[slot, j], before[j])


def test_the_sink_stays_exact_because_it_never_leaves_vram(tiny) -> None:  # noqa: ANN001
    cfg, model = tiny
    _, full, _ = prefilled(model, cfg)
    exact = {i: full.layers[i].keys[0, :, :BS].clone() for i in range(1, cfg.num_hidden_layers)}
    tier = _build(model, full)
    for i, layer in tier.tiers.items():
        assert torch.equal(layer.pool[0, :, 0], exact[i])


def test_the_quest_bound_is_taken_over_the_keys_that_are_actually_attended(tiny) -> None:  # noqa: ANN001
    cfg, model = tiny
    _, full, _ = prefilled(model, cfg)
    tier = _build(model, full)
    for layer in tier.tiers.values():
        for b in range(1, layer.n_sealed):
            keys = _dequantized(layer, b)[:, 0]
            assert (keys >= layer.kmin[0, :, b].unsqueeze(1)).all()
            assert (keys <= layer.kmax[0, :, b].unsqueeze(1)).all()
            assert torch.equal(layer.kmin[0, :, b], keys.amin(dim=1)) and torch.equal(layer.kmax[0, :, b], keys.amax(dim=1))


def test_decode_differs_from_the_bf16_tier_but_not_wildly(tiny) -> None:  # noqa: ANN001
    from lazykv_b200.tiered import TieredCache

    cfg, model = tiny
    ids, full, pre = prefilled(model, cfg)
    cont_steps = 40
    exact = TieredCache(full, K, BS, capacity_tokens=CAP, model=model, dense_layers=1, fetch="gather")
    ref = forced(model, exact, pre, ids, cont_steps)
    full.truncate(PROMPT)
    got = forced(model, _build(model, full), pre, ids, cont_steps)
    full.truncate(PROMPT)
    assert torch.isfinite(got).all()
    assert not torch.equal(got, ref)
    diff, spread = (got.float() - ref.float()).abs(), ref.float().std()
    assert diff.mean() < 0.02 * spread
    assert diff.max() < spread


def test_runs_fetch_is_refused(tiny) -> None:  # noqa: ANN001
    from lazykv_b200.tiered import TieredCache

    cfg, model = tiny
    _, full, _ = prefilled(model, cfg)
    with pytest.raises(ValueError, match="needs fetch='gather'"):
        TieredCache(full, K, BS, capacity_tokens=CAP, model=model, dense_layers=1, fetch="runs", quant="int8")


def test_a_bf16_host_pool_is_refused_for_an_int8_tier(tiny) -> None:  # noqa: ANN001
    from lazykv_b200.tiered import allocate_host_pools

    cfg, model = tiny
    _, full, _ = prefilled(model, cfg)
    wrong = allocate_host_pools(cfg.num_hidden_layers - 1, cfg.num_key_value_heads, cfg.head_dim, BS, CAP)
    with pytest.raises(ValueError, match="host pool must be pinned"):
        _build(model, full, host_pools=wrong)


def test_an_int8_host_pool_is_used_in_place(tiny) -> None:  # noqa: ANN001
    """allocate_host_pools(quant='int8') gives the exact record layout, and the tier writes into it."""
    from lazykv_b200.tiered import allocate_host_pools

    cfg, model = tiny
    _, full, _ = prefilled(model, cfg)
    pools = allocate_host_pools(cfg.num_hidden_layers - 1, cfg.num_key_value_heads, cfg.head_dim, BS, CAP, quant="int8")
    tier = _build(model, full, host_pools=pools)
    for i, layer in tier.tiers.items():
        assert layer.host.data_ptr() == pools[i - 1].data_ptr()
