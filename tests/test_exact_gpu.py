"""The exact tier (ExactTieredCache): the reference's rung-9 tests (tests/test_exact.py) on the
device, plus the int8 composition the reference refuses and this build allows."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from tests.tiny_model import BS, CAP, K, PROMPT, check_residency, forced, make_tiny, prefilled

pytestmark = pytest.mark.gpu


def _reference(keys: torch.Tensor, values: torch.Tensor, query: torch.Tensor, scaling: float) -> torch.Tensor:
    """Softmax attention over the whole key set in float64."""
    scores = torch.matmul(query.double(), keys.double().transpose(-1, -2)) * scaling
    return torch.matmul(torch.softmax(scores, dim=-1), values.double())


# -- the algebra (tests/test_exact.py:32-105), float32 on the device --------------------------------


def test_merging_two_halves_reconstructs_attention_over_the_whole() -> None:
    from lazykv_b200.exact import cpu_partial_attention, merge_lse

    torch.manual_seed(0)
    h, groups, n_blocks, d = 2, 4, 6, 16
    keys = torch.randn(h, n_blocks * BS, d, device="cuda")
    values = torch.randn(h, n_blocks * BS, d, device="cuda")
    query = torch.randn(h, groups, d, device="cuda")
    scaling = d**-0.5
    first = np.tile(np.arange(0, 2), (h, 1))
    second = np.tile(np.arange(2, n_blocks), (h, 1))
    out_a, lse_a = cpu_partial_attention(keys, values, query, scaling, BS, excluded=second)
    out_b, lse_b = cpu_partial_attention(keys, values, query, scaling, BS, excluded=first)
    merged, _ = merge_lse(out_a, lse_a, out_b, lse_b)
    want = _reference(keys, values, query, scaling)
    assert torch.allclose(merged.double(), want, atol=1e-5)


def test_an_empty_partial_contributes_nothing_instead_of_nan() -> None:
    from lazykv_b200.exact import cpu_partial_attention, merge_lse

    torch.manual_seed(1)
    h, groups, n_blocks, d = 2, 2, 4, 16
    keys, values = torch.randn(h, n_blocks * BS, d, device="cuda"), torch.randn(h, n_blocks * BS, d, device="cuda")
    query = torch.randn(h, groups, d, device="cuda")
    everything = np.tile(np.arange(n_blocks), (h, 1))
    empty_out, empty_lse = cpu_partial_attention(keys, values, query, d**-0.5, BS, excluded=everything)
    assert torch.isneginf(empty_lse).all() and torch.isfinite(empty_out).all()
    full_out, full_lse = cpu_partial_attention(keys, values, query, d**-0.5, BS, excluded=np.empty((h, 0), dtype=np.int64))
    merged, lse = merge_lse(full_out, full_lse, empty_out, empty_lse)
    assert torch.allclose(merged, full_out, atol=1e-6) and torch.equal(lse, full_lse)
    both, both_lse = merge_lse(empty_out, empty_lse, empty_out, empty_lse)
    assert torch.isneginf(both_lse).all() and (both == 0).all()


def test_the_merge_is_not_a_plain_average() -> None:
    from lazykv_b200.exact import merge_lse

    out_a = torch.tensor([[1.0, 0.0]], device="cuda")
    out_b = torch.tensor([[0.0, 1.0]], device="cuda")
    lse_a, lse_b = torch.tensor([2.0], device="cuda"), torch.tensor([0.0], device="cuda")
    merged, lse = merge_lse(out_a, lse_a, out_b, lse_b)
    wa = float(torch.exp(lse_a - lse))
    assert float(merged[0, 0]) == pytest.approx(wa, rel=1e-6)
    assert merged[0, 0] > merged[0, 1]
    assert float(lse) == pytest.approx(float(torch.logaddexp(lse_a, lse_b)), rel=1e-6)


def test_excluding_a_block_removes_exactly_that_block() -> None:
    from lazykv_b200.exact import cpu_partial_attention

    torch.manual_seed(2)
    h, groups, n_blocks, d = 2, 1, 5, 16
    keys, values = torch.randn(h, n_blocks * BS, d, device="cuda"), torch.randn(h, n_blocks * BS, d, device="cuda")
    query = torch.randn(h, groups, d, device="cuda")
    excluded = np.array([[2], [4]], dtype=np.int64)
    out, _ = cpu_partial_attention(keys, values, query, d**-0.5, BS, excluded)
    for j, drop in enumerate(excluded[:, 0]):
        keep = [t for t in range(n_blocks * BS) if not (drop * BS <= t < (drop + 1) * BS)]
        want = _reference(keys[j, keep], values[j, keep], query[j], d**-0.5)
        assert torch.allclose(out[j].double(), want, atol=1e-5)


# -- end to end on the tiny model (tests/test_exact.py:142-230) ----------------------------------------


@pytest.fixture(scope="module")
def tiny():  # noqa: ANN201
    return make_tiny()


def _within_delta(want: torch.Tensor, got: torch.Tensor, bar: float) -> float:
    delta = (want - got).abs().max().item()
    assert delta < bar, delta
    for i in (want.argmax(-1) != got.argmax(-1)).nonzero().flatten().tolist():
        top2 = want[i].topk(2).values
        assert (top2[0] - top2[1]).item() < 2 * delta, (i, top2, delta)
    return delta


@pytest.mark.parametrize("budget_blocks", [2, K])
@pytest.mark.parametrize(("fetch", "split"), [("gather", False), ("gather", True), ("zerocopy", False)])
def test_exact_tier_reproduces_the_full_cache(tiny, budget_blocks: int, fetch: str, split: bool) -> None:  # noqa: ANN001
    """split: the resident split (attention before the admit, the admit on a second stream)."""
    from lazykv_b200.exact import ExactTieredCache

    cfg, model = tiny
    ids, full, pre = prefilled(model, cfg)
    steps = 24
    want = forced(model, full, pre, ids, steps)
    full.truncate(PROMPT)
    n_slots = None if fetch == "zerocopy" else budget_blocks + 1
    cache = ExactTieredCache(full, budget_blocks, BS, capacity_tokens=CAP, dense_layers=1, fetch=fetch, n_slots=n_slots, resident_split=split)
    assert cache.resident_split == split
    got = forced(model, cache, pre, ids, steps)
    cache.close()
    full.truncate(PROMPT)
    _within_delta(want, got, 0.02)
    assert cache.exact.merges == (steps - 1) * (cfg.num_hidden_layers - 1)
    assert cache.exact.cold_tokens > 0
    if fetch == "gather":
        check_residency(cache)


def test_exact_tier_is_further_from_the_approximate_tier_than_from_the_full_cache(tiny) -> None:  # noqa: ANN001
    from lazykv_b200.exact import ExactTieredCache
    from lazykv_b200.tiered import TieredCache

    cfg, model = tiny
    ids, full, pre = prefilled(model, cfg)
    steps = 16
    reference = forced(model, full, pre, ids, steps)
    full.truncate(PROMPT)
    approx = TieredCache(full, 2, BS, capacity_tokens=CAP, dense_layers=1, fetch="gather", n_slots=3)
    approx_logits = forced(model, approx, pre, ids, steps)
    approx.close()
    full.truncate(PROMPT)
    exact = ExactTieredCache(full, 2, BS, capacity_tokens=CAP, dense_layers=1, fetch="gather", n_slots=3)
    exact_logits = forced(model, exact, pre, ids, steps)
    exact.close()
    assert (exact_logits - reference).abs().max() < (approx_logits - reference).abs().max()


def test_select_protocol_merge_reproduces_the_full_cache(tiny) -> None:  # noqa: ANN001
    """The reference's select -> SDPA -> merge protocol (exact.py:225-264) through merge()."""
    from lazykv_b200.exact import ExactTieredCache

    cfg, model = tiny
    ids, full, pre = prefilled(model, cfg)
    steps = 16
    want = forced(model, full, pre, ids, steps)
    full.truncate(PROMPT)
    cache = ExactTieredCache(full, K, BS, capacity_tokens=CAP, dense_layers=1, fetch="gather")
    cache.decode = lambda *args, **kw: None  # type: ignore[method-assign]
    got = forced(model, cache, pre, ids, steps)
    cache.close()
    _within_delta(want, got, 0.02)
    assert cache.exact.merges == (steps - 1) * (cfg.num_hidden_layers - 1)


def test_exact_tier_refuses_a_prefetch(tiny) -> None:  # noqa: ANN001
    from lazykv_b200.exact import ExactTieredCache

    cfg, model = tiny
    _, full, _ = prefilled(model, cfg)
    with pytest.raises(ValueError, match="prefetch"):
        ExactTieredCache(full, K, BS, capacity_tokens=CAP, dense_layers=1, fetch="gather", model=model, prefetch=True)


@pytest.mark.parametrize(("placement", "split"), [("host", False), ("device", False), ("host", True), ("device", True)])
def test_int8_exact_step_matches_the_oracle(tiny, placement: str, split: bool) -> None:  # noqa: ANN001
    """One exact int8 decode step of a tiered layer against the CPU restatement of the composition:
    sink and current block exact, every other sealed block as unpack(record) in bf16 (selected or
    not), merged. Float32 output within 1e-5 of the float64 oracle. With the resident split the
    chosen blocks not yet resident are attended from their records while the admit runs beside."""
    import oracle
    from lazykv_b200.exact import ExactTieredCache
    from tests.golden.inputs import to_np

    cfg, model = tiny
    _, full, _ = prefilled(model, cfg)
    sealed_kv = {i: (full.layers[i].keys[0, :, :PROMPT].clone(), full.layers[i].values[0, :, :PROMPT].clone()) for i in range(1, 4)}
    cache = ExactTieredCache(full, K, BS, capacity_tokens=CAP, dense_layers=1, fetch="gather", quant="int8", cold_placement=placement,
                             resident_split=split)
    gen = torch.Generator(device="cuda").manual_seed(3)
    for i, tier in cache.tiers.items():
        q = torch.randn((1, cfg.num_attention_heads, 1, cfg.head_dim), generator=gen, device="cuda").to(torch.bfloat16)
        scale = cfg.head_dim**-0.5
        out = tier.attend(q, scale, step=1, exact=True).clone()
        torch.cuda.synchronize()
        keys, values = sealed_kv[i]
        n = tier.n_sealed
        pairs = torch.stack([keys[:, : n * BS], values[:, : n * BS]], dim=1).unflatten(2, (n, BS)).permute(2, 0, 1, 3, 4)  # [n, h, 2, bs, d]
        cur = torch.zeros((tier.h, 2, BS, tier.d), dtype=keys.dtype, device=keys.device)
        cur[:, 0, : tier.fill] = keys[:, n * BS :]
        cur[:, 1, : tier.fill] = values[:, n * BS :]
        chosen = tier.chosen.cpu().numpy().astype(np.int64)
        r = oracle.tiered_decode(to_np(q[0, :, 0]), to_np(pairs), to_np(cur), tier.fill, K, scale, "bfloat16", quant="int8", selected=chosen)
        # The tier's own choice is the oracle's up to ties: the chosen set must reach the K-th bound.
        assert np.array_equal(np.sort(chosen, axis=1), np.sort(r["selected"], axis=1)) or _tied(r["bound"], chosen, K)
        want = r["out"].reshape(-1, tier.d)
        got = to_np(out)
        assert np.abs(got - want).max() <= 1e-5 * max(1.0, np.abs(want).max()), np.abs(got - want).max()
    cache.close()


def _tied(bound: np.ndarray, chosen: np.ndarray, k: int) -> bool:
    """Whether `chosen` [h, k] (block ids, candidates start at block 1) is a valid top-k of bound [h, n]."""
    for j in range(bound.shape[0]):
        kth = np.sort(bound[j])[::-1][k - 1]
        if (bound[j, chosen[j] - 1] < kth).any():
            return False
    return True


def test_int8_exact_tier_is_closer_to_the_full_cache_than_the_int8_tier(tiny) -> None:  # noqa: ANN001
    """The int8 exact tier attends to every block (dequantised): nearer the full cache than the
    approximate int8 tier, and within the quantisation's reach of it."""
    from lazykv_b200.exact import ExactTieredCache
    from lazykv_b200.tiered import TieredCache

    cfg, model = tiny
    ids, full, pre = prefilled(model, cfg)
    steps = 16
    reference = forced(model, full, pre, ids, steps)
    full.truncate(PROMPT)
    approx = TieredCache(full, 2, BS, capacity_tokens=CAP, dense_layers=1, fetch="gather", quant="int8")
    a = forced(model, approx, pre, ids, steps)
    approx.close()
    full.truncate(PROMPT)
    exact = ExactTieredCache(full, 2, BS, capacity_tokens=CAP, dense_layers=1, fetch="gather", quant="int8")
    e = forced(model, exact, pre, ids, steps)
    exact.close()
    assert exact.policy_name == "tiered_exact_int8"
    assert torch.isfinite(e).all()
    assert (e - reference).abs().max() < (a - reference).abs().max()
    spread = reference.float().std()
    assert (e - reference).abs().mean() < 0.02 * spread
