"""Layer-major tiered prefill (tests/test_tiered_prefill.py): the same tier, bit for bit, without
the selecting layers' prompt KV in the full cache."""

from __future__ import annotations

import pytest
import torch

from tests.tiny_model import BS, CAP, K, PROMPT, ids_for, make_tiny

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def tiny():  # noqa: ANN201
    return make_tiny()


def _reference(model, cfg, ids, chunk: int, cache_cls=None, **kw):  # noqa: ANN001, ANN202
    """Chunk-major prefill into a full GPU cache, then the tier built from it."""
    from lazykv_b200.cache import FullGPUCache
    from lazykv_b200.generate import prefill
    from lazykv_b200.tiered import TieredCache

    full = FullGPUCache(cfg.num_hidden_layers, CAP)
    pre = prefill(model, full, ids[:, :PROMPT], chunk_size=chunk)
    tier = (cache_cls or TieredCache)(full, K, BS, capacity_tokens=CAP, model=model, dense_layers=1, **kw)
    return pre.last_logits, tier


@pytest.mark.parametrize("chunk", [32, 100, 128])
@pytest.mark.parametrize(("prefetch", "quant"), [(False, None), (True, None), (False, "int8")])
def test_layer_major_prefill_matches_the_full_cache_path(tiny, chunk: int, prefetch: bool, quant: str | None) -> None:  # noqa: ANN001
    from lazykv_b200.generate import teacher_forced_decode
    from lazykv_b200.tiered_prefill import tiered_prefill

    cfg, model = tiny
    ids = ids_for(cfg)
    kw = {"prefetch": prefetch, "fetch": "gather", "quant": quant}
    ref_logits, ref = _reference(model, cfg, ids, chunk, **kw)
    got = tiered_prefill(model, ids[:, :PROMPT], chunk, K, BS, CAP, dense_layers=1, **kw)
    assert got.chunks == -(-PROMPT // chunk)
    assert torch.equal(got.last_logits, ref_logits)
    for i, t in got.cache.tiers.items():
        r = ref.tiers[i]
        assert (t.n_sealed, t.fill, t.length) == (r.n_sealed, r.fill, r.length)
        assert torch.equal(t.host[: t.n_sealed], r.host[: r.n_sealed])
        assert torch.equal(t.kmin[:, :, : t.n_sealed], r.kmin[:, :, : r.n_sealed])
        assert torch.equal(t.kmax[:, :, : t.n_sealed], r.kmax[:, :, : r.n_sealed])
        assert torch.equal(t.pool, r.pool)
        assert (t.slot_block == r.slot_block).all()
    assert torch.equal(got.full.layers[0].keys[:, :, :PROMPT], ref.full.layers[0].keys[:, :, :PROMPT])
    cont = ids[:, PROMPT : PROMPT + 40]
    a = torch.stack(list(teacher_forced_decode(model, ref, ref_logits, cont)))
    b = torch.stack(list(teacher_forced_decode(model, got.cache, got.last_logits, cont)))
    ref.close()
    got.cache.close()
    assert torch.equal(a, b)
    assert got.cache.counters.boundary_d2h_bytes == ref.counters.boundary_d2h_bytes


def test_layer_major_prefill_builds_the_exact_tier(tiny) -> None:  # noqa: ANN001
    from lazykv_b200.exact import ExactTieredCache
    from lazykv_b200.generate import teacher_forced_decode
    from lazykv_b200.tiered_prefill import tiered_prefill

    cfg, model = tiny
    ids = ids_for(cfg)
    ref_logits, ref = _reference(model, cfg, ids, 32, cache_cls=ExactTieredCache, fetch="gather", quant="int8")
    got = tiered_prefill(model, ids[:, :PROMPT], 32, K, BS, CAP, dense_layers=1, fetch="gather", quant="int8", cache_cls=ExactTieredCache)
    assert isinstance(got.cache, ExactTieredCache)
    cont = ids[:, PROMPT : PROMPT + 24]
    a = torch.stack(list(teacher_forced_decode(model, ref, ref_logits, cont)))
    b = torch.stack(list(teacher_forced_decode(model, got.cache, got.last_logits, cont)))
    ref.close()
    got.cache.close()
    assert torch.equal(a, b)
    assert got.cache.exact.merges == 23 * (cfg.num_hidden_layers - 1)


def test_selecting_layers_never_allocate_in_the_full_cache(tiny) -> None:  # noqa: ANN001
    from lazykv_b200.tiered_prefill import tiered_prefill

    cfg, model = tiny
    got = tiered_prefill(model, ids_for(cfg)[:, :PROMPT], 32, K, BS, CAP, dense_layers=1)
    got.cache.close()
    assert got.full.layers[0].is_initialized and got.full.layers[0].get_seq_length() == PROMPT
    assert not any(layer.is_initialized for layer in got.full.layers[1:])
    assert len(got.layer_s) == cfg.num_hidden_layers


def test_prompt_longer_than_capacity_is_refused(tiny) -> None:  # noqa: ANN001
    from lazykv_b200.tiered_prefill import tiered_prefill

    cfg, model = tiny
    with pytest.raises(ValueError, match="exceeds capacity"):
        tiered_prefill(model, ids_for(cfg)[:, :PROMPT], 32, K, BS, capacity_tokens=64, dense_layers=1)


def test_layer_major_prefill_stores_what_the_oracle_packs(tiny) -> None:  # noqa: ANN001
    """The tier the layer-major prefill writes, against the oracle (lazykv/quant.py:73-105 pack and
    unpack, lazykv/selection.py:142-144 min/max, lazykv/tiered.py:187-202): each selecting layer's int8
    records byte-exact with the oracle's pack of the KV the model computed (read from a chunk-major
    prefill's full cache), the metadata the min/max of the dequantised keys, the sink slot the exact
    first block and the current slot the unsealed tail."""
    import numpy as np

    import oracle as O
    from lazykv_b200.cache import FullGPUCache
    from lazykv_b200.generate import prefill
    from lazykv_b200.tiered_prefill import tiered_prefill

    cfg, model = tiny
    ids = ids_for(cfg)
    full = FullGPUCache(cfg.num_hidden_layers, CAP)
    prefill(model, full, ids[:, :PROMPT], chunk_size=32)
    got = tiered_prefill(model, ids[:, :PROMPT], 32, K, BS, CAP, dense_layers=1, fetch="gather", quant="int8")
    n_blocks, tail = divmod(PROMPT, BS)
    for i, t in got.cache.tiers.items():
        keys = full.layers[i].keys[0, :, :PROMPT].float().cpu().numpy()  # [h, T, d]
        values = full.layers[i].values[0, :, :PROMPT].float().cpu().numpy()
        h, _, d = keys.shape
        pairs = np.stack([keys[:, : n_blocks * BS], values[:, : n_blocks * BS]], axis=1).reshape(h, 2, n_blocks, BS, d).transpose(2, 0, 1, 3, 4)
        want = O.pack(pairs)  # [n, h, W]
        assert t.n_sealed == n_blocks and t.fill == tail
        assert np.array_equal(t.host[:n_blocks].numpy(), want)
        deq = O.unpack(want.reshape(n_blocks * h, -1), BS, d, "bfloat16").reshape(n_blocks, h, 2, BS, d)
        kmin, kmax = O.block_minmax(deq[:, :, 0].transpose(1, 0, 2, 3).reshape(h, n_blocks * BS, d), BS)
        assert np.array_equal(t.kmin[0, :, 1:n_blocks].float().cpu().numpy(), kmin[:, 1:])
        assert np.array_equal(t.kmax[0, :, 1:n_blocks].float().cpu().numpy(), kmax[:, 1:])
        assert np.array_equal(t.pool[0].float().cpu().numpy(), pairs[0])  # the sink stays exact
        cur = t.pool[t.tail_slot, :, :, :tail].float().cpu().numpy()
        assert np.array_equal(cur[:, 0], keys[:, n_blocks * BS :]) and np.array_equal(cur[:, 1], values[:, n_blocks * BS :])
    got.cache.close()
