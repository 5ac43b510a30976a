"""Session snapshots on the device tier: a restored session continues exactly as the saved one would
have (the reference's tests/test_snapshot.py), for the bf16 tier and for the int8 tier, which the
reference cannot snapshot."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from tests.tiny_model import BS, CAP, K, PROMPT, make_tiny

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def tiny():  # noqa: ANN201
    return make_tiny()


def _feed(model, cache, toks: list[int]) -> list[torch.Tensor]:  # noqa: ANN001
    from lazykv_b200.generate import cache_model_kwargs

    out = []
    ids = torch.empty((1, 1), dtype=torch.long, device="cuda")
    with torch.inference_mode():
        for t in toks:
            ids.fill_(t)
            out.append(model(input_ids=ids, past_key_values=cache, use_cache=True, logits_to_keep=1, **cache_model_kwargs(cache)).logits[0, -1].float())
    return out


def _direct_io_ok(path) -> bool:  # noqa: ANN001
    from lazykv_b200 import snapshot

    try:
        snapshot._DirectReader(path).close()
        return True
    except OSError:
        return False


@pytest.mark.parametrize("mid", [0, 5, 12, 20])  # 20: the tail is exactly full and not yet sealed (lazy seal)
@pytest.mark.parametrize("quant,rebuild,exact", [(None, "store", False), (None, "boundary", False), ("int8", "store", False),
                                                 ("int8", "store", True), (None, "store", True)])
def test_restored_session_continues_bit_identically(tiny, tmp_path, mid: int, quant: str | None, rebuild: str, exact: bool) -> None:  # noqa: ANN001
    from lazykv_b200 import snapshot
    from lazykv_b200.cache import FullGPUCache
    from lazykv_b200.exact import ExactTieredCache
    from lazykv_b200.generate import prefill
    from lazykv_b200.tiered import TieredCache

    cfg, model = tiny
    cls = ExactTieredCache if exact else TieredCache
    gen = torch.Generator(device="cuda").manual_seed(3)
    ids = torch.randint(0, cfg.vocab_size, (PROMPT + 40,), device="cuda", generator=gen)
    full = FullGPUCache(cfg.num_hidden_layers, CAP)
    pre = prefill(model, full, ids[:PROMPT], chunk_size=32)
    tier = cls(full, K, BS, CAP, model=model, dense_layers=1, fetch="gather", quant=quant)
    before = _feed(model, tier, ids[PROMPT : PROMPT + mid].tolist())
    logits = before[-1] if before else pre.last_logits
    if mid == 20:
        assert next(iter(tier.tiers.values())).fill == BS  # the case this parameter exists for
    path = tmp_path / "s.lkv"
    st = snapshot.save(tier, logits, path)
    assert path.stat().st_size == st.bytes_written and st.bytes_written % snapshot.ALIGN == 0
    assert snapshot.read_header(path)[0]["magic"] == (snapshot.MAGIC if quant is None else snapshot.MAGIC_INT8)
    saved = {i: (t.host[: t.n_sealed].clone(), t.kmin[:, :, : t.n_sealed].clone(), t.kmax[:, :, : t.n_sealed].clone(), t.pool[0].clone())
             for i, t in tier.tiers.items()}
    ref = _feed(model, tier, ids[PROMPT + mid :].tolist())
    tier.close()

    unbuffered = mid == 5 and _direct_io_ok(path)  # one case through O_DIRECT reads where the filesystem has them
    got_cache, got_logits, rs = snapshot.restore(path, K, CAP, cfg.num_hidden_layers, model=model, fetch="gather", unbuffered=unbuffered,
                                                 rebuild=rebuild, cache_cls=cls)
    assert type(got_cache) is cls and got_cache.quant == quant
    assert torch.equal(got_logits, logits.float())
    assert got_cache.get_seq_length(0) == PROMPT + mid and got_cache.get_seq_length(2) == PROMPT + mid
    # The store rebuild reproduces the saved state; the boundary one seals a tail that is exactly full
    # (as the constructor does at that length), which the next append would seal anyway.
    for i, t in got_cache.tiers.items() if rebuild == "store" else ():
        host, kmin, kmax, sink = saved[i]
        n = t.n_sealed
        assert torch.equal(t.host[:n], host) and torch.equal(t.pool[0], sink)
        assert torch.equal(t.kmin[:, :, :n], kmin) and torch.equal(t.kmax[:, :, :n], kmax)
    got = _feed(model, got_cache, ids[PROMPT + mid :].tolist())
    got_cache.close()
    assert all(torch.equal(a, b) for a, b in zip(got, ref, strict=True))
    assert rs.bytes_read > 0


@pytest.mark.parametrize("quant", [None, "int8"])
@pytest.mark.parametrize("n_slots", [None, 7])  # 7: spare slots beyond the budget stay empty
@pytest.mark.parametrize("length", [64, 70, 260])  # 64: no tail; 70: a tail; 260: many chunks
def test_from_store_builds_the_constructors_layer(length: int, n_slots: int | None, quant: str | None, monkeypatch) -> None:  # noqa: ANN001
    """A layer rebuilt from its host store equals the one the constructor builds from the same KV,
    in every tensor and table, across chunk edges (the int8 store from its records and the exact sink)."""
    from lazykv_b200 import tiered
    from lazykv_b200.tiered import TieredLayer

    monkeypatch.setattr(tiered, "BOUNDARY_CHUNK", 3)  # several chunks, seeded slots straddling an edge
    gen = torch.Generator(device="cuda").manual_seed(length)
    h, d = 2, 16
    keys = torch.randn((1, h, length, d), device="cuda", generator=gen).bfloat16()
    values = torch.randn((1, h, length, d), device="cuda", generator=gen).bfloat16()
    ref = TieredLayer(keys, values, K, BS, CAP, n_slots=n_slots, quant=quant)
    n, fill = divmod(length, BS)
    host = tiered.pinned_empty(tuple(ref.host.shape), ref.host.dtype)
    host[:n].copy_(ref.host[:n])
    tail = ref.pool[ref.tail_slot, :, :, :fill].cpu()
    got = TieredLayer.from_store(host, n, tail, K, BS, CAP, torch.device("cuda"), n_slots, quant=quant, sink=ref.pool[0].cpu())
    torch.cuda.synchronize()
    assert (got.n_sealed, got.fill, got.length) == (ref.n_sealed, ref.fill, ref.length)
    assert torch.equal(got.kmin[:, :, :n], ref.kmin[:, :, :n]) and torch.equal(got.kmax[:, :, :n], ref.kmax[:, :, :n])
    seed = min(ref.n_slots, n - 1)
    assert torch.equal(got.pool[: seed + 1], ref.pool[: seed + 1])
    assert torch.equal(got.pool[got.tail_slot], ref.pool[ref.tail_slot])
    for name in ("slot_block", "block_slot", "last_used", "evicted_at"):
        assert np.array_equal(getattr(got, name), getattr(ref, name)), name


def test_int8_snapshots_need_the_store_rebuild_and_the_sink(tiny, tmp_path) -> None:  # noqa: ANN001
    from lazykv_b200 import snapshot
    from lazykv_b200.cache import FullGPUCache
    from lazykv_b200.generate import prefill
    from lazykv_b200.tiered import TieredCache, TieredLayer

    cfg, model = tiny
    full = FullGPUCache(cfg.num_hidden_layers, CAP)
    pre = prefill(model, full, torch.arange(PROMPT, device="cuda") % cfg.vocab_size, chunk_size=32)
    tier = TieredCache(full, K, BS, CAP, dense_layers=1, fetch="gather", quant="int8")
    path = tmp_path / "x.lkv"
    snapshot.save(tier, pre.last_logits, path)
    with pytest.raises(ValueError, match="store"):
        snapshot.restore(path, K, CAP, cfg.num_hidden_layers, rebuild="boundary")
    layer = next(iter(tier.tiers.values()))
    with pytest.raises(ValueError, match="sink"):
        TieredLayer.from_store(layer.host, layer.n_sealed, layer.pool[layer.tail_slot, :, :, : layer.fill].cpu(), K, BS, CAP,
                               torch.device("cuda"), quant="int8")
    with pytest.raises(ValueError, match="store does not hold"):
        TieredLayer.from_store(layer.host, layer.n_sealed, layer.pool[layer.tail_slot, :, :, : layer.fill].cpu(), K, BS, CAP,
                               torch.device("cuda"), sink=layer.pool[0].cpu())
