"""Ragged continuous batching (config 3): several sequences of different lengths decoded in one
step, each through its own block table, against the reference's per-sequence composition (the
oracle's tiered_decode: Quest top-K, int8 store, exact merge) one sequence at a time."""

from __future__ import annotations

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

H, G, D, BS = 2, 4, 64, 16
SCALE = D**-0.5


def _kv(gen: torch.Generator, n: int) -> tuple[torch.Tensor, torch.Tensor]:
    keys = torch.randn((H, n, D), generator=gen, device="cuda") + torch.randn((H, 1, D), generator=gen, device="cuda") * 0.5
    values = torch.randn((H, n, D), generator=gen, device="cuda")
    return keys.bfloat16(), values.bfloat16()


def _oracle(keys: torch.Tensor, values: torch.Tensor, query: torch.Tensor, k: int, n: int) -> dict:
    """The reference's decode step for one sequence: keys / values [H, L, D] bf16, query [H*G, D],
    n sealed blocks (a full current block is sealed lazily, at the next append)."""
    from oracle import restatement as O

    fill = keys.shape[1] - n * BS
    kv = torch.stack([keys, values], dim=1).float().cpu().numpy()  # [H, 2, L, D]
    sealed = kv[:, :, : n * BS].reshape(H, 2, n, BS, D).transpose(2, 0, 1, 3, 4)
    current = np.zeros((H, 2, BS, D), dtype=np.float32)
    current[:, :, :fill] = kv[:, :, n * BS :]
    return O.tiered_decode(query.float().cpu().numpy(), sealed, current, fill, k, SCALE, model_dtype="bfloat16", quant="int8")


def _check(tier, ids: list[int], kv: dict, gen: torch.Generator, fetch: bool) -> None:  # noqa: ANN001
    q = torch.randn((len(ids) * H * G, D), generator=gen, device="cuda").bfloat16()
    out, lse, sel = tier.decode(ids, q, SCALE, fetch=fetch)
    torch.cuda.synchronize()
    for b, s in enumerate(ids):
        k = tier.k_of(s)
        want = _oracle(*kv[s], q[b * H * G : (b + 1) * H * G], k, tier.seqs[s].n_sealed)
        rows = slice(b * H, (b + 1) * H)
        got_sel = np.sort(sel[rows, :k].cpu().numpy(), axis=1)
        assert np.array_equal(got_sel, np.sort(want["selected"], axis=1)), (s, k)
        got = out[b * H * G : (b + 1) * H * G].double().cpu().numpy().reshape(H, G, D)
        np.testing.assert_allclose(got, want["out"], atol=1e-5)
        np.testing.assert_allclose(lse[b * H * G : (b + 1) * H * G].double().cpu().numpy().reshape(H, G), want["lse"], rtol=1e-5, atol=1e-5)


@pytest.mark.parametrize("placement", ["device", "host"])  # the int8 store in HBM, or pinned host memory read over the link
@pytest.mark.parametrize("fetch", [False, True])  # kept blocks read in place from the store, or fetched into HBM slots
def test_one_launch_matches_each_sequence_decoded_alone(fetch: bool, placement: str) -> None:
    from lazykv_b200 import kernels
    from lazykv_b200.ragged import RaggedTier

    gen = torch.Generator(device="cuda").manual_seed(11)
    tier = RaggedTier(H, G, D, BS, max_seqs=8, max_tokens=2048, store_blocks=1024, budget=0.25, cold_placement=placement)
    lengths = [40, 47, 100, 333, 700, 1500]  # 2 sealed blocks (all kept), a partial tail, many blocks
    kv = {}
    ids = []
    for n in lengths:
        keys, values = _kv(gen, n)
        s = tier.add(keys, values)
        kv[s] = (keys, values)
        ids.append(s)
    _check(tier, ids, kv, gen, fetch)
    assert kernels.device_status() == 0


@pytest.mark.parametrize("placement", ["device", "host"])
@pytest.mark.parametrize("fetch", [False, True])
def test_sequences_grow_seal_finish_and_are_replaced(fetch: bool, placement: str) -> None:
    from lazykv_b200 import kernels
    from lazykv_b200.ragged import RaggedTier

    gen = torch.Generator(device="cuda").manual_seed(12)
    tier = RaggedTier(H, G, D, BS, max_seqs=6, max_tokens=1024, store_blocks=256, budget=0.25, cold_placement=placement)
    kv = {}
    for n in (63, 64, 200, 511):  # a block-boundary length: the current block starts empty
        keys, values = _kv(gen, n)
        kv[tier.add(keys, values)] = (keys, values)
    for step in range(20):
        for s in list(kv):
            k1, v1 = _kv(gen, 1)
            tier.append(s, k1[:, 0], v1[:, 0])
            kv[s] = (torch.cat([kv[s][0], k1], dim=1), torch.cat([kv[s][1], v1], dim=1))
        if step in (3, 11):  # a sequence finishes, a new one takes a slot (and free store rows)
            gone = sorted(kv)[step % len(kv)]
            tier.drop(gone)
            del kv[gone]
            keys, values = _kv(gen, 90 + 7 * step)
            kv[tier.add(keys, values)] = (keys, values)
        if step % 4 == 3 or step == 19:
            _check(tier, sorted(kv), kv, gen, fetch)
    assert kernels.device_status() == 0


@pytest.mark.parametrize("fetch", [False, True])
def test_host_cold_tier_is_bit_identical_to_the_device_store(fetch: bool) -> None:
    """The store in pinned host memory (its records staged in HBM by mapped loads each step) gives
    the outputs, log-sum-exps and selections of the store in HBM, bit for bit; the host store holds
    the same records."""
    from lazykv_b200.ragged import RaggedTier

    tiers = [RaggedTier(H, G, D, BS, max_seqs=8, max_tokens=4096, store_blocks=2048, budget=0.0625, cold_placement=p) for p in ("device", "host")]
    gen = torch.Generator(device="cuda").manual_seed(21)
    ids = []
    for n in (33, 64, 777, 2049, 4000):
        keys, values = _kv(gen, n)
        slots = [t.add(keys, values) for t in tiers]
        assert slots[0] == slots[1]
        ids.append(slots[0])
    for _ in range(3):
        q = torch.randn((len(ids) * H * G, D), generator=gen, device="cuda").bfloat16()
        (oa, la, sa), (ob, lb, sb) = (t.decode(ids, q, SCALE, fetch=fetch) for t in tiers)
        assert torch.equal(oa, ob) and torch.equal(la, lb)
        for i, s in enumerate(ids):  # selection entries past a row's K are unspecified
            k = tiers[0].k_of(s)
            assert torch.equal(sa[i * H : (i + 1) * H, :k], sb[i * H : (i + 1) * H, :k])
        k1, v1 = _kv(gen, 1)
        for t in tiers:
            for s in ids:
                t.append(s, k1[:, 0], v1[:, 0])
    torch.cuda.synchronize()
    used = torch.tensor(sorted(r for seq in tiers[0].seqs.values() for r in seq.rows))
    assert used.numel() > 0
    assert torch.equal(tiers[0].records.cpu()[used], tiers[1].records_host[used])


def test_ragged_select_rejects_what_it_cannot_hold() -> None:
    from lazykv_b200.ragged import RaggedTier

    with pytest.raises(ValueError, match="tensor-core"):
        RaggedTier(H, G, 128, BS, 2, 1024, 64, 0.25)
    with pytest.raises(ValueError, match="cold_placement"):
        RaggedTier(H, G, D, BS, 2, 1024, 64, 0.25, cold_placement="disk")
    tier = RaggedTier(H, G, D, BS, max_seqs=1, max_tokens=256, store_blocks=8, budget=0.25)
    gen = torch.Generator(device="cuda").manual_seed(13)
    keys, values = _kv(gen, 100)
    tier.add(keys, values)
    with pytest.raises(RuntimeError, match="slots"):
        tier.add(keys, values)
