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


@pytest.mark.parametrize("fetch", [False, True])  # kept blocks read in place from the store, or fetched into HBM slots
def test_one_launch_matches_each_sequence_decoded_alone(fetch: bool) -> None:
    from lazykv_b200 import kernels
    from lazykv_b200.ragged import RaggedTier

    gen = torch.Generator(device="cuda").manual_seed(11)
    tier = RaggedTier(H, G, D, BS, max_seqs=8, max_tokens=2048, store_blocks=1024, budget=0.25)
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


@pytest.mark.parametrize("fetch", [False, True])
def test_sequences_grow_seal_finish_and_are_replaced(fetch: bool) -> None:
    from lazykv_b200 import kernels
    from lazykv_b200.ragged import RaggedTier

    gen = torch.Generator(device="cuda").manual_seed(12)
    tier = RaggedTier(H, G, D, BS, max_seqs=6, max_tokens=1024, store_blocks=256, budget=0.25)
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


def test_ragged_select_rejects_what_it_cannot_hold() -> None:
    from lazykv_b200.ragged import RaggedTier

    with pytest.raises(ValueError, match="tensor-core"):
        RaggedTier(H, G, 128, BS, 2, 1024, 64, 0.25)
    tier = RaggedTier(H, G, D, BS, max_seqs=1, max_tokens=256, store_blocks=8, budget=0.25)
    gen = torch.Generator(device="cuda").manual_seed(13)
    keys, values = _kv(gen, 100)
    tier.add(keys, values)
    with pytest.raises(RuntimeError, match="slots"):
        tier.add(keys, values)
