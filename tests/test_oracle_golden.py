"""Pin the CPU oracle to the reference: golden vectors from the reference's own functions.

The fixtures were written by `tests/golden/make_golden.py`, which ran lazykv.quant, lazykv.selection
and lazykv.exact on the seeded inputs of `tests/golden/inputs.py`. These tests regenerate the
inputs, run the oracle, and require bit-exact int8 records and dequantised values, the reference's
Quest bounds to within the accumulation-order rounding, index lists equal under the tie rule, and
merged attention within the float32 bar.
"""

from __future__ import annotations

import hashlib

import numpy as np
import pytest
import torch

import oracle as O
from tests.golden import inputs as I
from tests.parity import bf16_ulp_diff, f32_ulp_diff, golden, index_parity

Q = golden("quant")
S = golden("select")
E = golden("exact")


# -- int8 codec: lazykv/quant.py ---------------------------------------------------------------


def test_record_widths_match_the_reference() -> None:
    assert O.packed_pair_bytes(16, 64) == int(Q["width_16_64"]) == 2368
    assert O.packed_pair_bytes(64, 64) == int(Q["width_64_64"]) == 8704


@pytest.mark.parametrize("case", ["roundtrip", "outlier"])
def test_pack_is_byte_exact_on_the_reference_cases(case: str) -> None:
    x = I.from_bf16_np(Q[f"{case}_x"])
    assert np.array_equal(O.pack(x), Q[f"{case}_rec"])


def test_roundtrip_and_constant_group_dequantise_bit_exactly() -> None:
    rec = Q["roundtrip_rec"]
    assert np.array_equal(O.bf16_bits(O.unpack(rec, 64, 64, "bfloat16")), Q["roundtrip_bf16"])
    x = np.full((2, 2, 64, 64), 3.5, dtype=np.float32)
    assert np.array_equal(O.pack(x), Q["const_rec"])
    back = O.unpack(O.pack(x).reshape(2, -1), 64, 64, "bfloat16")
    assert np.array_equal(O.bf16_bits(back), Q["const_back"]) and np.all(back == 3.5)


def test_path_geometry_records_and_both_dequantised_dtypes_are_exact() -> None:
    lay = I.bf16_layer(seed=11, t=16 * 4)
    pairs = I.pairs_from_kv(lay["k"], lay["v"], 16)
    assert np.allclose(I.checksum(pairs), Q["g16_checksum"])
    rec = O.pack(I.to_np(pairs))
    assert np.array_equal(rec, Q["g16_rec"])
    flat = rec.reshape(-1, rec.shape[-1])
    assert np.array_equal(O.unpack(flat, 16, 64, "float32"), Q["g16_f32"])
    assert np.array_equal(O.bf16_bits(O.unpack(flat, 16, 64, "bfloat16")), Q["g16_bf16"])


def test_float32_input_and_extreme_ranges_are_exact() -> None:
    g = torch.Generator().manual_seed(12)
    x32 = torch.randn(16, 2, 16, 64, generator=g)
    assert np.allclose(I.checksum(x32), Q["f32_checksum"])
    assert np.array_equal(O.pack(x32.numpy()), Q["f32_rec"])
    ext = I.from_bf16_np(Q["ext_x"])
    assert np.array_equal(O.pack(ext), Q["ext_rec"])
    assert np.array_equal(O.bf16_bits(O.unpack(Q["ext_rec"], 16, 64, "bfloat16")), Q["ext_bf16"])


def test_codec_validation_matches_the_reference_messages() -> None:
    with pytest.raises(ValueError, match="uint8 records"):
        O.unpack(np.zeros((2, 7), np.uint8), 64, 64, "bfloat16")
    with pytest.raises(ValueError, match="KV pair"):
        O.pack(np.zeros((3, 3, 64, 64), np.float32))


# -- selection: lazykv/selection.py --------------------------------------------------------------


def _config1_meta() -> tuple[np.ndarray, np.ndarray, np.ndarray, int]:
    c1 = I.config1()
    assert np.allclose(np.concatenate([I.checksum(c1[k]) for k in ("k", "v", "q")]), S["config1_checksum"])
    kmin, kmax = O.block_minmax(c1["k"].numpy(), I.BS)
    n_full = kmin.shape[1] - 1
    return c1["q"].numpy(), kmin[:, 1:n_full], kmax[:, 1:n_full], int(S["config1_k"])


def test_blocks_for_budget_is_the_reference_rule() -> None:
    assert O.blocks_for_budget(0.25, 8192, 16) == int(S["config1_k"]) == 126
    assert O.blocks_for_budget(0.25, 131072, 16) == int(S["metric_k"]) == 2046
    for frac in (0.75, 0.25, 0.0625):
        assert (O.blocks_for_budget(frac, 32768, 64) + 2) * 64 <= frac * 32768


def test_config1_float32_bounds_and_indices_match_the_reference() -> None:
    q, kmin, kmax, k = _config1_meta()
    bound = O.quest_bound(q, kmin, kmax, "float32")
    # Same math, different float32 summation order (BLAS): a few units in the last place at most.
    assert f32_ulp_diff(bound, S["config1_bound"]).max() <= 64
    ours = O.top_blocks(bound, k) + 1
    par = index_parity(ours - 1, S["config1_idx"] - 1, S["config1_bound"], tie_tol=1e-5)
    assert par["bad"] == 0, par
    assert par["exact"] == ours.size  # no ties in float32 on this input


@pytest.mark.parametrize("case", ["bf16", "metric"])
def test_bf16_bounds_and_indices_match_the_reference(case: str) -> None:
    t = 4096 if case == "bf16" else 131072
    lay = I.bf16_layer(seed=21 if case == "bf16" else 31, t=t)
    names = ("k", "v", "q") if case == "bf16" else ("k", "q")
    assert np.allclose(np.concatenate([I.checksum(lay[x]) for x in names]), S[f"{case}_checksum"])
    kmin, kmax = O.block_minmax(I.to_np(lay["k"]), I.BS)
    nb = kmin.shape[1]
    bound = O.quest_bound(I.to_np(lay["q"]), kmin[:, 1 : nb - 1], kmax[:, 1 : nb - 1], "bfloat16")
    ref_bound = I.from_bf16_np(S[f"{case}_bound"])
    ulp = bf16_ulp_diff(bound, ref_bound)
    assert ulp.max() <= 1 and (ulp > 0).mean() < 0.01, (ulp.max(), (ulp > 0).mean())
    k = int(S[f"{case}_k"])
    ours = O.top_blocks(bound, k) + 1
    # bf16 bounds tie often (the reference measured ties at the K-th bound in most cells), and a
    # one-ulp rounding difference moves a block across the K-th bound: both are ties here.
    kth_ulp = np.abs(ref_bound).max() * 2.0**-7
    par = index_parity(ours - 1, S[f"{case}_idx"] - 1, ref_bound, tie_tol=kth_ulp)
    assert par["bad"] == 0, par
    if case == "bf16":
        b32 = O.quest_bound(I.to_np(lay["q"]), kmin[:, 1 : nb - 1], kmax[:, 1 : nb - 1], "float32")
        assert f32_ulp_diff(b32, S["bf16_bound_f32"]).max() <= 64
        ours32 = O.top_blocks(b32, k) + 1
        par = index_parity(ours32 - 1, S["bf16_idx_f32"] - 1, S["bf16_bound_f32"], tie_tol=1e-5)
        assert par["bad"] == 0, par


def test_float32_bound_breaks_the_bf16_tie_as_the_reference_does() -> None:
    q = np.ones((1, 2), np.float32)
    kt = np.array([[[256.0, 0.5], [256.0, 1.0]]], np.float32)
    b16 = O.quest_bound(q, kt, kt, "bfloat16")
    assert np.array_equal(b16, I.from_bf16_np(S["tie_bound_bf16"])) and b16[0, 0] == b16[0, 1]
    b32 = O.quest_bound(q, kt, kt, "float32")
    assert np.array_equal(b32, S["tie_bound_f32"])
    assert O.top_blocks(b32, 1)[0, 0] == S["tie_top1_f32"][0, 0] == 1
    # The tie rule on the bf16 tie: lower block id first.
    assert O.top_blocks(b16, 2)[0].tolist() == [0, 1]


def test_quest_bound_dominates_every_dot_product() -> None:
    rng = np.random.default_rng(3)
    q = rng.standard_normal((8, 16)).astype(np.float32)
    keys = rng.standard_normal((2, 10, 8, 16)).astype(np.float32)
    kmin, kmax = keys.min(2), keys.max(2)
    bound = O.quest_bound(q, kmin, kmax, "float32")
    exact = np.einsum("hgd,hntd->hgnt", q.reshape(2, 4, 16), keys).max(-1).max(1)
    assert (bound >= exact - 1e-5).all()


# -- exact merge: lazykv/exact.py ------------------------------------------------------------------


def test_merge_algebra_matches_the_reference() -> None:
    k, v, q = E["halves_k"], E["halves_v"], E["halves_q"]
    first = np.tile(np.arange(0, 2), (3, 1))
    second = np.tile(np.arange(2, 6), (3, 1))
    oa, la = O.cpu_partial_attention(k, v, q, 16**-0.5, 8, second)
    ob, lb = O.cpu_partial_attention(k, v, q, 16**-0.5, 8, first)
    np.testing.assert_allclose(oa, E["halves_oa"], rtol=1e-5, atol=1e-6)
    np.testing.assert_allclose(la, E["halves_la"], rtol=1e-6)
    out, lse = O.merge_lse(oa, la, ob, lb)
    np.testing.assert_allclose(out, E["halves_out"], rtol=1e-5, atol=1e-6)
    want, _ = O.dense_attention(q.reshape(-1, 16), k, v, 16**-0.5)
    np.testing.assert_allclose(O.merge_lse(*O.cpu_partial_attention(k, v, q, 16**-0.5, 8, second, np.float64), *O.cpu_partial_attention(k, v, q, 16**-0.5, 8, first, np.float64))[0].reshape(-1, 16), want, atol=1e-10)


def test_merge_weights_and_empty_partials() -> None:
    out, lse = O.merge_lse(np.array([[1.0, 0.0]], np.float32), np.array([2.0], np.float32), np.array([[0.0, 1.0]], np.float32), np.array([0.0], np.float32))
    np.testing.assert_allclose(out, E["weights_out"], rtol=1e-6)
    np.testing.assert_allclose(lse, E["weights_lse"], rtol=1e-6)
    out, lse = O.merge_lse(np.zeros((2, 3), np.float32), np.full(2, -np.inf, np.float32), np.ones((2, 3), np.float32), np.full(2, -np.inf, np.float32))
    assert np.array_equal(out, E["empty_out"]) and np.all(np.isneginf(lse)) and np.isfinite(out).all()
    keys = np.random.default_rng(1).standard_normal((2, 32, 8)).astype(np.float32)
    o, l = O.cpu_partial_attention(keys, keys, keys[:, :2], 8**-0.5, 8, np.tile(np.arange(4), (2, 1)))
    assert np.isneginf(l).all() and np.isfinite(o).all()


def test_config1_composition_matches_the_reference_in_float32() -> None:
    c1 = I.config1()
    k, v, q = c1["k"].numpy(), c1["v"].numpy(), c1["q"].numpy()
    n = 511
    sealed = np.stack([k[:, : n * 16], v[:, : n * 16]], 1).reshape(8, 2, n, 16, 64).transpose(2, 0, 1, 3, 4)
    current = np.stack([k[:, n * 16 :], v[:, n * 16 :]], 1)
    r = O.tiered_decode(q, sealed, current, 16, 126, 64**-0.5, model_dtype="float32", quant=None)
    par = index_parity(r["selected"] - 1, S["config1_idx"] - 1, S["config1_bound"], tie_tol=1e-5)
    assert par["bad"] == 0 and par["exact"] == r["selected"].size
    for part in ("hot", "cold"):
        np.testing.assert_allclose(r[f"{part}_out"], E[f"config1_{part}_out"], rtol=1e-5, atol=2e-6)
        np.testing.assert_allclose(r[f"{part}_lse"], E[f"config1_{part}_lse"], rtol=1e-6)
    np.testing.assert_allclose(r["out"], E["config1_out"], rtol=1e-5, atol=2e-6)
    # The merge is exact: it equals dense attention over the whole context.
    want, _ = O.dense_attention(q, k, v, 64**-0.5)
    np.testing.assert_allclose(r["out"].reshape(-1, 64), want, atol=1e-10)


def test_int8_exact_composition_matches_the_reference_composition() -> None:
    lay = I.bf16_layer(seed=41, t=4096 + 9)
    assert np.allclose(np.concatenate([I.checksum(lay[x]) for x in ("k", "v", "q")]), E["int8_checksum"])
    n, fill = 256, int(E["int8_fill"])
    pairs = I.to_np(I.pairs_from_kv(lay["k"], lay["v"], 16))
    cur = np.zeros((8, 2, 16, 64), np.float32)
    cur[:, 0, :fill] = I.to_np(lay["k"][:, n * 16 :])
    cur[:, 1, :fill] = I.to_np(lay["v"][:, n * 16 :])
    r = O.tiered_decode(I.to_np(lay["q"]), pairs, cur, fill, int(E["int8_k"]), 64**-0.5, "bfloat16", "int8")
    assert hashlib.sha256(r["records"].tobytes()).digest() == E["int8_rec_sha"].tobytes()
    ref_bound = I.from_bf16_np(E["int8_bound"])
    assert bf16_ulp_diff(O.quest_bound(I.to_np(lay["q"]), r["kmin"][:, 1:n], r["kmax"][:, 1:n]), ref_bound).max() <= 1
    par = index_parity(r["selected"] - 1, E["int8_idx"] - 1, ref_bound, tie_tol=np.abs(ref_bound).max() * 2.0**-7)
    assert par["bad"] == 0, par
    # Composed with the reference's own choice among tied blocks, the partials match in float32.
    r = O.tiered_decode(I.to_np(lay["q"]), pairs, cur, fill, int(E["int8_k"]), 64**-0.5, "bfloat16", "int8", selected=E["int8_idx"])
    for part in ("hot", "cold"):
        np.testing.assert_allclose(r[f"{part}_out"], E[f"int8_{part}_out"], rtol=1e-5, atol=2e-6)
        np.testing.assert_allclose(r[f"{part}_lse"], E[f"int8_{part}_lse"], rtol=1e-6)
    np.testing.assert_allclose(r["out"], E["int8_out"], rtol=1e-5, atol=2e-6)
    np.testing.assert_allclose(r["lse"], E["int8_lse"], rtol=1e-6)
