"""Kernel parity on the GPU, through the C ABI: each kernel against the oracle and the golden vectors.

Bars: int8 records, dequantised values, block metadata, Quest bounds and index lists bit-exact
with the oracle (index lists also equal to the reference's under the tie rule); attention partials
within 1e-5 relative of the float64 oracle (the kernels accumulate in float32).
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

import oracle as O
from tests.golden import inputs as I
from tests.parity import bf16_close, golden, index_parity

pytestmark = pytest.mark.gpu

Q = golden("quant")
S = golden("select")
E = golden("exact")
DEV = "cuda"


def _k():
    from lazykv_b200 import kernels

    return kernels


def _bf16(x: np.ndarray) -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(x, dtype=np.float32)).to(DEV).bfloat16()


def _rel(got: np.ndarray, want: np.ndarray) -> float:
    return float(np.abs(np.asarray(got, np.float64) - want).max() / max(np.abs(want).max(), 1e-30))


# -- codec -------------------------------------------------------------------------------------


@pytest.mark.parametrize("case,bs", [("roundtrip", 64), ("outlier", 64), ("ext", 16)])
def test_pack_matches_the_reference_records_byte_for_byte(case: str, bs: int) -> None:
    x = _bf16(I.from_bf16_np(Q[f"{case}_x"]))  # [n, 2, bs, d]
    rec = _k().pack_int8(x.unsqueeze(1)).squeeze(1).cpu().numpy()
    assert np.array_equal(rec, Q[f"{case}_rec"])


def test_pack_and_unpack_on_the_path_geometry() -> None:
    k = _k()
    lay = I.bf16_layer(seed=11, t=16 * 4)
    pairs = I.pairs_from_kv(lay["k"], lay["v"], 16).to(DEV)  # [4, 8, 2, 16, 64]
    rec = k.pack_int8(pairs)
    assert np.array_equal(rec.cpu().numpy(), Q["g16_rec"])
    flat = rec.reshape(-1, rec.shape[-1])
    assert np.array_equal(k.unpack_int8(flat, 16, 64, torch.float32).cpu().numpy(), Q["g16_f32"])
    got = k.unpack_int8(flat, 16, 64, torch.bfloat16).cpu().view(torch.int16).numpy().view(np.uint16)
    assert np.array_equal(got, Q["g16_bf16"])


def test_float32_pairs_and_constant_groups() -> None:
    k = _k()
    g = torch.Generator().manual_seed(12)
    x32 = torch.randn(16, 2, 16, 64, generator=g)
    assert np.array_equal(k.pack_int8(x32.to(DEV).unsqueeze(1)).squeeze(1).cpu().numpy(), Q["f32_rec"])
    c = torch.full((2, 1, 2, 64, 64), 3.5, dtype=torch.bfloat16, device=DEV)
    rec = k.pack_int8(c)
    assert np.array_equal(rec.squeeze(1).cpu().numpy(), Q["const_rec"])
    assert torch.equal(k.unpack_int8(rec.squeeze(1), 64, 64, torch.bfloat16), c.squeeze(1))


def test_pack_fuses_dequantised_pairs_and_metadata_over_them() -> None:
    k = _k()
    lay = I.bf16_layer(seed=5, t=16 * 40)
    pairs = I.pairs_from_kv(lay["k"], lay["v"], 16).to(DEV)  # [40, 8, 2, 16, 64]
    kmin = torch.full((8, 64, 64), 99.0, dtype=torch.bfloat16, device=DEV)
    kmax = torch.full_like(kmin, -99.0)
    deq = torch.empty_like(pairs)
    rec = k.pack_int8(pairs, kmin=kmin, kmax=kmax, first_block=3, deq=deq)
    want = O.unpack(rec.reshape(-1, rec.shape[-1]).cpu().numpy(), 16, 64, "bfloat16").reshape(40, 8, 2, 16, 64)
    assert np.array_equal(deq.float().cpu().numpy(), want)
    mn, mx = O.block_minmax(want[:, :, 0].transpose(1, 0, 2, 3).reshape(8, -1, 64), 16)
    assert np.array_equal(kmin[:, 3:43].float().cpu().numpy(), mn)
    assert np.array_equal(kmax[:, 3:43].float().cpu().numpy(), mx)
    assert (kmin[:, :3] == 99).all() and (kmin[:, 43:] == 99).all()


def test_fetch_scatters_records_and_pairs_into_slots() -> None:
    k = _k()
    lay = I.bf16_layer(seed=6, t=16 * 10)
    pairs = I.pairs_from_kv(lay["k"], lay["v"], 16).to(DEV)  # [10, 8, ...]
    rec = k.pack_int8(pairs)
    pool = torch.zeros((6, 8, 2, 16, 64), dtype=torch.bfloat16, device=DEV)
    src = torch.tensor([3 * 8 + 1, 7 * 8 + 5, 0 * 8 + 2], dtype=torch.int64, device=DEV)
    dst = torch.tensor([1 * 8 + 1, 4 * 8 + 5, 5 * 8 + 2], dtype=torch.int64, device=DEV)
    k.fetch_pairs(rec.reshape(-1, rec.shape[-1]), src, pool.view(-1, 2, 16, 64), dst, 16, 64)
    deq = k.unpack_int8(rec.reshape(-1, rec.shape[-1]), 16, 64, torch.bfloat16)
    for s, d in zip(src.tolist(), dst.tolist()):
        assert torch.equal(pool.view(-1, 2, 16, 64)[d], deq[s])
    pool2 = torch.zeros_like(pool)
    k.fetch_pairs(pairs.reshape(-1, 2, 16, 64), src, pool2.view(-1, 2, 16, 64), dst, 16, 64)
    for s, d in zip(src.tolist(), dst.tolist()):
        assert torch.equal(pool2.view(-1, 2, 16, 64)[d], pairs.reshape(-1, 2, 16, 64)[s])
    assert (pool2.view(-1, 2, 16, 64)[0] == 0).all()


def test_block_minmax_over_cache_layout() -> None:
    k = _k()
    keys = torch.randn(1, 8, 1000, 64, device=DEV).bfloat16()  # [1, h, T, d] cache layout
    kmin = torch.empty((8, 80, 64), dtype=torch.bfloat16, device=DEV)
    kmax = torch.empty_like(kmin)
    k.block_minmax(keys[0, :, : 62 * 16], 16, kmin, kmax)
    mn, mx = O.block_minmax(keys[0, :, : 62 * 16].float().cpu().numpy(), 16)
    assert np.array_equal(kmin[:, :62].float().cpu().numpy(), mn) and np.array_equal(kmax[:, :62].float().cpu().numpy(), mx)


# -- selection -----------------------------------------------------------------------------------


def test_config1_float32_selection_is_bit_exact() -> None:
    k = _k()
    c1 = I.config1()
    kmin, kmax = O.block_minmax(c1["k"].numpy(), 16)
    n_full = kmin.shape[1] - 1
    dmin, dmax = torch.from_numpy(kmin).to(DEV), torch.from_numpy(kmax).to(DEV)
    words = k.bitmap_words(kmin.shape[1])
    bitmap = torch.full((8, words), -1, dtype=torch.int32, device=DEV)
    idx, bound = k.quest_topk(c1["q"].to(DEV), dmin, dmax, 1, n_full - 1, 126, torch.float32, want_bound=True, bitmap=bitmap)
    want_bound = O.quest_bound(c1["q"].numpy(), kmin[:, 1:n_full], kmax[:, 1:n_full], "float32")
    assert np.array_equal(bound.cpu().numpy(), want_bound)
    want = O.top_blocks(want_bound, 126) + 1
    assert np.array_equal(idx.cpu().numpy(), want)
    par = index_parity(idx.cpu().numpy() - 1, S["config1_idx"] - 1, S["config1_bound"], tie_tol=1e-5)
    assert par["bad"] == 0 and par["exact"] == want.size
    bits = bitmap.cpu().numpy().view(np.uint32)
    for j in range(8):
        got = {b for b in range(words * 32) if (bits[j, b // 32] >> (b % 32)) & 1}
        assert got == set(want[j].tolist())


@pytest.mark.parametrize("case,seed,t", [("bf16", 21, 4096), ("metric", 31, 131072)])
def test_bf16_selection_is_bit_exact_with_the_oracle(case: str, seed: int, t: int) -> None:
    k = _k()
    lay = I.bf16_layer(seed=seed, t=t)
    keys = lay["k"].to(DEV)
    nb = t // 16
    kmin = torch.empty((8, nb, 64), dtype=torch.bfloat16, device=DEV)
    kmax = torch.empty_like(kmin)
    k.block_minmax(keys, 16, kmin, kmax)
    kk = int(S[f"{case}_k"])
    idx, bound = k.quest_topk(lay["q"].to(DEV), kmin, kmax, 1, nb - 2, kk, want_bound=True)
    omin, omax = O.block_minmax(I.to_np(lay["k"]), 16)
    want_bound = O.quest_bound(I.to_np(lay["q"]), omin[:, 1 : nb - 1], omax[:, 1 : nb - 1], "bfloat16")
    assert np.array_equal(bound.cpu().numpy(), want_bound)
    want = O.top_blocks(want_bound, kk) + 1
    assert np.array_equal(idx.cpu().numpy(), want)
    ref_bound = I.from_bf16_np(S[f"{case}_bound"])
    par = index_parity(idx.cpu().numpy() - 1, S[f"{case}_idx"] - 1, ref_bound, tie_tol=np.abs(ref_bound).max() * 2.0**-7)
    assert par["bad"] == 0, par
    # Ascending block-id order: the same set, no sort.
    by_id, _ = k.quest_topk(lay["q"].to(DEV), kmin, kmax, 1, nb - 2, kk, by_block=True)
    assert np.array_equal(by_id.cpu().numpy(), np.sort(want, axis=1))


def test_selection_edge_cases_k_equals_candidates_and_all_ties() -> None:
    k = _k()
    kmin = torch.zeros((2, 40, 16), dtype=torch.bfloat16, device=DEV)
    kmax = torch.zeros_like(kmin)
    q = torch.randn(8, 16, device=DEV).bfloat16()
    idx, _ = k.quest_topk(q, kmin, kmax, 1, 30, 30)
    assert idx.cpu().tolist() == [list(range(1, 31))] * 2  # every bound ties: ascending ids
    idx, _ = k.quest_topk(q, kmin, kmax, 1, 30, 7)
    assert idx.cpu().tolist() == [list(range(1, 8))] * 2


# -- attention -------------------------------------------------------------------------------------


def _config1_pool() -> tuple[dict, torch.Tensor]:
    c1 = I.config1()
    k, v = c1["k"], c1["v"]
    pool = I.pairs_from_kv(k, v, 16).to(DEV)  # [512, 8, 2, 16, 64] fp32, block id = slot
    return c1, pool


def test_config1_hot_and_cold_partials_match_the_reference() -> None:
    kern = _k()
    c1, pool = _config1_pool()
    sel = torch.from_numpy(S["config1_idx"].astype(np.int32)).to(DEV)
    blocks = torch.cat([torch.zeros((8, 1), dtype=torch.int32, device=DEV), sel, torch.full((8, 1), 511, dtype=torch.int32, device=DEV)], 1)
    strides = (8 * 2 * 16 * 64, 2 * 16 * 64, 64)
    q = c1["q"].to(DEV)
    out, lse = kern.hot_attention(q, pool, pool[:, :, 1], strides, blocks.contiguous(), 16, 64**-0.5, 16)
    assert _rel(out.view(8, 4, 64).cpu().numpy(), E["config1_hot_out"]) < 1e-5
    assert _rel(lse.view(8, 4).cpu().numpy(), E["config1_hot_lse"]) < 1e-6
    words = kern.bitmap_words(512)
    bitmap = torch.zeros((8, words), dtype=torch.int32, device=DEV)
    bm = np.zeros((8, words), np.uint32)
    for j in range(8):
        for b in S["config1_idx"][j].tolist() + [511]:
            bm[j, b // 32] |= np.uint32(1 << (b % 32))
    bitmap.copy_(torch.from_numpy(bm.view(np.int32)))
    cout, clse = kern.cold_attention(q, pool, 16, 1, 511, 64**-0.5, excluded=bitmap)
    assert _rel(cout.view(8, 4, 64).cpu().numpy(), E["config1_cold_out"]) < 1e-5
    assert _rel(clse.view(8, 4).cpu().numpy(), E["config1_cold_lse"]) < 1e-6
    merged, mlse = kern.lse_merge(torch.stack([out, cout]), torch.stack([lse, clse]))
    assert _rel(merged.view(8, 4, 64).cpu().numpy(), E["config1_out"]) < 1e-5
    want, _ = O.dense_attention(c1["q"].numpy(), c1["k"].numpy(), c1["v"].numpy(), 64**-0.5)
    assert _rel(merged.cpu().numpy(), want) < 1e-5


def test_empty_cold_set_and_empty_partials_merge_cleanly() -> None:
    kern = _k()
    q = torch.randn(8, 64, device=DEV)
    pool = torch.randn(4, 2, 2, 16, 64, device=DEV)
    words = 1
    allset = torch.full((2, words), -1, dtype=torch.int32, device=DEV)
    out, lse = kern.cold_attention(q, pool, 16, 1, 3, 0.125, excluded=allset)
    assert torch.isneginf(lse).all() and (out == 0).all()
    out0, lse0 = kern.cold_attention(q, pool, 16, 1, 0, 0.125)
    assert torch.isneginf(lse0).all() and (out0 == 0).all()
    full, flse = kern.cold_attention(q, pool, 16, 0, 4, 0.125)
    merged, mlse = kern.lse_merge(torch.stack([full, out]), torch.stack([flse, lse]))
    assert torch.allclose(merged, full, atol=1e-6) and torch.allclose(mlse, flse)
    both, blse = kern.lse_merge(torch.stack([out, out0]), torch.stack([lse, lse0]))
    assert (both == 0).all() and torch.isneginf(blse).all()


def test_merge_matches_the_reference_weights() -> None:
    kern = _k()
    outs = torch.tensor([[[1.0, 0.0]], [[0.0, 1.0]]], device=DEV)
    lses = torch.tensor([[2.0], [0.0]], device=DEV)
    out, lse = kern.lse_merge(outs, lses)
    np.testing.assert_allclose(out.cpu().numpy(), E["weights_out"], rtol=1e-6)
    np.testing.assert_allclose(lse.cpu().numpy(), E["weights_lse"], rtol=1e-6)


@pytest.mark.parametrize("fill", [1, 9, 16])
def test_int8_exact_step_matches_the_oracle_composition(fill: int) -> None:
    """The north-star layer step from kernels: pack -> select -> hot + cold -> merge."""
    kern = _k()
    lay = I.bf16_layer(seed=41, t=4096 + 9)
    n = 256
    pairs = I.pairs_from_kv(lay["k"], lay["v"], 16).to(DEV)  # [256, 8, 2, 16, 64]
    cur = torch.zeros((8, 2, 16, 64), dtype=torch.bfloat16, device=DEV)
    tail = torch.stack([lay["k"][:, n * 16 :], lay["v"][:, n * 16 :]], 1).to(DEV)  # [8, 2, 9, 64]
    live = min(fill, 9)
    cur[:, :, :live] = tail[:, :, :live]
    if fill > 9:
        cur[:, :, 9:fill] = torch.randn(8, 2, fill - 9, 64, generator=torch.Generator().manual_seed(fill)).bfloat16().to(DEV)
    kmin = torch.empty((8, n, 64), dtype=torch.bfloat16, device=DEV)
    kmax = torch.empty_like(kmin)
    deq = torch.empty_like(pairs)
    rec = kern.pack_int8(pairs, kmin=kmin, kmax=kmax, deq=deq)
    deq[0] = pairs[0]  # the sink stays exact
    kk = int(E["int8_k"])
    words = kern.bitmap_words(n + 1)
    bitmap = torch.zeros((8, words), dtype=torch.int32, device=DEV)
    q = lay["q"].to(DEV)
    sel, _ = kern.quest_topk(q, kmin, kmax, 1, n - 1, kk, bitmap=bitmap)
    pool = torch.cat([deq, cur[None]], 0)  # slot = block id; block n is the current block
    blocks = torch.cat([torch.zeros((8, 1), dtype=torch.int32, device=DEV), sel, torch.full((8, 1), n, dtype=torch.int32, device=DEV)], 1).contiguous()
    strides = (8 * 2 * 16 * 64, 2 * 16 * 64, 64)
    hot, hlse = kern.hot_attention(q, pool, pool[:, :, 1], strides, blocks, fill, 64**-0.5, 16)
    cold, clse = kern.cold_attention(q, rec, 16, 1, n - 1, 64**-0.5, excluded=bitmap)
    out32, lse = kern.lse_merge(torch.stack([hot, cold]), torch.stack([hlse, clse]))
    out, _ = kern.lse_merge(torch.stack([hot, cold]), torch.stack([hlse, clse]), torch.bfloat16)
    r = O.tiered_decode(I.to_np(lay["q"]), I.to_np(pairs.cpu()), I.to_np(cur.cpu()), fill, kk, 64**-0.5, "bfloat16", "int8")
    assert np.array_equal(sel.cpu().numpy(), r["selected"])
    assert _rel(hot.view(8, 4, 64).cpu().numpy(), r["hot_out"]) < 1e-5
    assert _rel(cold.view(8, 4, 64).cpu().numpy(), r["cold_out"]) < 1e-5
    assert _rel(lse.view(8, 4).cpu().numpy(), r["lse"]) < 1e-5
    # The merged output before its cast is within 1e-5 of the float64 composition; the bf16 output
    # is that value rounded, so it is within half a bf16 unit plus that tolerance of the composition
    # (bf16 rounding alone is up to 2^-8 relative, so a plain relative bar on it would test the format).
    assert _rel(out32.view(8, 4, 64).cpu().numpy(), r["out"]) < 1e-5
    assert bf16_close(out.float().view(8, 4, 64).cpu().numpy(), r["out"])
    if fill == 9:
        assert _rel(out32.view(8, 4, 64).cpu().numpy(), E["int8_out"]) < 2e-3


@pytest.mark.parametrize("n_cand", [1, 7, 100, 511, 513, 2000, 8190, 20000, 65536])
@pytest.mark.parametrize("bound", ["bf16", "f32"])
def test_cluster_select_matches_the_sorting_select(n_cand: int, bound: str) -> None:
    """Ascending-id selection (one thread-block cluster per KV head, scores and radix passes fused)
    against the single-CTA select with its descending sort: the same set for every k, including
    ties (coarsely quantised metadata makes many bounds equal) and a first-block offset; and the
    bitmap marks exactly that set."""
    k = _k()
    h, g, d, first = 8, 4, 64, 3
    gen = torch.Generator(device=DEV).manual_seed(n_cand)
    dt = torch.bfloat16 if bound == "bf16" else torch.float32
    base = torch.randn((h, first + n_cand, d), generator=gen, device=DEV)
    base = (base * 2).round() / 2  # coarse values: many exactly tied bounds
    kmin = (base - 0.5).to(dt)
    kmax = (base + 0.5).to(dt)
    q = torch.randn((h * g, d), generator=gen, device=DEV).to(dt)
    words = k.bitmap_words(first + n_cand + 1)
    if n_cand > 16384:  # beyond the sorting select's capacity: k = n_cand must return every id
        got, _ = k.quest_topk(q, kmin, kmax, first, n_cand, n_cand, by_block=True)
        assert np.array_equal(got.cpu().numpy(), np.tile(np.arange(first, first + n_cand), (h, 1)))
    for kk in sorted({1, max(1, n_cand // 4), max(1, n_cand - 1), n_cand} & set(range(1, 16385))):
        ref, _ = k.quest_topk(q, kmin, kmax, first, n_cand, kk)
        bm = torch.full((h, words), -1, dtype=torch.int32, device=DEV)
        got, _ = k.quest_topk(q, kmin, kmax, first, n_cand, kk, bitmap=bm, by_block=True)
        want = np.sort(ref.cpu().numpy(), axis=1)
        assert np.array_equal(got.cpu().numpy(), want), (kk, n_cand)
        bits = np.unpackbits(bm.cpu().numpy().view(np.uint8), bitorder="little").reshape(h, -1)
        for j in range(h):
            assert np.array_equal(np.nonzero(bits[j])[0], want[j])
    assert k.device_status() == 0


@pytest.mark.parametrize("d", [16, 32, 64, 128])
@pytest.mark.parametrize("dt", [torch.bfloat16, torch.float32])
@pytest.mark.parametrize("order", ["bound", "block"])
def test_bounds_and_selection_every_head_dim(d: int, dt: torch.dtype, order: str) -> None:
    """The scoring kernels stage metadata rows of d channels in shared memory (rotated 16-byte
    chunks); every head_dim the ABI takes, bounds bit-exact with the oracle and the selected set the
    oracle's, through both selects."""
    k = _k()
    h, g, n, kk = 4, 4, 300, 37
    gen = torch.Generator(device=DEV).manual_seed(d)
    kmin = torch.randn((h, n + 1, d), generator=gen, device=DEV).to(dt)
    kmax = (kmin.float() + torch.rand((h, n + 1, d), generator=gen, device=DEV)).to(dt)
    q = torch.randn((h * g, d), generator=gen, device=DEV).to(dt)
    mode = "bfloat16" if dt == torch.bfloat16 else "float32"
    want_bound = O.quest_bound(I.to_np(q), I.to_np(kmin[:, 1:]), I.to_np(kmax[:, 1:]), mode)
    idx, bound = k.quest_topk(q, kmin, kmax, 1, n, kk, want_bound=True, by_block=order == "block")
    assert np.array_equal(bound.cpu().numpy(), want_bound.astype(np.float32))  # exact (+0 and -0 compare equal)
    want = O.top_blocks(want_bound, kk) + 1
    got = idx.cpu().numpy()
    assert np.array_equal(np.sort(got, 1), np.sort(want, 1))
    if order == "bound":
        assert np.array_equal(got, want)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
@pytest.mark.parametrize("t,fill", [(1, 0), (1, 15), (5, 3), (16, 0)])
def test_append_tokens_writes_both_halves_at_the_fill(dtype: torch.dtype, t: int, fill: int) -> None:
    """lkv_append_tokens: keys / values [h, T, d] (strided views) land at token positions fill ..
    fill + T - 1 of the slot's two halves; nothing else in the pool changes."""
    from lazykv_b200 import kernels as K
    from lazykv_b200._lib import LkvError

    h, bs, d = 8, 16, 64
    gen = torch.Generator(device=DEV).manual_seed(t * 100 + fill)
    pool = torch.randn((4, h, 2, bs, d), generator=gen, device=DEV).to(dtype)
    kv = torch.randn((2, 1, h, t + 2, d), generator=gen, device=DEV).to(dtype)
    keys, values = kv[0, 0, :, 1 : t + 1], kv[1, 0, :, 2 : t + 2]  # [h, T, d], token stride d, head stride (t + 2) d
    want = pool.clone()
    want[2, :, 0, fill : fill + t] = keys
    want[2, :, 1, fill : fill + t] = values
    K.append_tokens(keys, values, pool[2], fill)
    assert torch.equal(pool, want)
    with pytest.raises(LkvError):  # past the end of the block
        K.append_tokens(keys, values, pool[2], bs - t + 1)
