"""Generate golden vectors by running the reference's own hot-path functions on seeded inputs.

Run where the reference is importable (it is Python; nothing is built):

    python tests/golden/make_golden.py /path/to/LazyKV

It imports `lazykv.selection`, `lazykv.quant` and `lazykv.exact` from that tree, runs them on the
inputs of `tests/golden/inputs.py`, and writes the outputs to `tests/golden/*.npz`. The GPU box
never runs this script: the fixtures it wrote are committed.
"""

from __future__ import annotations

import math
import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parents[1]))

from tests.golden import inputs as I  # noqa: E402


def main(ref_root: str) -> None:
    sys.path.insert(0, ref_root)
    from lazykv.exact import cpu_partial_attention, merge_lse
    from lazykv.quant import pack, packed_pair_bytes, unpack
    from lazykv.selection import blocks_for_budget, quest_bound, top_blocks

    torch.set_num_threads(8)
    out: dict[str, dict[str, np.ndarray]] = {"quant": {}, "select": {}, "exact": {}}

    # ---- int8 codec (lazykv/quant.py), including the cases tests/test_quant.py pins ----------
    q = out["quant"]
    q["width_16_64"] = np.array(packed_pair_bytes(16, 64))
    q["width_64_64"] = np.array(packed_pair_bytes(64, 64))
    torch.manual_seed(0)
    x = torch.randn(4, 2, 64, 64, dtype=torch.bfloat16) * 3  # test_quant.py:36-46
    q["roundtrip_x"] = I.bf16_np(x)
    q["roundtrip_rec"] = pack(x).numpy()
    q["roundtrip_bf16"] = I.bf16_np(unpack(pack(x), 64, 64, torch.bfloat16))
    torch.manual_seed(0)
    x = torch.randn(1, 2, 64, 64, dtype=torch.bfloat16)
    x[0, 0, :, 0] *= 500  # test_quant.py:49-56
    q["outlier_x"] = I.bf16_np(x)
    q["outlier_rec"] = pack(x).numpy()
    x = torch.full((2, 2, 64, 64), 3.5, dtype=torch.bfloat16)  # test_quant.py:59-62
    q["const_rec"] = pack(x).numpy()
    q["const_back"] = I.bf16_np(unpack(pack(x), 64, 64, torch.bfloat16))
    # The path's geometry (bs 16, d 64), bf16, with the key offset: 4 blocks x 8 heads = 32 pairs.
    lay = I.bf16_layer(seed=11, t=16 * 4)
    pairs = I.pairs_from_kv(lay["k"], lay["v"], 16)  # [4, 8, 2, 16, 64]
    q["g16_checksum"] = I.checksum(pairs)
    q["g16_rec"] = pack(pairs).numpy()
    q["g16_f32"] = unpack(pack(pairs).flatten(0, 1), 16, 64, torch.float32).numpy()
    q["g16_bf16"] = I.bf16_np(unpack(pack(pairs).flatten(0, 1), 16, 64, torch.bfloat16))
    # float32 input (config 1's cache dtype) and extreme ranges.
    g = torch.Generator().manual_seed(12)
    x32 = torch.randn(16, 2, 16, 64, generator=g)
    q["f32_checksum"] = I.checksum(x32)
    q["f32_rec"] = pack(x32).numpy()
    ext = torch.randn(4, 2, 16, 64, generator=g)
    ext[0] *= 2.0e4
    ext[1] *= 1.0e-30
    ext[2, :, :, 5] = 7.0
    ext[3, 1, 3] = -2.5
    ext = ext.bfloat16()
    q["ext_x"] = I.bf16_np(ext)
    q["ext_rec"] = pack(ext).numpy()
    q["ext_bf16"] = I.bf16_np(unpack(pack(ext), 16, 64, torch.bfloat16))

    # ---- selection (lazykv/selection.py) ------------------------------------------------------
    s = out["select"]
    c1 = I.config1()
    s["config1_checksum"] = np.concatenate([I.checksum(c1[k]) for k in ("k", "v", "q")])
    bs = I.BS
    nb = c1["k"].shape[1] // bs
    n_full = nb - 1  # the last block is full and is the current block (selection.py:153-158)
    kb = c1["k"].view(I.HKV, nb, bs, I.D)
    kmin, kmax = kb.amin(2)[None], kb.amax(2)[None]
    k1 = blocks_for_budget(0.25, c1["k"].shape[1], bs)
    qq = c1["q"].view(1, I.HQ, 1, I.D)
    s["config1_k"] = np.array(k1)
    s["config1_bound"] = quest_bound(qq, kmin[:, :, 1:n_full], kmax[:, :, 1:n_full])[0].numpy()
    s["config1_idx"] = (top_blocks(qq, kmin[:, :, 1:n_full], kmax[:, :, 1:n_full], k1) + 1)[0].numpy()
    # bf16 layer, 4,096 tokens (config 2's shapes, one layer): bound in bf16 and in float32.
    lay = I.bf16_layer(seed=21, t=4096)
    s["bf16_checksum"] = np.concatenate([I.checksum(lay[k]) for k in ("k", "v", "q")])
    nb = 4096 // bs
    kb = lay["k"].view(I.HKV, nb, bs, I.D)
    kmin, kmax = kb.amin(2)[None], kb.amax(2)[None]
    kk = blocks_for_budget(0.25, 4096, bs)
    qq = lay["q"].view(1, I.HQ, 1, I.D)
    s["bf16_k"] = np.array(kk)
    s["bf16_bound"] = I.bf16_np(quest_bound(qq, kmin[:, :, 1 : nb - 1], kmax[:, :, 1 : nb - 1])[0])
    s["bf16_idx"] = (top_blocks(qq, kmin[:, :, 1 : nb - 1], kmax[:, :, 1 : nb - 1], kk) + 1)[0].numpy()
    s["bf16_bound_f32"] = quest_bound(qq, kmin[:, :, 1 : nb - 1], kmax[:, :, 1 : nb - 1], torch.float32)[0].numpy()
    s["bf16_idx_f32"] = (top_blocks(qq, kmin[:, :, 1 : nb - 1], kmax[:, :, 1 : nb - 1], kk, torch.float32) + 1)[0].numpy()
    # The metric geometry's candidate count (8,190 per head at 128K), bf16, selection only.
    lay = I.bf16_layer(seed=31, t=131072)
    nb = 131072 // bs
    kb = lay["k"].view(I.HKV, nb, bs, I.D)
    kmin, kmax = kb.amin(2)[None], kb.amax(2)[None]
    kk = blocks_for_budget(0.25, 131072, bs)
    qq = lay["q"].view(1, I.HQ, 1, I.D)
    s["metric_checksum"] = np.concatenate([I.checksum(lay[k]) for k in ("k", "q")])
    s["metric_k"] = np.array(kk)
    s["metric_bound"] = I.bf16_np(quest_bound(qq, kmin[:, :, 1 : nb - 1], kmax[:, :, 1 : nb - 1])[0])
    s["metric_idx"] = (top_blocks(qq, kmin[:, :, 1 : nb - 1], kmax[:, :, 1 : nb - 1], kk) + 1)[0].numpy()
    # test_selection.py:121-132: float32 breaks a bf16 tie.
    qt = torch.ones((1, 1, 1, 2), dtype=torch.bfloat16)
    kt = torch.tensor([[[[256.0, 0.5], [256.0, 1.0]]]], dtype=torch.bfloat16)
    s["tie_bound_bf16"] = I.bf16_np(quest_bound(qt, kt, kt)[0])
    s["tie_bound_f32"] = quest_bound(qt, kt, kt, torch.float32)[0].numpy()
    s["tie_top1_f32"] = top_blocks(qt, kt, kt, 1, torch.float32)[0].numpy()

    # ---- exact merge (lazykv/exact.py) -----------------------------------------------------------
    e = out["exact"]
    torch.manual_seed(0)  # test_exact.py:32-49
    h, groups, n_blocks, d, b8 = 3, 2, 6, 16, 8
    keys, values, query = torch.randn(h, n_blocks * b8, d), torch.randn(h, n_blocks * b8, d), torch.randn(h, groups, d)
    first = np.tile(np.arange(0, 2), (h, 1))
    second = np.tile(np.arange(2, n_blocks), (h, 1))
    oa, la = cpu_partial_attention(keys, values, query, d**-0.5, b8, excluded=second)
    ob, lb = cpu_partial_attention(keys, values, query, d**-0.5, b8, excluded=first)
    mo, ml = merge_lse(oa, la, ob, lb)
    for name, t in (("halves_k", keys), ("halves_v", values), ("halves_q", query), ("halves_oa", oa), ("halves_la", la), ("halves_ob", ob), ("halves_lb", lb), ("halves_out", mo), ("halves_lse", ml)):
        e[name] = t.numpy()
    # merge weights: test_exact.py:72-84
    mo, ml = merge_lse(torch.tensor([[1.0, 0.0]]), torch.tensor([2.0]), torch.tensor([[0.0, 1.0]]), torch.tensor([0.0]))
    e["weights_out"], e["weights_lse"] = mo.numpy(), ml.numpy()
    # both empty
    mo, ml = merge_lse(torch.zeros(2, 3), torch.full((2,), float("-inf")), torch.ones(2, 3), torch.full((2,), float("-inf")))
    e["empty_out"], e["empty_lse"] = mo.numpy(), ml.numpy()

    # Config 1 composed end to end from the reference's functions (fp32, bs 16).
    k, v, qv = c1["k"], c1["v"], c1["q"]
    nb = k.shape[1] // bs
    n_full = nb - 1
    sel = s["config1_idx"]  # [8, 126], block ids
    scale = I.D**-0.5
    hot = np.concatenate([np.zeros((I.HKV, 1), np.int64), sel, np.full((I.HKV, 1), n_full)], axis=1)
    rest = np.array([[b for b in range(nb) if b not in set(hot[j].tolist())] for j in range(I.HKV)])
    qg = qv.view(I.HKV, I.HQ // I.HKV, I.D)
    ho, hl = cpu_partial_attention(k, v, qg, scale, bs, rest)
    co, cl = cpu_partial_attention(k, v, qg, scale, bs, hot)
    mo, ml = merge_lse(ho, hl, co, cl)
    e["config1_hot_out"], e["config1_hot_lse"] = ho.numpy(), hl.numpy()
    e["config1_cold_out"], e["config1_cold_lse"] = co.numpy(), cl.numpy()
    e["config1_out"], e["config1_lse"] = mo.numpy(), ml.numpy()

    # Config 2's path at one layer and 4,096 tokens, bf16 model, int8 cold tier, composed from the
    # reference's pack/unpack, top_blocks, cpu_partial_attention and merge_lse (the reference itself
    # refuses int8 + exact, lazykv/exact.py:165-168, so the composition is the specification).
    lay = I.bf16_layer(seed=41, t=4096 + 9)  # 256 sealed blocks + a current block with 9 tokens
    e["int8_checksum"] = np.concatenate([I.checksum(lay[x]) for x in ("k", "v", "q")])
    n_sealed, fill = 256, 9
    pairs = I.pairs_from_kv(lay["k"], lay["v"], bs)  # [256, 8, 2, 16, 64]
    rec = pack(pairs)  # [256, 8, W]
    deq_bf = unpack(rec.flatten(0, 1), bs, I.D, torch.bfloat16).view(n_sealed, I.HKV, 2, bs, I.D)
    deq_bf[0] = pairs[0]  # the sink never leaves VRAM: exact (tiered.py:200-202)
    keys_meta = deq_bf[:, :, 0].permute(1, 0, 2, 3)  # [h, n, bs, d]
    kmin, kmax = keys_meta.amin(2)[None], keys_meta.amax(2)[None]
    kk = blocks_for_budget(0.25, 4096 + fill, bs)
    qq = lay["q"].view(1, I.HQ, 1, I.D)
    idx = (top_blocks(qq, kmin[:, :, 1:n_sealed], kmax[:, :, 1:n_sealed], kk) + 1)[0].numpy()
    e["int8_k"] = np.array(kk)
    e["int8_bound"] = I.bf16_np(quest_bound(qq, kmin[:, :, 1:n_sealed], kmax[:, :, 1:n_sealed])[0])
    e["int8_idx"] = idx
    e["int8_rec_sha"] = np.frombuffer(__import__("hashlib").sha256(rec.numpy().tobytes()).digest(), dtype=np.uint8)
    cur = torch.zeros(I.HKV, 2, bs, I.D)
    cur[:, 0, :fill] = lay["k"][:, n_sealed * bs :].float()
    cur[:, 1, :fill] = lay["v"][:, n_sealed * bs :].float()
    # Hot: sink + selected (slot contents = bf16 dequantised) + current; laid out as one sequence
    # and attended with everything else excluded. Cold: the other sealed blocks as a fetch would
    # produce them (bf16 dequantised), in float32, as the exact pass attends to its mirror
    # (exact.py:189-192).
    full_hot = torch.cat([deq_bf.float(), cur[None]], dim=0)  # [n+1, h, 2, bs, d]
    full_cold = full_hot
    kh = full_hot[:, :, 0].permute(1, 0, 2, 3).reshape(I.HKV, -1, I.D)
    vh = full_hot[:, :, 1].permute(1, 0, 2, 3).reshape(I.HKV, -1, I.D)
    kc = full_cold[:, :, 0].permute(1, 0, 2, 3).reshape(I.HKV, -1, I.D)
    vc = full_cold[:, :, 1].permute(1, 0, 2, 3).reshape(I.HKV, -1, I.D)
    live = (n_sealed) * bs + fill
    hot_set = np.concatenate([np.zeros((I.HKV, 1), np.int64), idx], axis=1)
    cold_excl = np.concatenate([hot_set, np.full((I.HKV, 1), n_sealed)], axis=1)
    hot_excl = np.array([[b for b in range(n_sealed) if b not in set(hot_set[j].tolist())] for j in range(I.HKV)])
    qg = lay["q"].float().view(I.HKV, I.HQ // I.HKV, I.D)
    # Exclusion works on whole blocks, so the current block's live tail is its own partial.
    ho, hl = _partial_live(cpu_partial_attention, kh, vh, qg, scale, bs, hot_excl, live)
    co, cl = cpu_partial_attention(kc[:, : n_sealed * bs], vc[:, : n_sealed * bs], qg, scale, bs, cold_excl[:, :-1])
    mo, ml = merge_lse(ho, hl, co, cl)
    e["int8_fill"] = np.array(fill)
    e["int8_hot_out"], e["int8_hot_lse"] = ho.numpy(), hl.numpy()
    e["int8_cold_out"], e["int8_cold_lse"] = co.numpy(), cl.numpy()
    e["int8_out"], e["int8_lse"] = mo.numpy(), ml.numpy()

    for name, d in out.items():
        np.savez_compressed(HERE / f"{name}.npz", **d)
        print(name, {k: v.shape for k, v in d.items()})


def _partial_live(fn, k, v, q, scale, bs, excluded, live):  # noqa: ANN001, ANN202
    """cpu_partial_attention over blocks, with the current block cut at `live` tokens.

    The reference masks the current block's tail with an additive -inf (selection.py:65-69); the
    same is done here by attending the whole-block part and the live tail as two partials and
    merging them, which is the identity lazykv/exact.py:69-85 rests on.
    """
    from lazykv.exact import merge_lse

    full = (live // bs) * bs
    oa, la = fn(k[:, :full], v[:, :full], q, scale, bs, excluded)
    tail = live - full
    kt, vt = k[:, full:live], v[:, full:live]
    ob, lb = fn(kt, vt, q, scale, tail, np.empty((k.shape[0], 0), np.int64))
    return merge_lse(oa, la, ob, lb)


if __name__ == "__main__":
    if len(sys.argv) != 2:
        raise SystemExit("usage: make_golden.py <path to the LazyKV source tree>")
    main(sys.argv[1])
