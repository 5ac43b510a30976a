"""The attention kernels (tensor-core, TMA-pipelined and plain-load) and the fused exact call,
against the oracle.

The tensor-core stream kernel serves bf16 stores in device memory at d 64 or 128, bs 16, G <= 8; the TMA
kernel the other device-memory cases at G = 4, bs = 16, d in {64, 128}; the plain-load kernel every other
geometry and cold stores in mapped host memory. Every case is compared with float64 attention over
the same values (1e-5 of the max; int8 cold blocks as unpack in the model dtype), and the fused call
with the separate calls and their merge.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

import oracle as O

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _k():
    from lazykv_b200 import kernels

    return kernels


def _rel(got, want) -> float:  # noqa: ANN001
    got = np.asarray(got, np.float64)
    return float(np.abs(got - want).max() / max(np.abs(want).max(), 1e-30))


def _setup(h: int, g: int, d: int, bs: int, n: int, k: int, dtype: torch.dtype, seed: int):  # noqa: ANN202
    gen = torch.Generator().manual_seed(seed)
    kv = torch.randn(n, h, 2, bs, d, generator=gen)
    kv[:, :, 0] += torch.randn(1, h, 1, d, generator=gen) * 0.7
    kv = kv.to(dtype)
    q = torch.randn(h * g, d, generator=gen).to(dtype)
    sel = torch.stack([torch.randperm(n - 2, generator=gen)[:k] + 1 for _ in range(h)])  # ids in 1..n-2
    return kv, q, sel


def _oracle_sets(kv: torch.Tensor, q: torch.Tensor, sel: torch.Tensor, fill: int, cold_vals: np.ndarray, scale: float):  # noqa: ANN202
    """float64 (hot, cold, merged) for hot = [0, sel..., n-1 (fill live)], cold = 1..n-2 minus sel."""
    n, h, _, bs, d = kv.shape
    g = q.shape[0] // h
    x = kv.float().numpy()
    qg = q.float().numpy().reshape(h, g, d)
    ho, hl, co, cl = np.zeros((h, g, d)), np.zeros((h, g)), np.zeros((h, g, d)), np.zeros((h, g))
    for j in range(h):
        ids = [0] + sel[j].tolist() + [n - 1]
        kk = np.concatenate([x[b, j, 0] for b in ids])
        vv = np.concatenate([x[b, j, 1] for b in ids])
        valid = np.ones(len(kk), bool)
        valid[len(kk) - bs + fill:] = False
        ho[j], hl[j] = O.attend_tokens(qg[j], kk, vv, scale, valid)
        rest = sorted(set(range(1, n - 1)) - set(sel[j].tolist()))
        kc = np.concatenate([cold_vals[b, j, 0] for b in rest])
        vc = np.concatenate([cold_vals[b, j, 1] for b in rest])
        co[j], cl[j] = O.attend_tokens(qg[j], kc, vc, scale)
    out, lse = O.merge_lse(ho, hl, co, cl)
    return ho, hl, co, cl, out, lse


def _bitmap(sel: torch.Tensor, n: int) -> torch.Tensor:
    h = sel.shape[0]
    words = (n + 31) // 32
    bm = np.zeros((h, words), np.uint32)
    for j in range(h):
        for b in sel[j].tolist():
            bm[j, b // 32] |= np.uint32(1 << (b % 32))
    return torch.from_numpy(bm.view(np.int32)).to(DEV)


@pytest.mark.parametrize("d,bs,dtype,int8", [(64, 16, torch.bfloat16, True), (128, 16, torch.bfloat16, True), (64, 16, torch.float32, False),
                                             (64, 16, torch.bfloat16, False), (16, 8, torch.bfloat16, True), (64, 8, torch.float32, True)])
def test_hot_cold_and_fused_match_float64(d: int, bs: int, dtype: torch.dtype, int8: bool) -> None:
    _check_paths(d, bs, dtype, int8, 4)


@pytest.mark.parametrize("g", [1, 2, 8])
@pytest.mark.parametrize("int8", [True, False])
def test_head_dim_128_in_every_query_group(g: int, int8: bool) -> None:
    """head_dim 128 (the long-context geometry) through the tensor-core stream kernel at every group."""
    _check_paths(128, 16, torch.bfloat16, int8, g)


def _check_paths(d: int, bs: int, dtype: torch.dtype, int8: bool, g: int) -> None:
    K = _k()
    h, n, k, fill = 4, 300, 40, 5
    kv, q, sel = _setup(h, g, d, bs, n, k, dtype, seed=d + bs + int(int8))
    kvd, qd = kv.to(DEV), q.to(DEV)
    if int8:
        cold = K.pack_int8(kvd)
        cold_vals = K.unpack_int8(cold.view(-1, cold.shape[-1]), bs, d, dtype).float().view(n, h, 2, bs, d).cpu().numpy()
    else:
        cold = kvd
        cold_vals = kv.float().numpy()
    blocks = torch.cat([torch.zeros((h, 1), dtype=torch.int32), sel.int(), torch.full((h, 1), n - 1, dtype=torch.int32)], 1).to(DEV)
    strides = (h * 2 * bs * d, 2 * bs * d, d)
    bitmap = _bitmap(sel, n)
    scale = d**-0.5
    want = _oracle_sets(kv, q, sel, fill, cold_vals, scale)
    hot, hlse = K.hot_attention(qd, kvd, kvd[:, :, 1], strides, blocks, fill, scale, bs)
    cld, clse = K.cold_attention(qd, cold, bs, 1, n - 2, scale, excluded=bitmap)
    assert _rel(hot.view(h, g, d).cpu(), want[0]) < 1e-5 and _rel(hlse.view(h, g).cpu(), want[1]) < 1e-5
    assert _rel(cld.view(h, g, d).cpu(), want[2]) < 1e-5 and _rel(clse.view(h, g).cpu(), want[3]) < 1e-5
    po = torch.empty((2, h * g, d), device=DEV)
    pl = torch.empty((2, h * g), device=DEV)
    out, lse = K.exact_attention(qd, kvd, kvd[:, :, 1], strides, blocks, fill, cold, 1, n - 2, scale, bs, excluded=bitmap,
                                 out_dtype=torch.float32, parts=(po, pl))
    assert _rel(out.view(h, g, d).cpu(), want[4]) < 1e-5 and _rel(lse.view(h, g).cpu(), want[5]) < 1e-5
    assert _rel(po[0].cpu(), hot.cpu().numpy()) < 1e-6 and _rel(po[1].cpu(), cld.cpu().numpy()) < 1e-6
    assert K.device_status() == 0


def test_host_mapped_cold_store_reads_over_the_link() -> None:
    from lazykv_b200.pinned import device_view, pinned_empty

    K = _k()
    h, g, d, bs, n, k, fill = 8, 4, 64, 16, 200, 30, 16
    kv, q, sel = _setup(h, g, d, bs, n, k, torch.bfloat16, seed=77)
    kvd, qd = kv.to(DEV), q.to(DEV)
    rec = K.pack_int8(kvd)
    host = pinned_empty(tuple(rec.shape), torch.uint8)
    host.copy_(rec.cpu())
    mapped = device_view(host)
    bitmap = _bitmap(sel, n)
    # Device records go to the tensor-core stream kernel, mapped ones to the plain-load kernel: the same
    # values, two summation orders.
    a, al = K.cold_attention(qd, rec, bs, 1, n - 2, d**-0.5, excluded=bitmap)
    b, bl = K.cold_attention(qd, mapped, bs, 1, n - 2, d**-0.5, excluded=bitmap)
    assert _rel(b.cpu(), a.cpu().numpy()) < 1e-5 and _rel(bl.cpu(), al.cpu().numpy()) < 1e-6
    blocks = torch.cat([torch.zeros((h, 1), dtype=torch.int32), sel.int(), torch.full((h, 1), n - 1, dtype=torch.int32)], 1).to(DEV)
    strides = (h * 2 * bs * d, 2 * bs * d, d)
    o1, l1 = K.exact_attention(qd, kvd, kvd[:, :, 1], strides, blocks, fill, rec, 1, n - 2, d**-0.5, bs, excluded=bitmap, out_dtype=torch.float32)
    o2, l2 = K.exact_attention(qd, kvd, kvd[:, :, 1], strides, blocks, fill, mapped, 1, n - 2, d**-0.5, bs, excluded=bitmap, out_dtype=torch.float32)
    assert _rel(o2.cpu(), o1.cpu().numpy()) < 1e-5 and _rel(l2.cpu(), l1.cpu().numpy()) < 1e-6


def test_slot_map_indirection_and_all_excluded_heads() -> None:
    K = _k()
    h, g, d, bs, n, k = 8, 4, 64, 16, 100, 20
    kv, q, sel = _setup(h, g, d, bs, n, k, torch.bfloat16, seed=5)
    kvd, qd = kv.to(DEV), q.to(DEV)
    blocks = torch.cat([torch.zeros((h, 1), dtype=torch.int32), sel.int(), torch.full((h, 1), n - 1, dtype=torch.int32)], 1).to(DEV)
    # A pool with the listed blocks at shuffled slots, reached through slot_of.
    perm = torch.randperm(n, generator=torch.Generator().manual_seed(1))
    pool = kvd[perm.to(DEV)].contiguous()  # slot s holds block perm[s]
    inv = torch.empty(n, dtype=torch.int32)
    inv[perm] = torch.arange(n, dtype=torch.int32)
    slot_of = inv.repeat(h, 1).to(DEV).contiguous()
    strides = (h * 2 * bs * d, 2 * bs * d, d)
    a, al = K.hot_attention(qd, kvd, kvd[:, :, 1], strides, blocks, 7, d**-0.5, bs)
    b, bl = K.hot_attention(qd, pool, pool[:, :, 1], strides, blocks, 7, d**-0.5, bs, slot_of=slot_of)
    assert torch.equal(a, b) and torch.equal(al, bl)
    everything = torch.full((h, (n + 31) // 32), -1, dtype=torch.int32, device=DEV)
    rec = K.pack_int8(kvd)
    c, cl = K.cold_attention(qd, rec, bs, 1, n - 2, d**-0.5, excluded=everything)
    assert (c == 0).all() and torch.isneginf(cl).all()
    out, lse = K.exact_attention(qd, kvd, kvd[:, :, 1], strides, blocks, 7, rec, 1, n - 2, d**-0.5, bs, excluded=everything, out_dtype=torch.float32)
    assert torch.allclose(out, a, rtol=1e-6, atol=1e-7) and torch.allclose(lse, al, rtol=1e-6)


@pytest.mark.parametrize("g", [1, 2, 4, 8])
@pytest.mark.parametrize("layout", ["pool", "cache"])
def test_tensor_core_path_every_group_and_layout(g: int, layout: str) -> None:
    """bf16, d 64, bs 16: hot blocks through tensor maps over a slot pool [S, h, 2, bs, d] (rows
    outer) or a full cache [1, h, T, d] (heads outer), int8 and bf16-pairs cold stores, against
    float64 over the same values; and the same hot call with the row bound withheld (CUDA-core
    kernels) within float32 rounding of it."""
    K = _k()
    h, d, bs, n, k, fill = 8, 64, 16, 160, 24, 11
    kv, q, sel = _setup(h, g, d, bs, n, k, torch.bfloat16, seed=100 + g)
    kvd, qd = kv.to(DEV), q.to(DEV)
    blocks = torch.cat([torch.zeros((h, 1), dtype=torch.int32), sel.int(), torch.full((h, 1), n - 1, dtype=torch.int32)], 1).to(DEV)
    scale = d**-0.5
    if layout == "pool":
        kb, vb = kvd, kvd[:, :, 1]
        strides = (h * 2 * bs * d, 2 * bs * d, d)
    else:
        kb = kvd[:, :, 0].permute(1, 0, 2, 3).reshape(1, h, n * bs, d).contiguous()  # [1, h, T, d]
        vb = kvd[:, :, 1].permute(1, 0, 2, 3).reshape(1, h, n * bs, d).contiguous()
        strides = (bs * d, n * bs * d, d)
    rec = K.pack_int8(kvd)
    cold_vals = K.unpack_int8(rec.view(-1, rec.shape[-1]), bs, d, torch.bfloat16).float().view(n, h, 2, bs, d).cpu().numpy()
    want = _oracle_sets(kv, q, sel, fill, cold_vals, scale)
    hot, hlse = K.hot_attention(qd, kb, vb, strides, blocks, fill, scale, bs)
    assert _rel(hot.view(h, g, d).cpu(), want[0]) < 1e-5 and _rel(hlse.view(h, g).cpu(), want[1]) < 1e-5
    bitmap = _bitmap(sel, n)
    cld, clse = K.cold_attention(qd, rec, bs, 1, n - 2, scale, excluded=bitmap)
    assert _rel(cld.view(h, g, d).cpu(), want[2]) < 1e-5 and _rel(clse.view(h, g).cpu(), want[3]) < 1e-5
    out, lse = K.exact_attention(qd, kb, vb, strides, blocks, fill, rec, 1, n - 2, scale, bs, excluded=bitmap, out_dtype=torch.float32)
    assert _rel(out.view(h, g, d).cpu(), want[4]) < 1e-5 and _rel(lse.view(h, g).cpu(), want[5]) < 1e-5
    # bf16 pairs as the cold store (the bf16 exact tier)
    want_p = _oracle_sets(kv, q, sel, fill, kv.float().numpy(), scale)
    out_p, lse_p = K.exact_attention(qd, kb, vb, strides, blocks, fill, kvd, 1, n - 2, scale, bs, excluded=bitmap, out_dtype=torch.float32)
    assert _rel(out_p.view(h, g, d).cpu(), want_p[4]) < 1e-5 and _rel(lse_p.view(h, g).cpu(), want_p[5]) < 1e-5
    # The CUDA-core kernels (row bound withheld) agree to float32 rounding.
    from lazykv_b200 import _lib as L

    ref_o = torch.empty_like(hot)
    ref_l = torch.empty_like(hlse)
    ws = K.workspace(qd.device, K.attention_workspace_bytes(h, h * g, d, blocks.shape[1]))
    L.call("lkv_hot_attention", L.ptr(qd), h * g, h, d, bs, L.ptr(kb), L.ptr(vb), L.dtype_code(torch.bfloat16), *strides, 0, L.ptr(blocks),
           blocks.shape[1], None, 0, fill, scale, L.ptr(ref_o), L.ptr(ref_l), L.ptr(ws), ws.numel(), L.stream_handle(qd.device))
    assert _rel(ref_o.cpu(), hot.cpu().numpy()) < 1e-5 and _rel(ref_l.cpu(), hlse.cpu().numpy()) < 1e-6
    assert K.device_status() == 0


def test_selection_does_not_change_the_exact_int8_result() -> None:
    """Every sealed block is attended as unpack(record) in bf16 whether it is hot or cold, so two
    different selections give the same exact output up to float32 rounding."""
    K = _k()
    h, g, d, bs, n, k, fill = 8, 4, 64, 16, 200, 30, 9
    kv, q, _ = _setup(h, g, d, bs, n, k, torch.bfloat16, seed=9)
    kvd, qd = kv.to(DEV), q.to(DEV)
    rec = K.pack_int8(kvd)
    deq = K.unpack_int8(rec.view(-1, rec.shape[-1]), bs, d, torch.bfloat16).view(n, h, 2, bs, d)
    deq[0] = kvd[0]  # the sink stays exact
    strides = (h * 2 * bs * d, 2 * bs * d, d)
    outs = []
    for seed in (1, 2):
        gen = torch.Generator().manual_seed(seed)
        sel = torch.stack([torch.sort(torch.randperm(n - 2, generator=gen)[:k] + 1).values for _ in range(h)])
        blocks = torch.cat([torch.zeros((h, 1), dtype=torch.int32), sel.int(), torch.full((h, 1), n - 1, dtype=torch.int32)], 1).to(DEV)
        # The pool holds what a fetch produces: the dequantised blocks (and the exact sink / current).
        pool = deq.clone()
        pool[n - 1] = kvd[n - 1]
        out, lse = K.exact_attention(qd, pool, pool[:, :, 1], strides, blocks, fill, rec, 1, n - 2, d**-0.5, bs, excluded=_bitmap(sel, n),
                                     out_dtype=torch.float32)
        outs.append((out.cpu(), lse.cpu()))
    assert _rel(outs[0][0], outs[1][0].numpy()) < 2e-6 and _rel(outs[0][1], outs[1][1].numpy()) < 1e-6
