"""numpy restatement of the reference's hot-path algorithm (TEST INFRASTRUCTURE ONLY).

Every function names the reference file:line it restates; paths are within PS12007/LazyKV.
Two places fix a choice the reference leaves to its libraries, so that a GPU kernel can be held
to the bit:

* Quest bound accumulation order (`quest_bound`). The reference computes the bound with two
  matmuls (`lazykv/selection.py:49-53`), whose float32 accumulation order belongs to the BLAS.
  Here each dot product is accumulated left to right over the channels, one float32 product and
  one float32 add per channel, each rounded (no fused multiply-add). In bf16 mode each of the two
  dot products is rounded to bf16 and their sum is rounded to bf16 again, as the reference's two
  bf16 matmul outputs and bf16 add are. The kernel uses the same order.
* Top-K tie order (`top_blocks`). `torch.topk`'s order among equal values is unspecified
  (`lazykv/selection.py:56-62`). Here the order is descending bound, then ascending block id;
  +0.0 and -0.0 compare equal.

Everything else (the int8 record, the merge, the partial attention) follows the reference's own
float32 operation order, so the int8 records and dequantized values are bit-exact.
"""

from __future__ import annotations

import math

import numpy as np

F32 = np.float32
F64 = np.float64
TINY = np.finfo(np.float32).tiny
LEVELS = 255  # lazykv/quant.py:43
SCALE_BYTES = 2  # float16 scales and zeros, lazykv/quant.py:42


# -- bf16 helpers -----------------------------------------------------------------------------


def bf16_bits(x: np.ndarray) -> np.ndarray:
    """Round float32 values to bf16 (round to nearest, ties to even) and return the 16-bit patterns."""
    u = np.ascontiguousarray(x, dtype=F32).view(np.uint32)
    nan = (u & 0x7FFFFFFF) > 0x7F800000
    r = (u + 0x7FFF + ((u >> 16) & 1)) >> 16
    r = np.where(nan, (u >> 16) | 0x40, r)
    return r.astype(np.uint16)


def bf16_to_f32(bits: np.ndarray) -> np.ndarray:
    return (np.asarray(bits, dtype=np.uint32) << 16).view(F32)


def bf16_round(x: np.ndarray) -> np.ndarray:
    """float32 values rounded to the nearest bf16 value, returned as float32."""
    return bf16_to_f32(bf16_bits(x))


def to_dtype(x: np.ndarray, dtype: str) -> np.ndarray:
    """Cast float32 values to the model dtype ('float32' or 'bfloat16'), returned as float32."""
    if dtype == "float32":
        return np.asarray(x, dtype=F32)
    if dtype == "bfloat16":
        return bf16_round(np.asarray(x, dtype=F32))
    raise ValueError(f"unsupported dtype {dtype!r}")


# -- int8 record codec (lazykv/quant.py) --------------------------------------------------------


def packed_pair_bytes(block_size: int, head_dim: int) -> int:
    """Bytes of one packed (block, head) record: lazykv/quant.py:46-49."""
    return 2 * block_size * head_dim + 2 * SCALE_BYTES * head_dim + 2 * SCALE_BYTES * block_size


def record_offsets(block_size: int, head_dim: int) -> tuple[int, int, int, int, int]:
    """Cut points k payload | v payload | k scale | k zero | v scale | v zero: lazykv/quant.py:52-56."""
    s, n = SCALE_BYTES, block_size * head_dim
    return (n, 2 * n, 2 * n + s * head_dim, 2 * n + 2 * s * head_dim, 2 * n + 2 * s * head_dim + s * block_size)


def _affine(x: np.ndarray, axis: int) -> tuple[np.ndarray, np.ndarray, np.ndarray]:
    """Asymmetric int8 quantisation over `axis`, float32 arithmetic: lazykv/quant.py:59-70."""
    mn = x.min(axis=axis, keepdims=True).astype(F32)
    mx = x.max(axis=axis, keepdims=True).astype(F32)
    scale = np.maximum((mx - mn) / F32(LEVELS), F32(TINY)).astype(F32)
    q = np.rint((x.astype(F32) - mn) / scale)
    q = (np.clip(q, 0, LEVELS) - 128).astype(np.int8)
    with np.errstate(over="ignore"):  # float16 overflow to inf is what torch's .to(float16) does too
        return q, np.squeeze(scale, axis).astype(np.float16), np.squeeze(mn, axis).astype(np.float16)


def pack(blocks: np.ndarray) -> np.ndarray:
    """Pack KV pairs [..., 2, bs, d] (float32 holding model-dtype values) into uint8 records.

    Restates lazykv/quant.py:73-87: keys per channel (range over the block's tokens), values per
    token (range over head_dim); record = kq | vq | k_scale | k_zero | v_scale | v_zero.
    """
    *lead, two, bs, d = blocks.shape
    if two != 2:
        raise ValueError(f"expected a [..., 2, block_size, head_dim] KV pair, got {tuple(blocks.shape)}")
    x = np.asarray(blocks, dtype=F32).reshape(-1, 2, bs, d)
    kq, ks, kz = _affine(x[:, 0], axis=1)
    vq, vs, vz = _affine(x[:, 1], axis=2)
    parts = [kq.reshape(len(x), -1), vq.reshape(len(x), -1), ks, kz, vs, vz]
    rec = np.concatenate([np.ascontiguousarray(p).view(np.uint8).reshape(len(x), -1) for p in parts], axis=1)
    return rec.reshape(*lead, rec.shape[-1])


def unpack(records: np.ndarray, block_size: int, head_dim: int, dtype: str = "float32") -> np.ndarray:
    """Dequantise uint8 records [m, W] to [m, 2, bs, d]: lazykv/quant.py:90-105.

    `(q + 128) * scale + zero` in float32 with each operation rounded, then cast to `dtype`.
    """
    w = packed_pair_bytes(block_size, head_dim)
    if records.ndim != 2 or records.shape[1] != w:
        raise ValueError(f"expected [m, {w}] uint8 records, got {tuple(records.shape)}")
    o1, o2, o3, o4, o5 = record_offsets(block_size, head_dim)
    r = np.ascontiguousarray(records)
    m = r.shape[0]
    kq = r[:, :o1].copy().view(np.int8).reshape(m, block_size, head_dim)
    vq = r[:, o1:o2].copy().view(np.int8).reshape(m, block_size, head_dim)
    ks = r[:, o2:o3].copy().view(np.float16).astype(F32)
    kz = r[:, o3:o4].copy().view(np.float16).astype(F32)
    vs = r[:, o4:o5].copy().view(np.float16).astype(F32)
    vz = r[:, o5:].copy().view(np.float16).astype(F32)
    k = (kq.astype(F32) + F32(128)) * ks[:, None, :] + kz[:, None, :]
    v = (vq.astype(F32) + F32(128)) * vs[:, :, None] + vz[:, :, None]
    return to_dtype(np.stack([k.astype(F32), v.astype(F32)], axis=1), dtype)


# -- selection (lazykv/selection.py) ------------------------------------------------------------


def blocks_for_budget(fraction: float, total_tokens: int, block_size: int) -> int:
    """K such that sink + K + current fit the budget: lazykv/selection.py:72-74."""
    return max(1, math.floor(fraction * total_tokens / block_size) - 2)


def block_minmax(keys: np.ndarray, block_size: int) -> tuple[np.ndarray, np.ndarray]:
    """Channel-wise min/max of each block's keys, [h, n*bs, d] -> [h, n, d]: lazykv/selection.py:142-144."""
    h, t, d = keys.shape
    b = keys.reshape(h, t // block_size, block_size, d)
    return b.min(axis=2).astype(F32), b.max(axis=2).astype(F32)


def _seq_dot(qv: np.ndarray, m: np.ndarray) -> np.ndarray:
    """sum_c qv[h, g, c] * m[h, n, c], left to right over c, float32 product and add each rounded."""
    h, g, d = qv.shape
    acc = np.zeros((h, g, m.shape[1]), dtype=F32)
    for c in range(d):
        prod = (qv[:, :, c, None] * m[:, None, :, c]).astype(F32)
        acc = (acc + prod).astype(F32)
    return acc


def quest_bound(query: np.ndarray, kmin: np.ndarray, kmax: np.ndarray, mode: str = "bfloat16") -> np.ndarray:
    """Quest upper bound [h, n] per KV head and candidate block: lazykv/selection.py:38-53.

    `query` [Hq, d] (model-dtype values), `kmin`/`kmax` [h, n, d]. bound = max over the head's
    query group of q+ . kmax + q- . kmin, no 1/sqrt(d) (the reference applies none). `mode` is the
    dtype the reference computes in: 'bfloat16' rounds each dot product and their sum to bf16;
    'float32' keeps float32.
    """
    h, n, d = kmin.shape
    q = np.asarray(query, dtype=F32).reshape(h, -1, d)
    qp = np.maximum(q, F32(0))
    qn = (q - qp).astype(F32)
    a = _seq_dot(qp, np.asarray(kmax, dtype=F32))
    b = _seq_dot(qn, np.asarray(kmin, dtype=F32))
    if mode == "bfloat16":
        s = bf16_round(bf16_round(a) + bf16_round(b))
    elif mode == "float32":
        s = (a + b).astype(F32)
    else:
        raise ValueError(f"unsupported bound mode {mode!r}")
    out = s.max(axis=1).astype(F32)
    return out + F32(0)  # -0.0 -> +0.0, so the tie rule sees one zero


def top_blocks(bound: np.ndarray, k: int) -> np.ndarray:
    """Top-k candidate indices [h, k], descending bound then ascending index: lazykv/selection.py:56-62."""
    h, n = bound.shape
    out = np.empty((h, k), dtype=np.int64)
    ids = np.arange(n)
    for j in range(h):
        order = np.lexsort((ids, -bound[j].astype(F64)))
        out[j] = order[:k]
    return out


def canonical_order(bound_row: np.ndarray, idx_row: np.ndarray) -> np.ndarray:
    """Re-sort a reference top-k row by (descending bound, ascending index)."""
    order = np.lexsort((idx_row, -bound_row[idx_row].astype(F64)))
    return idx_row[order]


def current_block_mask(total: int, block_size: int, fill: int) -> np.ndarray:
    """Additive mask over the gathered keys, -inf past `fill` in the last block: lazykv/selection.py:65-69."""
    mask = np.zeros(total, dtype=F32)
    mask[total - block_size + fill :] = -np.inf
    return mask


# -- exact merge (lazykv/exact.py) ---------------------------------------------------------------


def merge_lse(out_a: np.ndarray, lse_a: np.ndarray, out_b: np.ndarray, lse_b: np.ndarray) -> tuple[np.ndarray, np.ndarray]:
    """Log-sum-exp merge of two partials, safe when both are empty: lazykv/exact.py:69-85."""
    dt = np.result_type(out_a, out_b, lse_a, lse_b)
    with np.errstate(invalid="ignore", over="ignore"):
        lse = np.logaddexp(lse_a, lse_b)
        finite = np.isfinite(lse)
        safe = np.where(finite, lse, 0)
        wa = np.where(finite, np.exp(lse_a - safe), 0).astype(dt)
        wb = np.where(finite, np.exp(lse_b - safe), 0).astype(dt)
    return (wa[..., None] * out_a + wb[..., None] * out_b).astype(dt), lse.astype(dt)


def cpu_partial_attention(keys: np.ndarray, values: np.ndarray, query: np.ndarray, scaling: float, block_size: int, excluded: np.ndarray, dtype=F32) -> tuple[np.ndarray, np.ndarray]:
    """Softmax partial over every block except `excluded` per KV head: lazykv/exact.py:88-127.

    `keys`/`values` [h, n*bs, d], `query` [h, g, d], `excluded` [h, e] block ids. Excluded columns
    are -inf before the row max; a head with nothing left returns lse = -inf and out = 0.
    `dtype=float32` follows the reference's own arithmetic; float64 is the parity ground truth.
    """
    h, total, d = keys.shape
    n_blocks = total // block_size
    k = np.asarray(keys, dtype=dtype)
    v = np.asarray(values, dtype=dtype)
    q = np.asarray(query, dtype=dtype)
    scores = np.matmul(q, k.transpose(0, 2, 1)) * dtype(scaling)
    if excluded.shape[1]:
        sv = scores.reshape(h, q.shape[1], n_blocks, block_size)
        for j in range(h):
            sv[j, :, excluded[j]] = -np.inf
    m = scores.max(axis=-1, keepdims=True)
    empty = np.isneginf(m)
    scores = scores - np.where(empty, 0, m)
    scores = np.exp(scores)
    scores = np.where(empty, 0, scores)
    norm = scores.sum(axis=-1, keepdims=True)
    scores = scores / np.maximum(norm, np.finfo(dtype).tiny)
    out = np.matmul(scores, v).astype(dtype)
    with np.errstate(divide="ignore"):
        lse = np.where(empty, -np.inf, m + np.log(norm)).squeeze(-1).astype(dtype)
    return out, lse


def attend_tokens(query: np.ndarray, keys: np.ndarray, values: np.ndarray, scaling: float, valid: np.ndarray | None = None) -> tuple[np.ndarray, np.ndarray]:
    """float64 softmax attention of query [g, d] over keys/values [T, d]; returns (out [g, d], lse [g])."""
    q = np.asarray(query, dtype=F64)
    s = q @ np.asarray(keys, dtype=F64).T * scaling
    if valid is not None:
        s[:, ~valid] = -np.inf
    if s.shape[1] == 0 or np.all(np.isneginf(s)):
        return np.zeros((q.shape[0], keys.shape[1])), np.full(q.shape[0], -np.inf)
    m = s.max(axis=1, keepdims=True)
    p = np.exp(s - m)
    l = p.sum(axis=1, keepdims=True)
    return (p / l) @ np.asarray(values, dtype=F64), (m + np.log(l))[:, 0]


# -- the north-star composition --------------------------------------------------------------------


def tiered_decode(
    query: np.ndarray,
    sealed: np.ndarray,
    current: np.ndarray,
    fill: int,
    k_blocks: int,
    scaling: float,
    model_dtype: str = "bfloat16",
    quant: str | None = "int8",
    bound_mode: str | None = None,
    selected: np.ndarray | None = None,
) -> dict[str, np.ndarray]:
    """One decode step of one selecting layer, as the reference's pieces compose (float64 math).

    `query` [Hq, d]; `sealed` [n_sealed, h, 2, bs, d] (the host pool's layout, lazykv/tiered.py:265);
    `current` [h, 2, bs, d] with `fill` live tokens. Block 0 (the sink) is always exact
    (lazykv/tiered.py:200-202); sealed blocks 1..n-1 hold `unpack(pack(block))` under int8
    (lazykv/tiered.py:187-197) in the model dtype, in the hot set and in the cold set alike: the
    exact pass attends to "what a fetch would have produced" (lazykv/exact.py:189-192, the rule its
    float32 mirror follows for the bf16 tier), so the output does not depend on which blocks were
    selected beyond float rounding; metadata is taken over the dequantised keys.
    Selected ids are `top_blocks(...) + 1` (lazykv/tiered.py:383-387). The hot set is
    [sink, selected in rank order, current] (lazykv/tiered.py:465-487); the cold set is every
    other sealed block (lazykv/exact.py:371-378). Returns hot/cold partials, the merged output
    and the selection. `selected` [h, K] block ids, when given, replaces the oracle's own selection
    (to compose with another implementation's choice among tied blocks).
    """
    n, h, _, bs, d = sealed.shape
    hq = query.shape[0]
    g = hq // h
    bound_mode = bound_mode or model_dtype
    if quant == "int8":
        rec = pack(sealed)  # [n, h, W]
        flat = rec.reshape(n * h, -1)
        hot_blocks = unpack(flat, bs, d, model_dtype).reshape(n, h, 2, bs, d)
        hot_blocks[0] = sealed[0]
        cold_blocks = hot_blocks
    elif quant is None:
        rec = None
        hot_blocks = cold_blocks = np.asarray(sealed, dtype=F32)
    else:
        raise ValueError(f"unknown quant {quant!r}")
    keys_meta = hot_blocks[:, :, 0].transpose(1, 0, 2, 3).reshape(h, n * bs, d)
    kmin, kmax = block_minmax(keys_meta, bs)
    q = to_dtype(query, model_dtype)
    bound = quest_bound(q, kmin[:, 1:n], kmax[:, 1:n], bound_mode)
    sel = top_blocks(bound, k_blocks) + 1 if selected is None else np.asarray(selected, dtype=np.int64)
    qg = q.reshape(h, g, d)
    hot_o = np.zeros((h, g, d))
    hot_l = np.zeros((h, g))
    cold_o = np.zeros((h, g, d))
    cold_l = np.zeros((h, g))
    for j in range(h):
        blocks = [hot_blocks[0, j]] + [hot_blocks[b, j] for b in sel[j]] + [current[j]]
        kk = np.concatenate([b[0] for b in blocks])
        vv = np.concatenate([b[1] for b in blocks])
        valid = np.ones(len(kk), dtype=bool)
        valid[len(kk) - bs + fill :] = False
        hot_o[j], hot_l[j] = attend_tokens(qg[j], kk, vv, scaling, valid)
        rest = sorted(set(range(1, n)) - set(sel[j].tolist()))
        if rest:
            kc = np.concatenate([cold_blocks[b, j, 0] for b in rest])
            vc = np.concatenate([cold_blocks[b, j, 1] for b in rest])
            cold_o[j], cold_l[j] = attend_tokens(qg[j], kc, vc, scaling)
        else:
            cold_o[j], cold_l[j] = 0.0, -np.inf
    out, lse = merge_lse(hot_o, hot_l, cold_o, cold_l)
    return {
        "records": rec,
        "kmin": kmin,
        "kmax": kmax,
        "bound": bound,
        "selected": sel,
        "hot_out": hot_o,
        "hot_lse": hot_l,
        "cold_out": cold_o,
        "cold_lse": cold_l,
        "out": out,
        "lse": lse,
    }


def dense_attention(query: np.ndarray, keys: np.ndarray, values: np.ndarray, scaling: float) -> tuple[np.ndarray, np.ndarray]:
    """float64 attention of query [Hq, d] over keys/values [h, T, d] with GQA: the exactness target."""
    h, t, d = keys.shape
    g = query.shape[0] // h
    out = np.zeros((h, g, d))
    lse = np.zeros((h, g))
    for j in range(h):
        out[j], lse[j] = attend_tokens(query.reshape(h, g, d)[j], keys[j], values[j], scaling)
    return out.reshape(-1, d), lse.reshape(-1)
