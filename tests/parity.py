"""Shared parity helpers: golden fixtures, ulp distances and the index-list comparison rule."""

from __future__ import annotations

from pathlib import Path

import numpy as np

GOLDEN = Path(__file__).resolve().parent / "golden"


def golden(name: str) -> dict[str, np.ndarray]:
    with np.load(GOLDEN / f"{name}.npz") as z:
        return {k: z[k] for k in z.files}


def f32_ulp_diff(a: np.ndarray, b: np.ndarray) -> np.ndarray:
    """Distance in float32 units in the last place (monotone integer map of the bit patterns)."""

    def key(x: np.ndarray) -> np.ndarray:
        i = np.ascontiguousarray(x, dtype=np.float32).view(np.int32).astype(np.int64)
        return np.where(i < 0, -(i & 0x7FFFFFFF), i)

    return np.abs(key(a) - key(b))


def bf16_ulp_diff(a: np.ndarray, b: np.ndarray) -> np.ndarray:
    """Distance in bf16 units in the last place between two arrays of bf16 values (as float32)."""
    return f32_ulp_diff(a, b) >> 16


def bf16_close(got: np.ndarray, want: np.ndarray, tol: float = 2e-5) -> bool:
    """A bf16 result is the bf16 rounding of a value within `tol` (relative to max|want|) of `want`:
    |got - want| <= 2^-8 |want| (half a bf16 unit) + tol * max|want|, elementwise."""
    got = np.asarray(got, np.float64)
    want = np.asarray(want, np.float64)
    return bool(np.all(np.abs(got - want) <= 2.0**-8 * np.abs(want) + tol * np.abs(want).max()))


def index_parity(ours: np.ndarray, ref: np.ndarray, bound: np.ndarray, tie_tol: float = 0.0) -> dict[str, int]:
    """Compare two top-K index lists [h, K] (candidate ids) under the tie rule.

    Lists must agree position by position, except that a position may differ where both entries'
    bounds are within `tie_tol` of the K-th bound of that head (an exact tie when `tie_tol` is 0).
    Returns counts; `bad` must be 0.
    """
    h, k = ours.shape
    exact = 0
    tie = 0
    bad = 0
    for j in range(h):
        kth = np.sort(bound[j])[::-1][k - 1]
        near = lambda b: abs(float(bound[j][b]) - float(kth)) <= tie_tol  # noqa: E731
        so, sr = set(ours[j].tolist()), set(ref[j].tolist())
        for b in so ^ sr:
            if not near(b):
                bad += 1
        for p in range(k):
            if ours[j, p] == ref[j, p]:
                exact += 1
            elif near(ours[j, p]) or near(ref[j, p]) or bound[j][ours[j, p]] == bound[j][ref[j, p]]:
                tie += 1
            else:
                bad += 1
    return {"exact": exact, "tie": tie, "bad": bad}


def lru_admit(chosen: np.ndarray, block_slot: np.ndarray, slot_block: np.ndarray, last_used: np.ndarray, evicted_at: np.ndarray,
              step: int) -> list[np.ndarray]:
    """The reference's admit rule (lazykv/tiered.py:389-463) per head on the host, updating the
    tables in place: chosen blocks not in a slot miss; victims are the slots not holding a chosen
    block, by (last_used, slot); misses take them in chosen order; every chosen slot is used at this
    step. -1 entries are padding. Returns each head's misses in chosen order."""
    misses = []
    for j in range(chosen.shape[0]):
        ch = chosen[j][chosen[j] >= 0]
        cur = block_slot[j, ch]
        kept = set((cur[cur >= 1] - 1).tolist())
        free = sorted((s for s in range(slot_block.shape[1]) if s not in kept), key=lambda s: (last_used[j, s], s))
        miss = [int(b) for b, c in zip(ch, cur) if c < 1]
        for i, b in enumerate(miss):
            v = free[i]
            old = slot_block[j, v]
            if old >= 0:
                block_slot[j, old] = -1
                evicted_at[j, old] = step
            slot_block[j, v] = b
            block_slot[j, b] = v + 1
        for b in ch:
            last_used[j, block_slot[j, b] - 1] = step
        misses.append(np.array(miss, dtype=np.int64))
    return misses
