"""Host side of ragged batching, without a GPU: the score kernel's chunk list and the attention's
CTA schedule (lkv_ragged_schedule is plain C in the library)."""

from __future__ import annotations

import numpy as np
import pytest


def test_work_list_covers_every_candidate_once_in_chunks() -> None:
    from lazykv_b200.ragged import CHUNK, work_list

    n_cand = np.array([1, CHUNK - 1, CHUNK, CHUNK + 1, 600, 8191])
    work = work_list(n_cand)
    want = [(r, c) for r in range(len(n_cand)) for c in range(0, int(n_cand[r]), CHUNK)]
    assert work.dtype == np.int32 and [tuple(x) for x in work.tolist()] == want


@pytest.mark.parametrize("n_sms", [1, 148])
def test_schedule_gives_each_row_its_ctas_and_partials(n_sms: int) -> None:
    from lazykv_b200.ragged import schedule

    rng = np.random.default_rng(0)
    items = np.concatenate([[3, 64, 65], rng.integers(3, 8194, size=509)]).astype(np.int32)  # config 3's rows and the edges
    sched, n_parts = schedule(items, n_sms)
    rows, idx, per, base = sched.T
    assert np.array_equal(np.unique(rows), np.arange(len(items)))  # every row, in order
    assert np.all(np.diff(rows) >= 0)
    for r in (0, 1, 2, 100, len(items) - 1):
        mine = sched[rows == r]
        P = mine[0, 2]
        assert len(mine) == P and np.array_equal(mine[:, 1], np.arange(P)) and np.all(mine[:, 2] == P)
        # a CTA's share of each of the two segments is at most ceil(n / P): list capacity 3072
        assert -(-int(items[r]) // P) + 2 <= 3072
    # partials: each row's block starts where the previous row's ended
    first = sched[np.r_[True, np.diff(rows) != 0]]
    assert np.array_equal(first[:, 3], np.r_[0, np.cumsum(first[:-1, 2])]) and n_parts == first[:, 2].sum()
    assert np.array_equal(base, first[rows, 3])


def test_schedule_rejects_a_negative_row() -> None:
    from lazykv_b200._lib import LkvError
    from lazykv_b200.ragged import schedule

    with pytest.raises(LkvError, match="items"):
        schedule(np.array([5, -1], dtype=np.int32), 148)
