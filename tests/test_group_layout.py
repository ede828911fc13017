"""The grouped-GEMM operand layout, restated on CPU: the per-row placement
that the grid-parallel layout kernel computes (for operand row r, the last
expert whose tile-aligned base is <= r, then entry r - base or padding) must
equal the sequential layout (experts' rows one after another, each run padded
to a multiple of the token tile), including experts with no tokens."""

import numpy as np
import pytest

N_EXPERT = 32


def _sequential(counts, slots_of, tt, rpad):
    slots, rowof, tiles, base = [-1] * rpad, {}, [], 0
    for e in range(N_EXPERT):
        for i, sl in enumerate(slots_of[e]):
            slots[base + i] = sl
            rowof[sl] = base + i
        nt = (counts[e] + tt - 1) // tt
        tiles += [(e, base + tt * k) for k in range(nt)]
        base += nt * tt
    return slots, rowof, tiles


def _per_row(counts, slots_of, tt, rpad):
    nt = [(c + tt - 1) // tt for c in counts]
    base = np.concatenate([[0], np.cumsum([n * tt for n in nt])])
    tile0 = np.concatenate([[0], np.cumsum(nt)])
    tiles = []
    for i in range(int(tile0[-1])):
        e = 0
        while tile0[e + 1] <= i:
            e += 1
        tiles.append((e, int(base[e] + tt * (i - tile0[e]))))
    slots, rowof = [-1] * rpad, {}
    for r in range(rpad):
        if r >= base[-1]:
            continue
        lo, hi = 0, N_EXPERT - 1
        while lo < hi:
            mid = (lo + hi + 1) >> 1
            if base[mid] <= r:
                lo = mid
            else:
                hi = mid - 1
        i = r - base[lo]
        if i < counts[lo]:
            slots[r] = slots_of[lo][i]
            rowof[slots_of[lo][i]] = r
    return slots, rowof, tiles


@pytest.mark.parametrize("seed,n,tt", [(0, 1, 16), (1, 7, 16), (2, 64, 16), (3, 300, 32), (4, 1024, 128), (5, 3840, 128)])
def test_per_row_layout_equals_sequential(seed, n, tt):
    rng = np.random.default_rng(seed)
    # each token picks 4 distinct experts; skew the choice so some experts get none
    weights = rng.random(N_EXPERT) ** 4
    slots_of = [[] for _ in range(N_EXPERT)]
    for tok in range(n):
        ex = rng.choice(N_EXPERT, 4, replace=False, p=weights / weights.sum())
        for rank, e in enumerate(ex):
            slots_of[e].append(tok * 4 + rank)
    counts = [len(s) for s in slots_of]
    rpad = n * 4 + N_EXPERT * tt
    a = _sequential(counts, slots_of, tt, rpad)
    b = _per_row(counts, slots_of, tt, rpad)
    assert a == b
    assert len(a[1]) == n * 4  # every slot has an operand row
