"""The decode step's attention split, restated on CPU: for a position pos the
32-position chunks 0..pos/32 are dealt to at most 32 tasks per KV head, each
task runs an online softmax over its chunks, and the last task merges the
partials. Checks that every position is covered once, the task bounds the
kernel relies on (at most 4 chunks per task, at most 32 tasks), and that the
merged output equals a direct softmax-weighted sum."""

import numpy as np
import pytest

SPLIT, MAX_CPT, MAX_TASKS = 32, 4, 32


def _tasks(pos):
    nchunk = pos // SPLIT + 1
    cpt = (nchunk + 31) // 32
    nth = (nchunk + cpt - 1) // cpt
    return [(j * cpt, min(j * cpt + cpt, nchunk)) for j in range(nth)], cpt


@pytest.mark.parametrize("pos", [0, 1, 31, 32, 511, 1023, 1024, 2047, 3899, 4095])
def test_partition_and_merge(pos):
    tasks, cpt = _tasks(pos)
    assert cpt <= MAX_CPT and len(tasks) <= MAX_TASKS
    covered = [t for c0, c1 in tasks for c in range(c0, c1) for t in range(c * SPLIT, min(c * SPLIT + SPLIT, pos + 1))]
    assert covered == list(range(pos + 1))

    rng = np.random.default_rng(pos)
    s = rng.standard_normal(pos + 1) * 3.0  # scores of one head
    v = rng.standard_normal((pos + 1, 64))
    parts = []
    for c0, c1 in tasks:
        m, l, o = -np.inf, 0.0, np.zeros(64)
        for c in range(c0, c1):
            t = np.arange(c * SPLIT, min(c * SPLIT + SPLIT, pos + 1))
            mn = max(m, s[t].max())
            scale = np.exp(m - mn)  # 0 on the first chunk
            p = np.exp(s[t] - mn)
            l = l * scale + p.sum()
            o = o * scale + p @ v[t]
            m = mn
        parts.append((m, l, o))
    M = max(m for m, _, _ in parts)
    w = [np.exp(m - M) for m, _, _ in parts]
    L = sum(l * wi for (_, l, _), wi in zip(parts, w))
    out = sum(o * wi for (_, _, o), wi in zip(parts, w)) / L
    ref = np.exp(s - s.max()) @ v / np.exp(s - s.max()).sum()
    assert np.allclose(out, ref, rtol=1e-12, atol=1e-12)
