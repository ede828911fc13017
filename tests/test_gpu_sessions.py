"""Independent sessions decoded together (lfm_batch_*) against the same
sessions run one at a time through the single-session path.

Contract: a session slot behaves like the reference's single session
(forward_token semantics, resident_graph.rs:90-101; sessions switched by
snapshot/restore in persistent.rs:164-176). Each session is prefilled with its
own prompt (the single-session prompt path, so first tokens and states are
identical), then all sessions advance one token per batched step. The batched
step computes every matrix as a multi-token tensor-core GEMM with hi/lo
activations (one padded 16-token tile below 16 sessions): logits within 1e-2
of the single-session decode kernel, the parity bar of the full model. Inputs are teacher-forced with the
single-session tokens so every step compares identical inputs; tokens must
agree wherever the single-session top-2 margin exceeds twice the tolerance.
"""

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def engine(synth_model, cuda_lib):
    import lfm2_b200
    e = lfm2_b200.GpuEngine(synth_model, 0)
    e.set_ctx(256)
    yield e
    e.close()


def _single(e, prompt, steps):
    e.reset_session()
    lg = e.forward(prompt, 0)
    toks, logits = [int(np.argmax(lg))], []
    pos = len(prompt)
    for _ in range(steps):
        lg = e.forward(np.array([toks[-1]], np.uint32), pos)
        logits.append(lg)
        toks.append(int(np.argmax(lg)))
        pos += 1
    return toks, logits


@pytest.mark.parametrize("n_sess,tol", [(5, 1e-2), (20, 1e-2)])
def test_batch_matches_single_sessions(engine, n_sess, tol):
    rng = np.random.default_rng(n_sess)
    steps = 6
    lens = rng.integers(5, 120, n_sess)
    prompts = [rng.integers(0, 128000, int(n)).astype(np.uint32) for n in lens]
    ref = [_single(engine, p, steps) for p in prompts]
    engine.batch_create(n_sess)
    firsts = [engine.batch_prefill(i, p) for i, p in enumerate(prompts)]
    assert firsts == [r[0][0] for r in ref]
    worst = 0.0
    for step in range(steps):
        toks = [r[0][step] for r in ref]
        pos = [len(p) + step for p in prompts]
        nxt = engine.batch_decode(np.arange(n_sess), toks, pos)
        for i in range(n_sess):
            lg = engine.batch_logits(i)
            rl = ref[i][1][step]
            d = float(np.abs(lg - rl).max())
            worst = max(worst, d)
            top = np.sort(rl)[-2:]
            if top[1] - top[0] > 2 * tol:
                assert int(nxt[i]) == ref[i][0][step + 1], (i, step)
    assert worst <= tol, worst


def test_batch_subset_and_order(engine):
    """A step may take any subset of sessions in any order; the others keep
    their state."""
    rng = np.random.default_rng(3)
    prompts = [rng.integers(0, 128000, n).astype(np.uint32) for n in (9, 30, 17)]
    ref = [_single(engine, p, 2) for p in prompts]
    engine.batch_create(3)
    for i, p in enumerate(prompts):
        engine.batch_prefill(i, p)
    # step 1: sessions 2 and 0 (reversed order); session 1 waits
    n1 = engine.batch_decode([2, 0], [ref[2][0][0], ref[0][0][0]], [len(prompts[2]), len(prompts[0])])
    assert list(n1) == [ref[2][0][1], ref[0][0][1]]
    # step 2: all three, session 1 at its first decode position
    n2 = engine.batch_decode([1, 0, 2], [ref[1][0][0], ref[0][0][1], ref[2][0][1]],
                             [len(prompts[1]), len(prompts[0]) + 1, len(prompts[2]) + 1])
    assert list(n2) == [ref[1][0][1], ref[0][0][2], ref[2][0][2]]


def test_batch_validation(engine):
    import lfm2_b200
    engine.batch_create(2)
    engine.batch_prefill(0, np.arange(1, 5, dtype=np.uint32))
    with pytest.raises(lfm2_b200.LfmError):
        engine.batch_decode([0, 0], [1, 1], [4, 4])  # duplicate session
    with pytest.raises(lfm2_b200.LfmError):
        engine.batch_decode([2], [1], [4])  # session out of range
    with pytest.raises(lfm2_b200.LfmError):
        engine.batch_decode([0], [1], [256])  # position beyond the context
    with pytest.raises(lfm2_b200.LfmError):
        engine.batch_prefill(5, np.arange(1, 5, dtype=np.uint32))
    # batch_logits takes only entries of the last batch_decode step
    with pytest.raises(lfm2_b200.LfmError, match="not an entry"):
        engine.batch_logits(0)  # no step yet
    engine.batch_decode([0], [1], [4])
    assert engine.batch_logits(0).shape == (128000,)
    with pytest.raises(lfm2_b200.LfmError, match="not an entry"):
        engine.batch_logits(1)  # a slot, but not an entry of that one-session step


def test_prefill_many_matches_one_by_one(engine):
    """lfm_batch_prefill_many (several prompts in one pass) leaves every
    session in the state the one-by-one prefill leaves it in: same next
    tokens, and a following batched decode step gives the same logits (the
    one-by-one path trims the last layer's FFN to the last token and runs it
    with the decode kernels, hence the 2e-3 bound)."""
    rng = np.random.default_rng(41)
    lens = [3, 70, 1, 129, 16]
    prompts = [rng.integers(0, 128000, n).astype(np.uint32) for n in lens]
    sess = [4, 0, 2, 1, 3]
    engine.batch_create(5)
    one = [engine.batch_prefill(s, p) for s, p in zip(sess, prompts)]
    pos = [len(p) for p in prompts]
    n1 = engine.batch_decode(sess, one, pos)
    l1 = [engine.batch_logits(i) for i in range(5)]
    engine.batch_create(5)
    many = engine.batch_prefill_many(sess, prompts)
    assert list(many) == one
    n2 = engine.batch_decode(sess, list(many), pos)
    l2 = [engine.batch_logits(i) for i in range(5)]
    worst = max(float(np.abs(a - b).max()) for a, b in zip(l1, l2))
    assert worst <= 2e-3, worst
    assert list(n1) == list(n2)
