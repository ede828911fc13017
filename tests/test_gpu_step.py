"""The persistent decode step (one cooperative kernel per token, the default;
LFM_STEP=0 selects the kernel chain) against the CPU oracle and against the
kernel chain.

Same contract as the full-model tests (engine/src/main.rs:174-195 greedy loop,
identical tokens, per-step logits max-abs <= 1e-2), plus: a long
device-resident decode loop gives the same tokens as the kernel chain, and the
per-stage trace record is well formed.
"""

import os

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

LOGIT_TOL = 1e-2
PROMPT_LEN, N_GEN, EOS = 16, 8, 7


def _engine(path, step):
    import lfm2_b200
    old = os.environ.get("LFM_STEP")
    os.environ["LFM_STEP"] = "1" if step else "0"
    try:
        return lfm2_b200.GpuEngine(path, 0)
    finally:
        if old is None:
            del os.environ["LFM_STEP"]
        else:
            os.environ["LFM_STEP"] = old


@pytest.fixture(scope="module")
def step_engine(synth_model, cuda_lib):
    e = _engine(synth_model, True)
    yield e
    e.close()


def test_step_path_selected(step_engine):
    step_engine.set_ctx(64)
    step_engine.forward(np.array([1, 2, 3], np.uint32), 0)
    info = step_engine.info()
    assert info["decode_path"] == "persistent-step", info
    # embed; per layer mixer (QKV, ATTN, RESID or CONV, RESID) + FFN (SWIGLU,
    # DOWN28 or XSWIGLU, XDOWN: routing is folded into the residual stage); lm_head
    assert info["step_stages"] == 1 + 6 * 3 + 18 * 2 + 2 * 2 + 22 * 2 + 1


@pytest.fixture(scope="module")
def oracle_greedy(synth_model, oracle_mod):
    p = np.random.default_rng(0).integers(0, 128000, PROMPT_LEN).astype(np.uint32)
    o = oracle_mod.OracleEngine(synth_model, kv_f16=True)
    o.set_ctx(PROMPT_LEN + N_GEN + 16)
    otoks, ologits = o.greedy(p, N_GEN, EOS)
    o.close()
    return p, otoks, ologits


def _greedy_matches(e, oracle_greedy):
    p, otoks, ologits = oracle_greedy
    e.set_ctx(PROMPT_LEN + N_GEN + 16)
    e.reset_session()
    logits = [e.forward(p, 0)]
    toks = []
    for step in range(N_GEN):
        t = int(np.argmax(logits[-1]))
        if t == EOS:
            break
        toks.append(t)
        logits.append(e.forward(np.array([t], np.uint32), PROMPT_LEN + step))
    assert toks == otoks
    g = np.stack(logits)
    assert g.shape == ologits.shape
    assert np.abs(g - ologits).max() <= LOGIT_TOL


def test_step_greedy_matches_oracle(step_engine, oracle_greedy):
    _greedy_matches(step_engine, oracle_greedy)


def test_chain_greedy_matches_oracle(synth_model, cuda_lib, oracle_greedy):
    """The kernel chain (LFM_STEP=0) on the same contract."""
    e = _engine(synth_model, False)
    try:
        _greedy_matches(e, oracle_greedy)
        assert e.info()["decode_path"].startswith("kernel-chain")
    finally:
        e.close()


def test_step_decode_loop_matches_chain(step_engine, synth_model):
    p = np.random.default_rng(7).integers(0, 128000, 64).astype(np.uint32)
    chain = _engine(synth_model, False)
    try:
        runs = []
        for e in (step_engine, chain):
            e.set_ctx(256)
            e.reset_session()
            first = int(np.argmax(e.forward(p, 0)))
            toks, ms = e.decode_loop(first, len(p), 48)
            assert ms > 0
            runs.append(toks)
        assert chain.info()["decode_path"].startswith("kernel-chain")
        assert runs[0] == runs[1]
    finally:
        chain.close()


def test_step_trace_record(step_engine):
    e = step_engine
    e.set_ctx(64)
    e.reset_session()
    first = int(np.argmax(e.forward(np.arange(1, 9, dtype=np.uint32), 0)))
    e.step_trace(True)
    e.decode_loop(first, 8, 2)
    tr = e.step_trace(False)
    ns = e.info()["step_stages"]
    assert tr is not None and tr.shape[0] == ns and tr.shape[2] == 8
    start, done = tr[:, :, 0].astype(np.int64), tr[:, :, 3].astype(np.int64)
    assert (start > 0).all() and (done >= start).all()
    # every CTA starts stage s+1 only after the whole grid finished stage s
    assert (start[1:].min(axis=1) >= done[:-1].min(axis=1)).all()
    # ring stages report their tile counts; their sum over CTAs is the stage's tile count
    assert tr[-1, :, 5].sum() == 128000 // 16


def test_step_long_context_matches_chain(step_engine, synth_model):
    """Config 3's tail: greedy decode from position 3840 to the 4096-token
    limit, persistent step vs kernel chain (two independent decode paths over
    the same prefilled state: identical tokens)."""
    p = np.random.default_rng(11).integers(0, 128000, 3840).astype(np.uint32)
    chain = _engine(synth_model, False)
    try:
        runs = []
        for e in (step_engine, chain):
            e.set_ctx(4096)
            e.reset_session()
            first = int(np.argmax(e.forward(p, 0)))
            toks, _ = e.decode_loop(first, len(p), 4096 - len(p))
            runs.append([first] + toks)
        assert runs[0] == runs[1]
    finally:
        chain.close()
