"""Full-model parity of the B200 engine with the CPU oracle.

Synthetic seeded LFM2.5-8B-A1B Q6_K model; a 16-token seeded prompt, 8 greedy
tokens, run through the oracle's `--cpu --tokens` loop (engine/src/main.rs:
174-195) with f16-rounded K/V (LFM_KV_F16=1 semantics) and through the engine's
C ABI. Contract: identical greedy tokens, per-step logits max-abs <= 1e-2, and a
margin audit (teacher_audit.rs:10-15: a step is only decisive when
2 * max_abs < top1 - top2).
"""

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

LOGIT_TOL = 1e-2
PROMPT_LEN, N_GEN, EOS = 16, 8, 7


def prompt_ids(seed=0, n=PROMPT_LEN):
    return np.random.default_rng(seed).integers(0, 128000, n).astype(np.uint32)


@pytest.fixture(scope="module")
def engine(synth_model, cuda_lib):
    import lfm2_b200
    e = lfm2_b200.GpuEngine(synth_model, 0)
    yield e
    e.close()


@pytest.fixture(scope="module")
def oracle_run(synth_model, oracle_mod):
    o = oracle_mod.OracleEngine(synth_model, kv_f16=True)
    p = prompt_ids()
    o.set_ctx(PROMPT_LEN + N_GEN + 16)
    toks, logits = o.greedy(p, N_GEN, EOS)
    snap = o.snapshot(PROMPT_LEN + len(toks))
    o.close()
    return p, toks, logits, snap


def gpu_greedy(engine, prompt, n, eos):
    """main.rs:174-195 on the engine: forward(prompt, 0) then forward([t], pos)."""
    engine.set_ctx(len(prompt) + n + 16)
    engine.reset_session()
    logits = [engine.forward(prompt, 0)]
    toks = []
    for step in range(n):
        t = int(np.argmax(logits[-1]))
        if t == eos:
            break
        toks.append(t)
        logits.append(engine.forward(np.array([t], np.uint32), len(prompt) + step))
    return toks, np.stack(logits)


def margin(l):
    s = np.sort(l)[::-1]
    return float(s[0] - s[1])


def test_config0_tokens_and_logits(engine, oracle_run):
    p, otoks, ologits, _ = oracle_run
    gtoks, glogits = gpu_greedy(engine, p, N_GEN, EOS)
    steps = min(len(ologits), len(glogits))
    report = []
    for s in range(steps):
        d = np.abs(glogits[s].astype(np.float64) - ologits[s].astype(np.float64))
        rel = np.sqrt((d ** 2).sum() / (ologits[s].astype(np.float64) ** 2).sum())
        report.append((s, float(d.max()), float(rel), margin(ologits[s])))
    for s, mx, rel, mg in report:
        assert mx <= LOGIT_TOL, f"step {s}: max-abs {mx} rel-L2 {rel} margin {mg}"
        assert 2 * mx < mg, f"step {s}: near tie (margin {mg}, max-abs {mx})"
    assert gtoks == otoks, (gtoks, otoks, report)


def test_forward_token_path_matches(engine, oracle_run):
    """api_stream.rs:55-77: reset, 64-token prefill chunks via forward_token
    (device argmax), then decode via forward_token."""
    p, otoks, _, _ = oracle_run
    engine.set_ctx(4096)
    engine.reset_session()
    nxt = engine.forward_token(p, 0)
    pos, out = len(p), []
    for _ in range(N_GEN):
        if nxt == EOS:
            break
        out.append(nxt)
        nxt = engine.forward_token(np.array([nxt], np.uint32), pos)
        pos += 1
    assert out == otoks
    c = engine.counters()
    assert c["graph_replays"] > 0 and c["gpu_argmax"] > 0


def test_generate_matches(engine, oracle_run):
    p, otoks, _, _ = oracle_run
    engine.set_ctx(4096)
    engine.reset_session()
    assert engine.generate(p, N_GEN, EOS) == otoks


def test_chunked_prefill_matches_single(engine):
    """A 100-token prompt prefilled in one forward vs 64 + 36 chunks."""
    p = prompt_ids(3, 100)
    engine.set_ctx(4096)
    engine.reset_session()
    a = engine.forward(p, 0)
    engine.reset_session()
    engine.forward(p[:64], 0)
    b = engine.forward(p[64:], 64)
    assert np.abs(a - b).max() < 1e-3
    assert int(np.argmax(a)) == int(np.argmax(b))


def test_replay_is_deterministic(engine):
    """replay_state_check.rs: the same session twice gives bit-equal logits."""
    p = prompt_ids(5, 12)
    runs = []
    for _ in range(2):
        engine.set_ctx(64)
        engine.reset_session()
        l0 = engine.forward(p, 0)
        t = int(np.argmax(l0))
        l1 = engine.forward(np.array([t], np.uint32), len(p))
        l2 = engine.forward(np.array([int(np.argmax(l1))], np.uint32), len(p) + 1)
        runs.append(np.stack([l0, l1, l2]))
    assert np.array_equal(runs[0].view(np.uint32), runs[1].view(np.uint32))
    assert np.array_equal(engine.snapshot_resident_logits(), runs[1][2])


def test_snapshot_matches_oracle_state(engine, oracle_run):
    p, otoks, _, osnap = oracle_run
    gpu_greedy(engine, p, N_GEN, EOS)
    valid = PROMPT_LEN + len(otoks)
    g = np.frombuffer(engine.snapshot_resident_cache(valid), dtype=np.float32)
    assert g.size == osnap.size
    d = np.abs(g.astype(np.float64) - osnap.astype(np.float64))
    # K/V are fp16 values; conv state f32: agreement to the logit tolerance
    assert d.max() < 5e-2, d.max()
    assert np.sqrt((d ** 2).sum() / (osnap.astype(np.float64) ** 2).sum()) < 1e-3


def test_snapshot_restore_roundtrip(engine):
    """persistent.rs sessions: snapshot after a prefill, run something else,
    restore, continue: same tokens as the uninterrupted session."""
    p = prompt_ids(7, 20)
    engine.set_ctx(128)
    engine.reset_session()
    nxt = engine.forward_token(p, 0)
    snap = engine.snapshot_resident_cache(len(p))
    straight = []
    t, pos = nxt, len(p)
    for _ in range(4):
        straight.append(t)
        t = engine.forward_token(np.array([t], np.uint32), pos)
        pos += 1
    engine.reset_session()
    engine.forward_token(prompt_ids(8, 30), 0)
    engine.restore_session(len(p), snap)
    resumed = []
    t, pos = nxt, len(p)
    for _ in range(4):
        resumed.append(t)
        t = engine.forward_token(np.array([t], np.uint32), pos)
        pos += 1
    assert resumed == straight
    with pytest.raises(Exception):
        engine.restore_session(len(p), snap[:-4])  # truncated snapshot


def test_validation_errors(engine):
    import lfm2_b200
    engine.set_ctx(32)
    with pytest.raises(lfm2_b200.LfmError, match="token out of range"):
        engine.forward(np.array([128000], np.uint32), 0)
    with pytest.raises(lfm2_b200.LfmError, match="context"):
        engine.forward(prompt_ids(1, 8), 30)
    with pytest.raises(lfm2_b200.LfmError, match="1..64"):
        engine.forward_token(prompt_ids(1, 65), 0)
    with pytest.raises(lfm2_b200.LfmError):
        engine.set_ctx(5000)
    # the engine still works afterwards
    engine.set_ctx(64)
    engine.reset_session()
    assert 0 <= engine.forward_token(prompt_ids(2, 4), 0) < 128000
