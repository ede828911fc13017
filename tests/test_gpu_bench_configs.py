"""Parity of the benchmark configurations with the CPU oracle.

The headline numbers of bench.py are measured on config 2 (a 512-token seeded
prompt, then greedy batch-1 decode from position 512) and config 3 (a
3840-token prompt, then decode up to the 4096-token limit). These tests run
exactly those inputs through the engine's C ABI and through the oracle's
restatement of the reference CPU path (engine/src/lfm.rs:290-694 forward,
engine/src/main.rs:174-195 greedy loop, f16-rounded K/V as with LFM_KV_F16=1).

Contract (as in the config-0 tests): every compared logits vector within
max-abs 1e-2 of the oracle's; the argmax equal wherever the oracle's top-2
margin exceeds twice the observed error (teacher_audit.rs:10-15); greedy token
streams identical when every step is decisive. Decode steps are teacher-forced
with the oracle's tokens, so one near-tie cannot desynchronise the rest.

The attention-boundary test walks one session to the decode positions where
the persistent step kernel's attention partition changes shape: 32-position
chunks, at most 32 tasks per KV head, 1-4 chunks per task (one chunk and its
ragged successor at 31/32; 32 single-chunk tasks at 1023; two chunks per task
from 1024; three from 2048; four from 3072), each step compared with the
oracle's f64 attention.
"""

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

TOL = 1e-2
NEVER = 0xFFFFFFFF  # an EOS id outside the vocabulary: greedy runs never stop early


def prompt(n, seed):
    """bench.py's seeded prompt (same generator and range)."""
    return np.random.default_rng(seed).integers(0, 128000, n).astype(np.uint32)


def margin(l):
    s = np.sort(l)[::-1]
    return float(s[0] - s[1])


def check_logits(got, ref, what):
    err = float(np.abs(got.astype(np.float64) - ref.astype(np.float64)).max())
    assert err <= TOL, f"{what}: max-abs {err}"
    if margin(ref) > 2 * err:
        assert int(np.argmax(got)) == int(np.argmax(ref)), f"{what}: argmax differs (margin {margin(ref)})"
    return err


@pytest.fixture(scope="module")
def engine(synth_model, cuda_lib):
    import lfm2_b200
    e = lfm2_b200.GpuEngine(synth_model, 0)
    e.set_ctx(4096)
    yield e
    e.close()


@pytest.fixture(scope="module")
def config2_oracle(synth_model, oracle_mod):
    """Config 2 on the oracle: prompt(512, 7), then 16 greedy tokens."""
    o = oracle_mod.OracleEngine(synth_model, kv_f16=True)
    try:
        o.set_ctx(4096)
        p = prompt(512, 7)
        toks, logits = o.greedy(p, 17, NEVER)
    finally:
        o.close()
    return p, toks, logits


def test_config2_prefill_and_teacher_forced_decode(engine, config2_oracle):
    p, otoks, ologits = config2_oracle
    engine.reset_session()
    check_logits(engine.forward(p, 0), ologits[0], "config 2 prefill (512 tokens)")
    for i in range(16):
        got = engine.forward(np.array([otoks[i]], np.uint32), 512 + i)
        check_logits(got, ologits[i + 1], f"config 2 decode at position {512 + i}")


def test_config2_greedy_tokens(engine, config2_oracle):
    """bench.py's timed loop (lfm_decode_loop after forward(prompt)) and the
    api_stream path (64-token forward_token chunks, then forward_token per
    step) both give the oracle's greedy tokens."""
    p, otoks, ologits = config2_oracle
    decisive = all(margin(ologits[i]) > 2 * TOL for i in range(len(otoks)))
    engine.reset_session()
    first = int(np.argmax(engine.forward(p, 0)))
    toks, _ = engine.decode_loop(first, 512, 16)
    stream = [first] + toks
    engine.reset_session()
    nxt = 0
    for off in range(0, 512, 64):
        nxt = engine.forward_token(p[off:off + 64], off)
    api = [nxt]
    for i in range(16):
        api.append(engine.forward_token(np.array([api[-1]], np.uint32), 512 + i))
    if decisive:
        assert stream == otoks[:17]
        assert api == otoks[:17]
    else:  # equal up to the first near-tie step
        k = next(i for i in range(len(otoks)) if margin(ologits[i]) <= 2 * TOL)
        assert stream[:k + 1] == otoks[:k + 1] and api[:k + 1] == otoks[:k + 1]


def test_config3_prefill_and_long_context_decode(engine, synth_model, oracle_mod):
    """Config 3: prompt(3840, 11) prefilled in one call, 8 teacher-forced
    decode steps at 3840..3847, a 244-token chunk at 3848..4091 through the
    prompt path with 3848 cached positions, then 4 decode steps ending at the
    4096-token limit (position 4095)."""
    p = prompt(3840, 11)
    chunk = prompt(244, 12)
    o = oracle_mod.OracleEngine(synth_model, kv_f16=True)
    try:
        o.set_ctx(4096)
        engine.reset_session()
        ref = o.forward(p, 0)
        check_logits(engine.forward(p, 0), ref, "config 3 prefill (3840 tokens)")
        for i in range(8):
            t = np.array([int(np.argmax(ref))], np.uint32)
            ref = o.forward(t, 3840 + i)
            check_logits(engine.forward(t, 3840 + i), ref, f"config 3 decode at position {3840 + i}")
        ref = o.forward(chunk, 3848)
        check_logits(engine.forward(chunk, 3848), ref, "244-token chunk at position 3848")
        for pos in range(4092, 4096):
            t = np.array([int(np.argmax(ref))], np.uint32)
            ref = o.forward(t, pos)
            check_logits(engine.forward(t, pos), ref, f"decode at position {pos}")
    finally:
        o.close()


def test_step_attention_partition_boundaries(engine, synth_model, oracle_mod):
    """Decode steps at 31/32 (one chunk, then a ragged second), 1023/1024
    (32 one-chunk tasks, then two chunks per task), 2048 (three) and 3072
    (four), the positions between them filled by prompt-path chunks."""
    o = oracle_mod.OracleEngine(synth_model, kv_f16=True)
    try:
        o.set_ctx(4096)
        engine.reset_session()
        pos, seed = 0, 300
        for stop in (31, 1023, 2048, 3072):
            if stop > pos:
                ids = prompt(stop - pos, seed)
                seed += 1
                ref = o.forward(ids, pos)
                check_logits(engine.forward(ids, pos), ref, f"chunk {pos}..{stop - 1}")
                pos = stop
            for _ in range(2):
                t = np.array([int(np.argmax(ref))], np.uint32)
                ref = o.forward(t, pos)
                check_logits(engine.forward(t, pos), ref, f"decode at position {pos}")
                pos += 1
    finally:
        o.close()
