"""Prompt lengths around the tensor-core GEMM's tile boundaries against the
CPU oracle.

The prompt path picks a token tile of 16/32/64/128 tokens per GEMM (the
smallest holding the prompt, or for the routed experts the average expert's
share), splits single-tile GEMMs over K, and pads the last tile; attention
walks 128-position key tiles. Lengths just past each boundary exercise the
padding and the split; prompts of 2-15 tokens run in one padded 16-token tile. Contract as in the full-model tests (lfm.rs forward,
main.rs:174-195): last-token logits max-abs <= 1e-2 against the oracle, same
argmax wherever the oracle's top-2 margin exceeds twice the observed error.
"""

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

TOL = 1e-2


@pytest.fixture(scope="module")
def engine(synth_model, cuda_lib):
    import lfm2_b200
    e = lfm2_b200.GpuEngine(synth_model, 0)
    yield e
    e.close()


@pytest.mark.parametrize("n", [2, 4, 8, 15, 17, 33, 65, 129, 200])
def test_prefill_logits_vs_oracle(engine, synth_model, oracle_mod, n):
    p = np.random.default_rng(1000 + n).integers(0, 128000, n).astype(np.uint32)
    o = oracle_mod.OracleEngine(synth_model, kv_f16=True)
    try:
        o.set_ctx(n + 16)
        ref = o.forward(p, 0)
    finally:
        o.close()
    engine.set_ctx(n + 16)
    engine.reset_session()
    got = engine.forward(p, 0)
    err = float(np.abs(got - ref).max())
    assert err <= TOL, err
    top = np.sort(ref)[-2:]
    if top[1] - top[0] > 2 * err:
        assert int(np.argmax(got)) == int(np.argmax(ref))


def test_expanded_weights_bit_identical(engine, synth_model):
    """The prompt GEMMs over load-time expanded fp16 weights (the default)
    compute exactly what the on-chip dequantising GEMMs compute
    (LFM_PREFILL_X16=0): same A operand values, MMAs and fold."""
    import os

    import lfm2_b200
    old = os.environ.get("LFM_PREFILL_X16")
    os.environ["LFM_PREFILL_X16"] = "0"
    try:
        plain = lfm2_b200.GpuEngine(synth_model, 0)
    finally:
        if old is None:
            del os.environ["LFM_PREFILL_X16"]
        else:
            os.environ["LFM_PREFILL_X16"] = old
    try:
        for n in (2, 17, 200, 1000):
            p = np.random.default_rng(2000 + n).integers(0, 128000, n).astype(np.uint32)
            outs = []
            for e in (engine, plain):
                e.set_ctx(1024 + 16)
                e.reset_session()
                outs.append(e.forward(p, 0))
            assert np.array_equal(outs[0].view(np.uint32), outs[1].view(np.uint32)), n
    finally:
        plain.close()
