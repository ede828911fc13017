"""Pin the CPU oracle to the reference's own known-answer tests (CPU only).

Each test restates a reference test and its vectors:
  engine/src/q6k.rs:199-290          fp16 round trip, known Q6_K blocks, matvec consistency
  engine/tests/dequant_mirror.rs     512 xorshift blocks, bit-exact byte-addressed dequant
  engine/src/main.rs:287-317         lane argmax == scalar argmax incl. ties, NaN, +-inf, tails
  engine/src/bin/resident_check.rs:35-84   router order / stable ties / probabilities (1e-6)
  engine/src/kernels/resident.rs:119-145   integer f32->f16 RNE used for the K/V cache
"""

import struct

import numpy as np
import pytest


def test_fp16_roundtrip(oracle_mod):
    # q6k.rs:199-204
    for v in (1.0, -2.5):
        assert oracle_mod.f16_bits_to_f32(oracle_mod.f32_to_f16_bits(v)) == v


def _block(d_bits: int, scales=1):
    b = np.zeros(210, dtype=np.uint8)
    b[208] = d_bits & 0xFF
    b[209] = d_bits >> 8
    b[192:208] = scales
    return b


def test_dequant_single_known_block(oracle_mod):
    # q6k.rs:206-235: d = 1.0, all scales +1, ql[0] low nibble 5 -> -27.
    b = _block(0x3C00)
    b[0] = 0x05
    out = oracle_mod.dequant_blocks(b)
    assert out[0] == -27.0
    for k in (64, 32, 96, 16, 48, 80, 112):
        assert out[k] == -32.0


def test_dequant_scale_and_d(oracle_mod):
    # q6k.rs:238-250: d = 2.0, ql[0] = 15 -> 2 * 1 * -17 = -34.
    b = _block(0x4000)
    b[0] = 0x0F
    assert oracle_mod.dequant_blocks(b)[0] == -34.0


def test_matvec_consistency(oracle_mod):
    # q6k.rs:253-290: 256x4, one block per row, f64 accumulation.
    w = np.zeros(4 * 210, dtype=np.uint8)
    for o in range(4):
        off = o * 210
        w[off + 208], w[off + 209] = 0x00, 0x3C
        w[off + 192: off + 208] = 1
        w[off] = o + 1
    x = np.array([(i % 7) * 0.5 for i in range(256)], dtype=np.float32)
    out = oracle_mod.q6k_matvec_f64(w, 256, 4, x)
    rows = oracle_mod.dequant_blocks(w).reshape(4, 256)
    expect = np.array([np.float32(np.sum(rows[o].astype(np.float64) * x.astype(np.float64))) for o in range(4)])
    assert np.array_equal(out, expect)


def _xorshift_blocks(n=512):
    """engine/tests/dequant_mirror.rs:51-74 (same PRNG, same forced bytes)."""
    s = 0x9E3779B97F4A7C15
    M = (1 << 64) - 1
    blocks = []
    for _ in range(n):
        b = np.empty(210, dtype=np.uint8)
        for i in range(210):
            s ^= (s << 13) & M
            s ^= s >> 7
            s ^= (s << 17) & M
            b[i] = (s >> 11) & 0xFF
        b[208], b[209] = 0x00, 0x3B
        b[192], b[193], b[200] = 0x80, 0xFF, 0x9C
        blocks.append(b)
    return np.stack(blocks)


def test_dequant_mirror_bit_exact(oracle_mod):
    blocks = _xorshift_blocks()
    ref = oracle_mod.dequant_blocks(blocks.reshape(-1)).reshape(-1, 256)
    mism = 0
    for i in range(len(blocks)):
        for k in range(256):
            m = oracle_mod.shader_dequant(blocks[i], k)
            if np.float32(m).view(np.uint32) != ref[i, k].view(np.uint32):
                mism += 1
    assert mism == 0
    # the forced -128 / -1 / -100 scale groups are exercised
    assert (ref[:, 0:16] != 0).any()


def _argmax_scalar(xs):
    best, value = 0, -np.inf
    for i, v in enumerate(xs):
        if v > value:
            best, value = i, v
    return best


def test_lane_argmax_matches_scalar(oracle_mod):
    # main.rs:287-317
    seed = 17
    for n in range(257):
        xs = []
        for _ in range(n):
            seed = (seed * 1664525 + 1013904223) & 0xFFFFFFFF
            xs.append(seed)
        a = np.array(xs, dtype=np.uint32).view(np.float32)
        with np.errstate(invalid="ignore"):
            assert oracle_mod.argmax(a) == _argmax_scalar(a)
            for v in (np.nan, -np.inf, np.inf, 0.0, -0.0, 1.0):
                a2 = np.full(n, v, dtype=np.float32)
                assert oracle_mod.argmax(a2) == _argmax_scalar(a2)
        if n > 8:
            # the reference's xs is all 1.0 here (last fill value)
            a = np.full(n, 1.0, dtype=np.float32)
            a[7] = 2.0
            a[8] = 2.0
            assert oracle_mod.argmax(a) == 7


@pytest.mark.parametrize("experts", [4, 32, 64])
def test_route_semantics(oracle_mod, experts):
    # resident_check.rs:35-84: token 0 all-zero logits (full ties), others varied.
    n = 3
    logits = np.array([0.0 if i < experts else ((i * 13 % 19) - 9) / 8.0 for i in range(n * experts)],
                      dtype=np.float32)
    bias = np.zeros(experts, dtype=np.float32)
    for j in range(n):
        lg = logits[j * experts:(j + 1) * experts]
        p = (1.0 / (1.0 + np.exp(-lg.astype(np.float32)))).astype(np.float32)
        ids = sorted(range(experts), key=lambda i: (-p[i], i))
        s = np.float32(0.0)
        for i in ids[:4]:
            s = np.float32(s + p[i])
        s = max(s, np.float32(6.103515625e-5))
        sel, w = oracle_mod.route(lg, bias)
        assert list(sel) == ids[:4]
        for r in range(4):
            assert abs(w[r] - p[ids[r]] / s) < 1e-6


def _half_round_bits(x: float) -> int:
    """kernels/resident.rs:119-145, the reference's integer f32->f16 RNE."""
    bits = struct.unpack("<I", struct.pack("<f", x))[0]
    M = 0xFFFFFFFF
    sign = (bits >> 16) & 0x8000
    mag = bits & 0x7FFFFFFF
    exp = mag >> 23
    rounded = (mag + 0xFFF + ((mag >> 13) & 1)) & M
    normal = ((rounded - 0x38000000) & M) >> 13
    shift = (126 - exp) & 31
    mant = (mag & 0x7FFFFF) | 0x800000
    base = mant >> shift
    rem = mant & (((1 << shift) - 1) & M)
    halfway = (1 << ((shift - 1) & 31)) & M
    inc = 1 if (halfway < rem or (rem == halfway and (base & 1) == 1)) else 0
    sub = 0 if exp < 102 else base + inc
    finite = sub if exp < 113 else (0x7C00 if rounded >= 0x47800000 else normal)
    nan = 0x7E00 | ((mag >> 13) & 0x3FF)
    res = nan if 0x7F800000 < mag else finite
    return (sign | res) & 0xFFFF


def test_f16_rne_matches_reference_integer_rounding(oracle_mod):
    rng = np.random.default_rng(5)
    vals = []
    for e in range(90, 160):  # through subnormal, normal and overflow ranges
        for m in rng.integers(0, 1 << 23, size=24):
            for s in (0, 1):
                vals.append((s << 31) | (e << 23) | int(m))
    # exact halfway cases around the subnormal and normal boundaries
    for e in (102, 103, 112, 113, 120):
        vals.append((e << 23) | 0x1000)
        vals.append((e << 23) | 0x3000)
    for b in vals:
        x = struct.unpack("<f", struct.pack("<I", b & 0xFFFFFFFF))[0]
        got = oracle_mod.f32_to_f16_bits(x)
        assert got == _half_round_bits(x), hex(b)
        # and IEEE RNE as numpy implements it
        assert got == int(np.array([x], dtype=np.float32).astype(np.float16).view(np.uint16)[0]), hex(b)


def test_threaded_matmul_is_bit_identical_to_one_thread(oracle_mod):
    # The CPU baseline runs the oracle on every host core; threads split output
    # rows only, so each row's sum keeps its order and the results must not
    # change with the thread count.
    rng = np.random.default_rng(5)
    in_dim, out_dim, n = 2048, 256, 3
    w = rng.integers(0, 256, out_dim * (in_dim // 256) * 210, dtype=np.uint8).reshape(-1, 210)
    w[:, 208], w[:, 209] = 0x00, 0x1C  # small fp16 d
    x = rng.standard_normal(in_dim * n).astype(np.float32)
    L = oracle_mod.lib()
    before = L.oracle_num_threads()
    try:
        L.oracle_set_threads(1)
        one = oracle_mod.q6k_matmul_f32(w.ravel(), in_dim, out_dim, x, n)
        L.oracle_set_threads(4)
        four = oracle_mod.q6k_matmul_f32(w.ravel(), in_dim, out_dim, x, n)
    finally:
        L.oracle_set_threads(before)
    assert np.isfinite(one).all()
    assert np.array_equal(one, four)


def _rank_top4(score):
    """The decode step's selection rule, restated: every expert's rank is the
    number of experts with a higher score plus the lower-indexed experts with
    an equal one (a NaN score ranks last); ranks 0..3 are picked in order."""
    s = np.where(np.isnan(score), -np.inf, score).astype(np.float32)
    n = s.size
    rank = [int(np.sum(s > s[i]) + np.sum(s[:i] == s[i])) for i in range(n)]
    assert sorted(rank) == list(range(n))  # a permutation: one expert per rank
    return [rank.index(r) for r in range(4)]


@pytest.mark.parametrize("seed", range(8))
def test_one_round_rank_selection_matches_reference_top4(oracle_mod, seed):
    # kernels/resident.rs:58-99: highest score first, the lower index first
    # among equal scores. Logits on a coarse grid make many exact ties.
    rng = np.random.default_rng(seed)
    lg = (rng.integers(-8, 9, 32) / 4.0).astype(np.float32)
    bias = np.zeros(32, dtype=np.float32) if seed % 2 == 0 else (rng.integers(-4, 5, 32) / 16.0).astype(np.float32)
    p = (1.0 / (1.0 + np.exp(-lg))).astype(np.float32)
    sel, _ = oracle_mod.route(lg, bias)
    assert _rank_top4(p + bias) == list(sel)
