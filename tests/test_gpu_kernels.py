"""Kernel-level parity of the CUDA path against the CPU oracle, through the C ABI.

Mirrors the reference's hardware screens:
  q6_check.rs:73-137        Q6_K matvec vs f64 CPU reference, rel-L2 < 1e-3, finite
  dequant_mirror.rs:49-91   dequant bit-exact (here: the GPU kernel vs the oracle)
  resident_check.rs:35-84   router order / stable ties / probability tolerance 1e-6
  optimization_check.rs:122-149  GPU argmax with NaN, ties and tails
"""

import ctypes

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _torch():
    import torch
    return torch


def _ptr(t):
    return ctypes.c_void_p(t.data_ptr())


def random_q6(rng, nblocks, full_scale_range=False):
    """Q6_K blocks with the synthetic distribution (or int8 scales over the
    whole range, including -128, like the real quantiser produces)."""
    import synth_gguf
    raw = synth_gguf.random_q6k_blocks(rng, nblocks).reshape(nblocks, 210)
    if full_scale_range:
        raw[:, 192:208] = rng.integers(-128, 128, size=(nblocks, 16)).astype(np.int8).view(np.uint8)
        raw[::7, 192] = 0x80
    return raw.reshape(-1)


def upload(cuda_lib, raw, in_dim, rows):
    import lfm2_b200
    torch = _torch()
    nbytes = cuda_lib.lfm_q6k_device_bytes(in_dim, rows)
    assert nbytes == raw.size
    dev = torch.empty(nbytes, dtype=torch.uint8, device="cuda")
    lfm2_b200.ops_check(cuda_lib.lfm_q6k_upload(raw.ctypes.data_as(ctypes.c_void_p), in_dim, rows, _ptr(dev)),
                        "upload")
    return dev


def activation(in_dim, n):
    # q6_check.rs:73-79
    kk = np.arange(in_dim * n) % in_dim
    v = (kk.astype(np.float32) * np.float32(0.03125))
    return (np.sin(v) * 0.5 + (kk % 3) * 0.01 - 0.25).astype(np.float32)


@pytest.mark.parametrize("in_dim", [256, 1792, 2048, 7168])
@pytest.mark.parametrize("full", [False, True])
def test_dequant_bit_exact(cuda_lib, oracle_mod, in_dim, full):
    import lfm2_b200
    torch = _torch()
    rng = np.random.default_rng(in_dim + int(full))
    rows = 96
    raw = random_q6(rng, rows * in_dim // 256, full)
    w = upload(cuda_lib, raw, in_dim, rows)
    out = torch.empty(rows * in_dim, dtype=torch.float32, device="cuda")
    lfm2_b200.ops_check(cuda_lib.lfm_q6k_dequant(_ptr(w), in_dim, rows, 0, rows, _ptr(out), None), "dequant")
    torch.cuda.synchronize()
    got = out.cpu().numpy()
    ref = oracle_mod.dequant_blocks(raw)
    assert np.array_equal(got.view(np.uint32), ref.view(np.uint32))


def test_dequant_mirror_blocks_bit_exact(cuda_lib, oracle_mod):
    from test_oracle_pins import _xorshift_blocks
    import lfm2_b200
    torch = _torch()
    blocks = _xorshift_blocks().reshape(-1)  # 512 blocks = 64 rows of 2048
    w = upload(cuda_lib, blocks, 2048, 64)
    out = torch.empty(64 * 2048, dtype=torch.float32, device="cuda")
    lfm2_b200.ops_check(cuda_lib.lfm_q6k_dequant(_ptr(w), 2048, 64, 0, 64, _ptr(out), None), "dequant")
    torch.cuda.synchronize()
    assert np.array_equal(out.cpu().numpy().view(np.uint32), oracle_mod.dequant_blocks(blocks).view(np.uint32))


# every matrix shape of the decode step (in -> out), plus the lm_head
SHAPES = [(2048, 2048), (2048, 512), (2048, 6144), (2048, 7168), (7168, 2048), (2048, 1792), (1792, 2048),
          (2048, 128000), (2048, 65536)]


@pytest.mark.parametrize("in_dim,out_dim", SHAPES)
def test_matvec_vs_f64(cuda_lib, oracle_mod, in_dim, out_dim):
    import lfm2_b200
    torch = _torch()
    rng = np.random.default_rng(out_dim * 7 + in_dim)
    raw = random_q6(rng, out_dim * in_dim // 256)
    w = upload(cuda_lib, raw, in_dim, out_dim)
    x = activation(in_dim, 1)
    xd = torch.from_numpy(x).cuda()
    y = torch.empty(out_dim, dtype=torch.float32, device="cuda")
    lfm2_b200.ops_check(cuda_lib.lfm_q6k_matmul(_ptr(w), in_dim, out_dim, _ptr(xd), 1, _ptr(y), None), "matmul")
    torch.cuda.synchronize()
    got = y.cpu().numpy().astype(np.float64)
    ref = oracle_mod.q6k_matvec_f64(raw, in_dim, out_dim, x).astype(np.float64)
    rel = np.sqrt(((got - ref) ** 2).sum() / max((ref ** 2).sum(), 1e-30))
    assert np.isfinite(got).all()
    assert rel < 1e-5, rel  # the reference's screen is 1e-3 (q6_check.rs:136)


@pytest.mark.parametrize("n", [2, 3, 5, 8, 16, 64, 100])
def test_matmul_columns_vs_oracle(cuda_lib, oracle_mod, n):
    import lfm2_b200
    torch = _torch()
    rng = np.random.default_rng(n)
    in_dim, out_dim = 2048, 7 * 64 + 5  # partial row tile
    raw = random_q6(rng, out_dim * in_dim // 256)
    w = upload(cuda_lib, raw, in_dim, out_dim)
    x = rng.normal(0, 1, size=in_dim * n).astype(np.float32)
    xd = torch.from_numpy(x).cuda()
    y = torch.empty(out_dim * n, dtype=torch.float32, device="cuda")
    lfm2_b200.ops_check(cuda_lib.lfm_q6k_matmul(_ptr(w), in_dim, out_dim, _ptr(xd), n, _ptr(y), None), "matmul")
    torch.cuda.synchronize()
    got = y.cpu().numpy().astype(np.float64)
    ref = oracle_mod.q6k_matmul_f32(raw, in_dim, out_dim, x, n).astype(np.float64)
    rel = np.sqrt(((got - ref) ** 2).sum() / (ref ** 2).sum())
    assert rel < 1e-5, rel


@pytest.mark.parametrize("in_dim,out_dim", [(2048, 1792), (1792, 2048)])
def test_routed_experts(cuda_lib, oracle_mod, in_dim, out_dim):
    import lfm2_b200
    torch = _torch()
    rng = np.random.default_rng(11 + in_dim)
    n_expert = 32
    raw = random_q6(rng, n_expert * out_dim * in_dim // 256)
    w = upload(cuda_lib, raw, in_dim, n_expert * out_dim)
    ids = np.array([31, 0, 17, 5], dtype=np.int32)
    x = rng.normal(0, 1, size=4 * in_dim).astype(np.float32)
    idd = torch.from_numpy(ids).cuda()
    xd = torch.from_numpy(x).cuda()
    y = torch.empty(4 * out_dim, dtype=torch.float32, device="cuda")
    lfm2_b200.ops_check(cuda_lib.lfm_q6k_routed(_ptr(w), in_dim, out_dim, n_expert, _ptr(idd), _ptr(xd), in_dim,
                                                _ptr(y), None), "routed")
    torch.cuda.synchronize()
    got = y.cpu().numpy().reshape(4, out_dim)
    row_bytes = in_dim // 256 * 210
    for s in range(4):
        e = ids[s]
        we = raw[e * out_dim * row_bytes:(e + 1) * out_dim * row_bytes]
        ref = oracle_mod.q6k_matvec_f64(we, in_dim, out_dim, x[s * in_dim:(s + 1) * in_dim])
        rel = np.sqrt(((got[s] - ref) ** 2).sum() / (ref ** 2).sum())
        assert rel < 1e-5, (s, rel)


@pytest.mark.parametrize("experts", [4, 32])
def test_route_matches_oracle(cuda_lib, oracle_mod, experts):
    import lfm2_b200
    torch = _torch()
    n = 3
    # resident_check.rs:39-47 vectors (token 0: all-equal logits -> stable ties)
    logits = np.array([0.0 if i < experts else ((i * 13 % 19) - 9) / 8.0 for i in range(n * experts)],
                      dtype=np.float32)
    rng = np.random.default_rng(experts)
    logits = np.concatenate([logits, rng.normal(0, 2, size=64 * experts).astype(np.float32)])
    n += 64
    bias = np.concatenate([np.zeros(experts), rng.normal(0, 0.01, size=0)]).astype(np.float32)
    ld, bd = torch.from_numpy(logits).cuda(), torch.from_numpy(bias).cuda()
    sel = torch.empty(n * 4, dtype=torch.int32, device="cuda")
    sw = torch.empty(n * 4, dtype=torch.float32, device="cuda")
    lfm2_b200.ops_check(cuda_lib.lfm_route(_ptr(ld), _ptr(bd), experts, n, _ptr(sel), _ptr(sw), None), "route")
    torch.cuda.synchronize()
    s, w = sel.cpu().numpy().reshape(n, 4), sw.cpu().numpy().reshape(n, 4)
    for j in range(n):
        rs, rw = oracle_mod.route(logits[j * experts:(j + 1) * experts], bias)
        assert list(s[j]) == list(rs), j
        assert np.abs(w[j] - rw).max() < 1e-6


@pytest.mark.parametrize("length", [1, 63, 513, 128003])
def test_argmax_nan_ties_tails(cuda_lib, oracle_mod, length):
    import lfm2_b200
    torch = _torch()
    # optimization_check.rs:122-149
    v = -(np.arange(length) % 101).astype(np.float32)
    if length > 1:
        v[0] = np.nan
        v[-1] = 3.0
    vd = torch.from_numpy(v).cuda()
    out = torch.zeros(1, dtype=torch.int32, device="cuda")
    lfm2_b200.ops_check(cuda_lib.lfm_argmax(_ptr(vd), length, _ptr(out), None), "argmax")
    torch.cuda.synchronize()
    assert int(out.item()) == length - 1 == oracle_mod.argmax(v) or (length == 1 and int(out.item()) == 0)
    # ties -> lowest index; all-NaN -> 0
    t = np.zeros(length, dtype=np.float32)
    t[length // 3:] = 1.0
    td = torch.from_numpy(t).cuda()
    lfm2_b200.ops_check(cuda_lib.lfm_argmax(_ptr(td), length, _ptr(out), None), "argmax")
    torch.cuda.synchronize()
    assert int(out.item()) == oracle_mod.argmax(t)
    nd = torch.full((length,), float("nan"), device="cuda")
    lfm2_b200.ops_check(cuda_lib.lfm_argmax(_ptr(nd), length, _ptr(out), None), "argmax")
    torch.cuda.synchronize()
    assert int(out.item()) == 0
