"""The tensor-core (tcgen05) GEMM core of the prompt path against numpy.

fp16 operands are exact in fp32, so the reference is the fp32 (float64
checked) product of the same fp16 values; the tensor core accumulates in fp32.
"""

import ctypes

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _ptr(t):
    return ctypes.c_void_p(t.data_ptr())


@pytest.mark.parametrize("m,n,k", [(128, 256, 64), (256, 512, 1024), (384, 256, 2048)])
def test_tc_gemm_f16_matches_numpy(cuda_lib, m, n, k):
    import torch

    import lfm2_b200
    rng = np.random.default_rng(m + n + k)
    a = rng.standard_normal((m, k)).astype(np.float16)
    b = rng.standard_normal((n, k)).astype(np.float16)
    ad, bd = torch.from_numpy(a).cuda(), torch.from_numpy(b).cuda()
    c = torch.full((m, n), float("nan"), device="cuda")
    lfm2_b200.ops_check(cuda_lib.lfm_tc_gemm_f16(_ptr(ad), _ptr(bd), m, n, k, _ptr(c), None), "tc_gemm_f16")
    ref = a.astype(np.float64) @ b.astype(np.float64).T
    got = c.cpu().numpy().astype(np.float64)
    assert np.isfinite(got).all()
    err = np.abs(got - ref).max() / np.abs(ref).max()
    assert err < 1e-5, err


def test_tc_gemm_f16_rejects_bad_shapes(cuda_lib):
    import torch
    a = torch.zeros(128, 64, dtype=torch.float16, device="cuda")
    c = torch.zeros(128, 256, device="cuda")
    assert cuda_lib.lfm_tc_gemm_f16(_ptr(a), _ptr(a), 128, 100, 64, _ptr(c), None) != 0


# ---------------------------------------------------------------- Q6_K prompt GEMM
# Tolerances (relative L2 over the whole output, against the float64 product
# of the exactly dequantised weights): the synthetic scales (|sc| <= 32) make
# every weight integer sc*(q-32) exact in fp16 and the hi/lo activation pair
# carries ~22 bits, so the error is fp32 accumulation alone (< 1e-5, the bar
# of the CUDA-core path). With scales over the whole int8 range, odd products
# above 2048 round to the nearest even integer: < 2e-4.
TOL_SYNTH, TOL_FULL = 1e-5, 2e-4


def _q6(cuda_lib, rng, in_dim, rows, full=False):
    from test_gpu_kernels import random_q6, upload
    raw = random_q6(rng, rows * in_dim // 256, full)
    return raw, upload(cuda_lib, raw, in_dim, rows)


def _rel(got, ref):
    return float(np.sqrt(((got - ref) ** 2).sum() / max((ref ** 2).sum(), 1e-300)))


@pytest.mark.parametrize("in_dim,rows,n,full", [
    (2048, 2048, 100, False), (2048, 512, 64, False), (2048, 6144, 130, False), (7168, 2048, 257, False),
    (1792, 2048, 33, False), (2048, 7168, 1, False), (2048, 1792, 300, True), (7168, 2048, 128, True)])
def test_prompt_gemm_vs_f64(cuda_lib, oracle_mod, in_dim, rows, n, full):
    import torch

    import lfm2_b200
    rng = np.random.default_rng(in_dim * 3 + rows + n)
    raw, w = _q6(cuda_lib, rng, in_dim, rows, full)
    x = rng.normal(0, 1, size=(n, in_dim)).astype(np.float32)
    y = torch.full((n, rows), float("nan"), device="cuda")
    xd = torch.from_numpy(x).cuda()
    lfm2_b200.ops_check(cuda_lib.lfm_q6k_prompt_gemm(_ptr(w), in_dim, rows, _ptr(xd), n, _ptr(y), None),
                        "prompt_gemm")
    got = y.cpu().numpy().astype(np.float64)
    wf = oracle_mod.dequant_blocks(raw).reshape(rows, in_dim).astype(np.float64)
    ref = x.astype(np.float64) @ wf.T
    assert np.isfinite(got).all()
    assert _rel(got, ref) < (TOL_FULL if full else TOL_SYNTH), _rel(got, ref)


def test_prompt_gemm_row_scaling(cuda_lib, oracle_mod):
    """Activation rows far outside fp16 range (large, tiny, zero, mixed
    magnitudes) go through the per-row power-of-two scaling."""
    import torch

    import lfm2_b200
    rng = np.random.default_rng(5)
    in_dim, rows, n = 2048, 256, 6
    raw, w = _q6(cuda_lib, rng, in_dim, rows)
    x = rng.normal(0, 1, size=(n, in_dim)).astype(np.float32)
    x[0] *= 1e7
    x[1] *= 1e-7
    x[2] = 0
    x[3, ::2] *= 1e4  # two magnitudes in one row
    x[4, 5] = 3e30
    y = torch.full((n, rows), float("nan"), device="cuda")
    xd = torch.from_numpy(x).cuda()
    lfm2_b200.ops_check(cuda_lib.lfm_q6k_prompt_gemm(_ptr(w), in_dim, rows, _ptr(xd), n, _ptr(y), None),
                        "prompt_gemm")
    got = y.cpu().numpy().astype(np.float64)
    wf = oracle_mod.dequant_blocks(raw).reshape(rows, in_dim).astype(np.float64)
    ref = x.astype(np.float64) @ wf.T
    assert (got[2] == 0).all()
    for t in (0, 1, 3, 4, 5):
        assert _rel(got[t], ref[t]) < TOL_SYNTH, (t, _rel(got[t], ref[t]))


@pytest.mark.parametrize("in_dim,rows,x_div,n", [(2048, 1792, 4, 50), (1792, 2048, 1, 50), (2048, 1792, 4, 200),
                                                 (2048, 1792, 4, 1)])
def test_prompt_grouped_vs_f64(cuda_lib, oracle_mod, in_dim, rows, x_div, n):
    """Routed experts through the grouped tile table: per-token distinct top-4
    experts, several experts unused, one expert chosen by every token (more
    than one 128-slot tile when n > 128)."""
    import torch

    import lfm2_b200
    rng = np.random.default_rng(in_dim + n + x_div)
    n_expert = 32
    raw, w = _q6(cuda_lib, rng, in_dim, n_expert * rows)
    ids = np.zeros((n, 4), np.int32)
    for t in range(n):
        others = rng.choice(np.arange(4, 20), 3, replace=False)  # experts 0-2 and 20-31 never, 3 always
        ids[t] = np.concatenate([[3], others])[rng.permutation(4)]
    xrows = n if x_div == 4 else 4 * n
    x = rng.normal(0, 1, size=(xrows, in_dim)).astype(np.float32)
    y = torch.full((4 * n, rows), float("nan"), device="cuda")
    idd, xd = torch.from_numpy(ids.reshape(-1)).cuda(), torch.from_numpy(x).cuda()
    lfm2_b200.ops_check(cuda_lib.lfm_q6k_prompt_grouped(_ptr(w), in_dim, rows, n_expert, _ptr(idd), _ptr(xd), x_div,
                                                        n, _ptr(y), None), "prompt_grouped")
    got = y.cpu().numpy().astype(np.float64)
    wf = oracle_mod.dequant_blocks(raw).reshape(n_expert, rows, in_dim).astype(np.float64)
    ref = np.empty_like(got)
    for q in range(4 * n):
        ref[q] = wf[ids.reshape(-1)[q]] @ x[q // x_div].astype(np.float64)
    assert np.isfinite(got).all()
    assert _rel(got, ref) < TOL_SYNTH, _rel(got, ref)


def test_prompt_grouped_slot_lists_over_several_passes(cuda_lib, oracle_mod):
    """5000 tokens = 20000 (token, rank) slots: the per-expert slot lists are
    built in two passes of 16384 slots, and every slot's row must still land
    in its expert's list in slot order (checked through the GEMM result)."""
    import torch

    import lfm2_b200
    rng = np.random.default_rng(5000)
    in_dim, rows, n = 512, 128, 5000
    raw, w = _q6(cuda_lib, rng, in_dim, 32 * rows)
    ids = np.stack([rng.choice(32, 4, replace=False) for _ in range(n)]).astype(np.int32).reshape(-1)
    x = rng.normal(0, 1, size=(n, in_dim)).astype(np.float32)
    y = torch.full((4 * n, rows), float("nan"), device="cuda")
    idd, xd = torch.from_numpy(ids).cuda(), torch.from_numpy(x).cuda()
    lfm2_b200.ops_check(cuda_lib.lfm_q6k_prompt_grouped(_ptr(w), in_dim, rows, 32, _ptr(idd), _ptr(xd), 4, n,
                                                        _ptr(y), None), "prompt_grouped")
    got = y.cpu().numpy().astype(np.float64)
    wf = oracle_mod.dequant_blocks(raw).reshape(32, rows, in_dim).astype(np.float64)
    ref = np.empty_like(got)
    x64 = x.astype(np.float64)
    for e in range(32):
        q = np.nonzero(ids == e)[0]
        ref[q] = x64[q // 4] @ wf[e].T
    assert np.isfinite(got).all()
    assert _rel(got, ref) < TOL_SYNTH, _rel(got, ref)


def test_prompt_grouped_unaligned_ids_and_repeats(cuda_lib):
    """The slot lists read the expert ids four at a time when the id array is
    16-byte aligned and one at a time otherwise: both give the same result.
    A token naming one expert twice would grow that expert's list past its
    capacity: the list stops there and the call returns LFM_ERR_ARG."""
    import torch

    import lfm2_b200
    rng = np.random.default_rng(17)
    in_dim, rows, n = 2048, 128, 300
    raw, w = _q6(cuda_lib, rng, in_dim, 32 * rows)
    ids = np.stack([rng.choice(32, 4, replace=False) for _ in range(n)]).astype(np.int32).reshape(-1)
    x = torch.from_numpy(rng.normal(0, 1, size=(n, in_dim)).astype(np.float32)).cuda()
    buf = torch.zeros(4 * n + 1, dtype=torch.int32, device="cuda")
    buf[: 4 * n] = torch.from_numpy(ids).cuda()
    ya = torch.zeros((4 * n, rows), device="cuda")
    lfm2_b200.ops_check(cuda_lib.lfm_q6k_prompt_grouped(_ptr(w), in_dim, rows, 32, _ptr(buf), _ptr(x), 4, n,
                                                        _ptr(ya), None), "aligned ids")
    buf[1:] = torch.from_numpy(ids).cuda()  # the same ids 4 bytes further on
    yb = torch.zeros((4 * n, rows), device="cuda")
    lfm2_b200.ops_check(cuda_lib.lfm_q6k_prompt_grouped(_ptr(w), in_dim, rows, 32,
                                                        ctypes.c_void_p(buf.data_ptr() + 4), _ptr(x), 4, n,
                                                        _ptr(yb), None), "unaligned ids")
    assert torch.equal(ya, yb)
    same = torch.full((4 * n,), 5, dtype=torch.int32, device="cuda")
    st = cuda_lib.lfm_q6k_prompt_grouped(_ptr(w), in_dim, rows, 32, _ptr(same), _ptr(x), 4, n, _ptr(ya), None)
    assert st == 1  # LFM_ERR_ARG
    assert b"distinct" in cuda_lib.lfm_ops_error()
    lfm2_b200.ops_check(cuda_lib.lfm_q6k_prompt_grouped(_ptr(w), in_dim, rows, 32, _ptr(buf), _ptr(x), 4, n,
                                                        _ptr(yb), None), "after the rejected call")


def test_prompt_gemm_rejects_bad_shapes(cuda_lib):
    import torch
    w = torch.zeros(100 * 8 * 210, dtype=torch.uint8, device="cuda")
    x = torch.zeros(2048, device="cuda")
    y = torch.zeros(100, device="cuda")
    assert cuda_lib.lfm_q6k_prompt_gemm(_ptr(w), 2048, 100, _ptr(x), 1, _ptr(y), None) != 0
    assert cuda_lib.lfm_q6k_prompt_grouped(_ptr(w), 2048, 128, 8, _ptr(x), _ptr(x), 4, 1, _ptr(y), None) != 0


@pytest.mark.parametrize("m,k", [(128, 64), (256, 128), (128, 1024)])
def test_tc_gemm_f16_mn_major_b(cuda_lib, m, k):
    """MN-major second operand (rows of 64 contiguous values, like the V cache)."""
    import torch

    import lfm2_b200
    rng = np.random.default_rng(m * 7 + k)
    a = rng.standard_normal((m, k)).astype(np.float16)
    b = rng.standard_normal((k, 64)).astype(np.float16)
    ad, bd = torch.from_numpy(a).cuda(), torch.from_numpy(b).cuda()
    c = torch.full((m, 64), float("nan"), device="cuda")
    lfm2_b200.ops_check(cuda_lib.lfm_tc_gemm_f16_bmn(_ptr(ad), _ptr(bd), m, k, _ptr(c), None), "tc_gemm_f16_bmn")
    ref = a.astype(np.float64) @ b.astype(np.float64)
    got = c.cpu().numpy().astype(np.float64)
    assert np.isfinite(got).all()
    err = np.abs(got - ref).max() / np.abs(ref).max()
    assert err < 1e-5, err


# ------------------------------------------------- expanded fp16 weight operand
def _q6_ints(raw):
    """sc * (q - 32) of every weight of Q6_K blocks (q6k.rs:74-146 without d):
    ql[128], qh[64], int8 scales[16], fp16 d per 210-byte block."""
    b = raw.reshape(-1, 210)
    ql, qh = b[:, :128].astype(np.int32), b[:, 128:192].astype(np.int32)
    sc = b[:, 192:208].view(np.int8).astype(np.int32)
    out = np.empty((b.shape[0], 256), np.int32)
    for h in range(2):
        l = np.arange(32)
        lq, hq = ql[:, 64 * h:64 * h + 64], qh[:, 32 * h:32 * h + 32]
        q = [(lq[:, l] & 15) | ((hq[:, l] & 3) << 4), (lq[:, l + 32] & 15) | (((hq[:, l] >> 2) & 3) << 4),
             (lq[:, l] >> 4) | (((hq[:, l] >> 4) & 3) << 4), (lq[:, l + 32] >> 4) | (((hq[:, l] >> 6) & 3) << 4)]
        for j in range(4):
            s = sc[:, 8 * h + 2 * j + l // 16]
            out[:, 128 * h + 32 * j + l] = s * (q[j] - 32)
    return out.reshape(-1)


@pytest.mark.parametrize("in_dim,rows,full", [(2048, 256, False), (1792, 128, True)])
def test_expand_f16_exact(cuda_lib, oracle_mod, in_dim, rows, full):
    """The expanded operand holds sc*(q-32) rounded to fp16 (exact up to 2048;
    with full-range scales, odd products above 2048 round to even, as in the
    on-chip path); d times the integers is the reference dequantisation to
    within its own f32 rounding."""
    import torch

    import lfm2_b200
    rng = np.random.default_rng(in_dim + rows)
    raw, w = _q6(cuda_lib, rng, in_dim, rows, full)
    w16 = torch.full((rows, in_dim), float("nan"), dtype=torch.float16, device="cuda")
    lfm2_b200.ops_check(cuda_lib.lfm_q6k_expand_f16(_ptr(w), in_dim, rows, _ptr(w16), None), "expand_f16")
    torch.cuda.synchronize()
    got = w16.cpu().numpy().astype(np.float64).reshape(-1)
    ints = _q6_ints(raw)
    assert np.array_equal(got, ints.astype(np.float16).astype(np.float64))
    d = raw.reshape(-1, 210)[:, 208:210].copy().view(np.float16).astype(np.float64)
    deq = oracle_mod.dequant_blocks(raw).astype(np.float64)
    assert np.allclose((ints.reshape(-1, 256) * d).reshape(-1), deq, rtol=2.0 ** -23, atol=0)


@pytest.mark.parametrize("in_dim,rows,n,full", [(2048, 2048, 100, False), (2048, 6144, 3, False),
                                                (7168, 2048, 257, True), (2048, 512, 1000, False)])
def test_prompt_gemm_x16_bit_identical(cuda_lib, oracle_mod, in_dim, rows, n, full):
    """Reading the expanded operand gives the on-chip-dequantising GEMM's
    output bit for bit (same integers, same MMAs, same fold order)."""
    import torch

    import lfm2_b200
    rng = np.random.default_rng(in_dim + 7 * rows + n)
    raw, w = _q6(cuda_lib, rng, in_dim, rows, full)
    w16 = torch.empty((rows, in_dim), dtype=torch.float16, device="cuda")
    lfm2_b200.ops_check(cuda_lib.lfm_q6k_expand_f16(_ptr(w), in_dim, rows, _ptr(w16), None), "expand_f16")
    x = rng.normal(0, 1, size=(n, in_dim)).astype(np.float32)
    xd = torch.from_numpy(x).cuda()
    ya = torch.full((n, rows), float("nan"), device="cuda")
    yb = torch.full((n, rows), float("nan"), device="cuda")
    lfm2_b200.ops_check(cuda_lib.lfm_q6k_prompt_gemm(_ptr(w), in_dim, rows, _ptr(xd), n, _ptr(ya), None), "gemm")
    lfm2_b200.ops_check(cuda_lib.lfm_q6k_prompt_gemm_x16(_ptr(w), _ptr(w16), in_dim, rows, _ptr(xd), n, _ptr(yb),
                                                         None), "gemm_x16")
    a, b = ya.cpu().numpy(), yb.cpu().numpy()
    assert np.isfinite(b).all()
    assert np.array_equal(a.view(np.uint32), b.view(np.uint32))
    wf = oracle_mod.dequant_blocks(raw).reshape(rows, in_dim).astype(np.float64)
    ref = x.astype(np.float64) @ wf.T
    assert _rel(b.astype(np.float64), ref) < (TOL_FULL if full else TOL_SYNTH)


@pytest.mark.parametrize("in_dim,rows,x_div,n", [(2048, 1792, 4, 300), (1792, 2048, 1, 77), (1792, 2048, 1, 1200)])
def test_prompt_grouped_x16_bit_identical(cuda_lib, oracle_mod, in_dim, rows, x_div, n):
    import torch

    import lfm2_b200
    rng = np.random.default_rng(in_dim + n + 11 * x_div)
    n_expert = 32
    raw, w = _q6(cuda_lib, rng, in_dim, n_expert * rows)
    w16 = torch.empty((n_expert * rows, in_dim), dtype=torch.float16, device="cuda")
    lfm2_b200.ops_check(cuda_lib.lfm_q6k_expand_f16(_ptr(w), in_dim, n_expert * rows, _ptr(w16), None),
                        "expand_f16")
    ids = np.stack([rng.permutation(n_expert)[:4] for _ in range(n)]).astype(np.int32)
    xrows = n if x_div == 4 else 4 * n
    x = rng.normal(0, 1, size=(xrows, in_dim)).astype(np.float32)
    idd, xd = torch.from_numpy(ids.reshape(-1)).cuda(), torch.from_numpy(x).cuda()
    ya = torch.full((4 * n, rows), float("nan"), device="cuda")
    yb = torch.full((4 * n, rows), float("nan"), device="cuda")
    lfm2_b200.ops_check(cuda_lib.lfm_q6k_prompt_grouped(_ptr(w), in_dim, rows, n_expert, _ptr(idd), _ptr(xd), x_div,
                                                        n, _ptr(ya), None), "grouped")
    lfm2_b200.ops_check(cuda_lib.lfm_q6k_prompt_grouped_x16(_ptr(w), _ptr(w16), in_dim, rows, n_expert, _ptr(idd),
                                                            _ptr(xd), x_div, n, _ptr(yb), None), "grouped_x16")
    a, b = ya.cpu().numpy(), yb.cpu().numpy()
    assert np.isfinite(b).all()
    assert np.array_equal(a.view(np.uint32), b.view(np.uint32))


def test_expand_rejects_bad_arguments(cuda_lib):
    import torch
    w = torch.zeros(128 * 8 * 210, dtype=torch.uint8, device="cuda")
    out = torch.zeros(128 * 2048 + 8, dtype=torch.float16, device="cuda")
    misaligned = ctypes.c_void_p(out.data_ptr() + 2)
    assert cuda_lib.lfm_q6k_expand_f16(_ptr(w), 2048, 128, misaligned, None) != 0
    assert cuda_lib.lfm_q6k_expand_f16(_ptr(w), 100, 128, _ptr(out), None) != 0
    x = torch.zeros(2048, device="cuda")
    y = torch.zeros(128, device="cuda")
    assert cuda_lib.lfm_q6k_prompt_gemm_x16(_ptr(w), misaligned, 2048, 128, _ptr(x), 1, _ptr(y), None) != 0


_TWO_SM_CHECK = r"""
import ctypes, sys
import numpy as np
import torch
sys.path[:0] = [sys.argv[1], sys.argv[2]]
import lfm2_b200
from test_gpu_kernels import random_q6
lib = lfm2_b200.lib()
P = lambda t: ctypes.c_void_p(t.data_ptr())
def up(raw, in_dim, rows):
    dev = torch.empty(raw.size, dtype=torch.uint8, device="cuda")
    lfm2_b200.ops_check(lib.lfm_q6k_upload(raw.ctypes.data_as(ctypes.c_void_p), in_dim, rows, P(dev)), "upload")
    return dev
def exp16(w, in_dim, rows):
    w16 = torch.empty((rows, in_dim), dtype=torch.float16, device="cuda")
    lfm2_b200.ops_check(lib.lfm_q6k_expand_f16(P(w), in_dim, rows, P(w16), None), "expand")
    return w16
rng = np.random.default_rng(77)
for in_dim, rows, n in [(2048, 2048, 300), (7168, 2048, 129), (2048, 6144, 1000)]:
    w = up(random_q6(rng, rows * in_dim // 256, True), in_dim, rows)
    w16 = exp16(w, in_dim, rows)
    x = torch.from_numpy(rng.normal(0, 1, size=(n, in_dim)).astype(np.float32)).cuda()
    ya = torch.full((n, rows), float("nan"), device="cuda")
    yb = torch.full((n, rows), float("nan"), device="cuda")
    lfm2_b200.ops_check(lib.lfm_q6k_prompt_gemm(P(w), in_dim, rows, P(x), n, P(ya), None), "gemm")
    lfm2_b200.ops_check(lib.lfm_q6k_prompt_gemm_x16(P(w), P(w16), in_dim, rows, P(x), n, P(yb), None), "gemm_x16")
    assert torch.isfinite(yb).all()
    assert torch.equal(ya.view(torch.int32), yb.view(torch.int32)), (in_dim, rows, n)
for in_dim, rows, x_div, n in [(1792, 2048, 1, 1200), (2048, 1792, 4, 1500)]:
    w = up(random_q6(rng, 32 * rows * in_dim // 256), in_dim, 32 * rows)
    w16 = exp16(w, in_dim, 32 * rows)
    ids = torch.from_numpy(np.stack([rng.permutation(32)[:4] for _ in range(n)]).astype(np.int32).ravel()).cuda()
    x = torch.from_numpy(rng.normal(0, 1, size=((n if x_div == 4 else 4 * n), in_dim)).astype(np.float32)).cuda()
    ya = torch.full((4 * n, rows), float("nan"), device="cuda")
    yb = torch.full((4 * n, rows), float("nan"), device="cuda")
    lfm2_b200.ops_check(lib.lfm_q6k_prompt_grouped(P(w), in_dim, rows, 32, P(ids), P(x), x_div, n, P(ya), None), "g")
    lfm2_b200.ops_check(lib.lfm_q6k_prompt_grouped_x16(P(w), P(w16), in_dim, rows, 32, P(ids), P(x), x_div, n,
                                                       P(yb), None), "g_x16")
    assert torch.isfinite(yb).all()
    assert torch.equal(ya.view(torch.int32), yb.view(torch.int32)), (in_dim, rows, n)
print("OK")
"""


def test_two_sm_gemm_bit_identical():
    """The 2-SM (cta_group::2, M=256) form of the expanded-weight GEMM, which
    serves 128-token tiles when LFM_PREFILL_2SM=1, gives the 1-SM results bit
    for bit (dense and grouped; run in a child process because the switch is
    read once per process)."""
    import os
    import subprocess
    import sys
    here = os.path.dirname(os.path.abspath(__file__))
    pkg = os.path.join(os.path.dirname(here), "lfm2-w9100-rust_b200")
    env = dict(os.environ, LFM_PREFILL_2SM="1")
    r = subprocess.run([sys.executable, "-c", _TWO_SM_CHECK, here, pkg], env=env, capture_output=True, text=True,
                       timeout=600)
    assert r.returncode == 0 and r.stdout.strip().endswith("OK"), r.stdout[-2000:] + r.stderr[-2000:]
