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
