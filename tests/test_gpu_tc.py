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
