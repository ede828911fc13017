"""Tensor-core causal GQA prompt attention against a float64 reference.

Contract (lfm.rs:395-437, the reference's prompt attention; GPU kernel
kernels.rs:672-763): token j at position start + j, query head h reads KV
head h // 4; scores q.k / 8 over positions 0..start+j, softmax, weighted sum
of V. The K/V caches are fp16 [8][ctx][64] (the engine's layout), q is fp32.
Tolerance: q and the probabilities enter the tensor cores as fp16 hi/lo
pairs (about 22 bits) with fp32 accumulation: max-abs error < 2e-5 on outputs
of magnitude ~1 and relative L2 < 1e-5.
"""

import ctypes

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _ptr(t):
    return ctypes.c_void_p(t.data_ptr())


def _reference(q, kc, vc, start, n):
    out = np.zeros((n, 32 * 64))
    k64, v64 = kc.astype(np.float64), vc.astype(np.float64)
    for j in range(n):
        p = start + j
        for h in range(32):
            kh = h // 4
            s = k64[kh, :p + 1] @ q[j, h * 64:(h + 1) * 64].astype(np.float64) / 8.0
            w = np.exp(s - s.max())
            out[j, h * 64:(h + 1) * 64] = (w / w.sum()) @ v64[kh, :p + 1]
    return out


@pytest.mark.parametrize("start,n,ctx", [(0, 1, 64), (0, 31, 64), (0, 200, 512), (100, 64, 512), (0, 300, 300),
                                         (3900, 196, 4096), (129, 33, 1024)])
def test_attention_prefill_vs_f64(cuda_lib, start, n, ctx):
    import torch

    import lfm2_b200
    rng = np.random.default_rng(start * 7 + n + ctx)
    q_stride = 2048 + 1024  # the engine's fused q|k|v rows
    q = np.zeros((n, q_stride), np.float32)
    q[:, :2048] = rng.normal(0, 1.5, size=(n, 2048))
    kc = np.zeros((8, ctx, 64), np.float16)
    vc = np.zeros((8, ctx, 64), np.float16)
    kc[:, :start + n] = rng.normal(0, 1, size=(8, start + n, 64)).astype(np.float16)
    vc[:, :start + n] = rng.normal(0, 1, size=(8, start + n, 64)).astype(np.float16)
    qd, kd, vd = (torch.from_numpy(a).cuda() for a in (q, kc, vc))
    out = torch.full((n, 2048), float("nan"), device="cuda")
    lfm2_b200.ops_check(cuda_lib.lfm_attention_prefill(_ptr(qd), q_stride, _ptr(kd), _ptr(vd), ctx, start, n,
                                                        _ptr(out), 2048, None), "attention_prefill")
    got = out.cpu().numpy().astype(np.float64)
    ref = _reference(q[:, :2048], kc, vc, start, n)
    assert np.isfinite(got).all()
    assert np.abs(got - ref).max() < 2e-5, np.abs(got - ref).max()
    rel = np.sqrt(((got - ref) ** 2).sum() / (ref ** 2).sum())
    assert rel < 1e-5, rel


def test_attention_prefill_rejects_bad_range(cuda_lib):
    import torch
    x = torch.zeros(4096, device="cuda")
    assert cuda_lib.lfm_attention_prefill(_ptr(x), 2048, _ptr(x), _ptr(x), 64, 60, 8, _ptr(x), 2048, None) != 0
