"""lfm_argmax_noalloc against lfm_argmax, through the C ABI.

lfm_argmax_noalloc is for callers that may not allocate device memory at call
time (a host whose memory pool already owns the whole device, or code running
where the CUDA allocator must not be entered): it takes its scratch from a
fixed array inside the library instead of cudaMallocAsync. Its index must be
the one lfm_argmax returns, on every call, including back-to-back calls that
reuse the array left over by the previous call.

This file is named to be collected last, so that a run stopping at the first
failure has run every other test before it.
"""

import ctypes

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _ptr(t):
    return ctypes.c_void_p(t.data_ptr())


def _both(cuda_lib, xd, n):
    import lfm2_b200
    import torch
    out_a = torch.full((1,), -1, dtype=torch.int32, device="cuda")
    out_b = torch.full((1,), -1, dtype=torch.int32, device="cuda")
    lfm2_b200.ops_check(cuda_lib.lfm_argmax(_ptr(xd), n, _ptr(out_a), None), "argmax")
    lfm2_b200.ops_check(cuda_lib.lfm_argmax_noalloc(_ptr(xd), n, _ptr(out_b), None), "argmax_noalloc")
    torch.cuda.synchronize()
    return int(out_a.item()), int(out_b.item())


@pytest.mark.parametrize("length", [1, 63, 1025, 128000, 1 << 22])
def test_noalloc_argmax_matches_allocating_entry_point(cuda_lib, length):
    import torch
    rng = np.random.default_rng(length)
    # two different inputs on two calls in a row: the second call starts from
    # the partials and counter the first one left in the shared array
    for trial in range(2):
        v = rng.standard_normal(length).astype(np.float32)
        if length > 4:
            v[rng.integers(0, length, size=3)] = np.nan
            v[rng.integers(0, length, size=2)] = v[~np.isnan(v)].max()  # ties -> lowest index
        xd = torch.from_numpy(v).cuda()
        a, b = _both(cuda_lib, xd, length)
        assert a == b, (length, trial, a, b)
        # lowest index of the maximum over the non-NaN values, computed here
        # (all values finite except the planted NaNs)
        m = np.nanmax(v)
        assert b == int(np.flatnonzero(v == m)[0])


def test_noalloc_argmax_all_nan_and_ties(cuda_lib):
    import torch
    n = 70001
    xd = torch.full((n,), float("nan"), device="cuda")
    assert _both(cuda_lib, xd, n) == (0, 0)
    t = torch.zeros(n, device="cuda")
    t[n // 3:] = 1.0
    assert _both(cuda_lib, t, n) == (n // 3, n // 3)


def test_noalloc_argmax_rejects_oversize(cuda_lib):
    import torch
    xd = torch.zeros(4, device="cuda")
    out = torch.zeros(1, dtype=torch.int32, device="cuda")
    st = cuda_lib.lfm_argmax_noalloc(_ptr(xd), (1 << 30) + 1, _ptr(out), None)
    assert st != 0
    assert "exceeds the maximum" in cuda_lib.lfm_ops_error().decode()
    assert cuda_lib.lfm_argmax_noalloc(_ptr(xd), 0, _ptr(out), None) != 0
