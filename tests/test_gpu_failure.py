"""Failure detection on the GPU without a fault (DESIGN: failure detection).

Every device-side wait of the library is bounded (about one second of SM
cycles) and reports through a status word instead of trapping or spinning
forever. This test makes such a wait run out — an mbarrier that nothing
completes — and checks that the kernel returned with the timeout status, that
the wait lasted about its budget, and that the context is still usable for a
normal kernel-level call afterwards.
"""

import ctypes

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def test_bounded_wait_times_out_and_context_survives(cuda_lib):
    import torch

    import lfm2_b200
    status = ctypes.c_uint32(0)
    cycles = ctypes.c_uint64(0)
    lfm2_b200.ops_check(cuda_lib.lfm_selftest_wait_timeout(ctypes.byref(status), ctypes.byref(cycles)),
                        "selftest_wait_timeout")
    assert status.value == 1  # the bounded wait gave up and raised the status word
    assert 1.9e9 <= cycles.value <= 2.5e9  # WAIT_CYCLES = 2e9 SM cycles, plus the last polls
    # the context is intact: a normal call works and gives the right answer
    x = torch.tensor([1.0, 5.0, -2.0, 5.0, 3.0], device="cuda")
    out = torch.zeros(1, dtype=torch.int32, device="cuda")
    lfm2_b200.ops_check(cuda_lib.lfm_argmax(ctypes.c_void_p(x.data_ptr()), 5, ctypes.c_void_p(out.data_ptr()), None),
                        "argmax")
    torch.cuda.synchronize()
    assert int(out.item()) == 1
