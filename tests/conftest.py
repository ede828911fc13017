"""Shared fixtures. `-m gpu` tests need a B200; everything else runs on CPU."""

import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(ROOT, "lfm2-w9100-rust_b200")
ORACLE = os.path.join(ROOT, "oracle")
for p in (PKG, ORACLE, ROOT):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) GPU")


@pytest.fixture(scope="session")
def synth_model():
    """Path of the seeded synthetic LFM2 Q6_K GGUF (written on first use)."""
    import synth_gguf
    return synth_gguf.ensure_gguf(synth_gguf.default_model_path(1234), 1234)


@pytest.fixture(scope="session")
def oracle_mod():
    import oracle
    oracle.build()
    return oracle


@pytest.fixture(scope="session")
def cuda_lib():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    import lfm2_b200
    return lfm2_b200.lib()
