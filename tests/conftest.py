"""Shared pytest setup: the `gpu` marker, import paths and fixtures.

Tests marked `gpu` need a B200 (sm_100) and call the product library
libx100gemm_b200.so through its C ABI; everything else runs on CPU.
"""
import os
import sys

import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
for sub in ("oracle", "x100-gemm_b200"):
    p = os.path.join(REPO, sub)
    if p not in sys.path:
        sys.path.insert(0, p)
GOLDEN = os.path.join(REPO, "tests", "golden")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 GPU (sm_100a) and the CUDA library")


@pytest.fixture(scope="session")
def golden_dir():
    return GOLDEN
