"""Shared test setup: import paths, the `gpu` marker, and small helpers."""
import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, os.path.join(ROOT, "cdcl-gptq_b200"))
sys.path.insert(0, os.path.join(ROOT, "oracle"))
GOLDEN = os.path.join(ROOT, "tests", "golden")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")


def has_gpu():
    try:
        import torch

        return torch.cuda.is_available()
    except Exception:
        return False


@pytest.fixture(scope="session")
def gpu():
    if not has_gpu():
        pytest.skip("no CUDA device")
    import cdclq

    cdclq.lib()  # the library must load: no fallback exists
    return True


def assert_layers_identical(a, b, what=""):
    """Bit-exact comparison of two quantized layers (codes, scales, zeros, perm, gbits)."""
    assert np.array_equal(a.perm, b.perm), f"{what}: permutation differs"
    assert np.array_equal(a.gbits, b.gbits), f"{what}: gbits differ"
    nd = int(np.count_nonzero(a.codes != b.codes))
    assert nd == 0, f"{what}: {nd} of {a.codes.size} codes differ"
    assert np.array_equal(a.scales, b.scales), f"{what}: scales differ"
    assert np.array_equal(a.zeros, b.zeros), f"{what}: zeros differ"
