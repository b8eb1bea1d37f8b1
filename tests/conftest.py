"""Test configuration.

Markers:
  gpu  -- needs a CUDA (sm_100) device; runs the kernels of libnpub.so and
          compares them with the oracle (oracle/).

CPU tests (-m "not gpu") check the oracle against the golden fixtures in
tests/golden/, the host-side logic, and that the C ABI library loads and
exports every entry point declared in include/npub.h.
"""
import os
import subprocess
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
GOLDEN = os.path.join(ROOT, "tests", "golden")
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA sm_100 device (B200)")


@pytest.fixture(scope="session", autouse=True)
def _oracle_built():
    """Build the oracle's C restatement (and the reference simulator when the
    reference tree is present) once per session."""
    subprocess.run(["make", "-s", "-C", os.path.join(ROOT, "oracle")], check=True,
                   stdout=subprocess.DEVNULL)
    yield


@pytest.fixture(scope="session")
def libnpub_path():
    from npu_comp_b200 import _lib
    if not os.path.exists(_lib.LIB_PATH):
        from npu_comp_b200 import build
        build.build()
    return _lib.LIB_PATH


@pytest.fixture(scope="session")
def examples():
    return dict(np.load(os.path.join(GOLDEN, "examples.npz")))


@pytest.fixture(scope="session")
def cuda_device():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from npu_comp_b200 import _lib
    _lib.load()
    return torch.device("cuda", 0)


@pytest.fixture()
def rng():
    return np.random.default_rng(1234)
