"""Shared fixtures.  CPU tests (-m "not gpu") check the oracle against the
reference's golden vectors, the host-side logic of the library and its
exported C ABI; GPU tests (-m gpu) are the parity tests of the kernels."""
import os
import subprocess
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(ROOT, "k-mamba_b200")
sys.path.insert(0, PKG)
sys.path.insert(0, os.path.join(ROOT, "oracle"))
os.environ.setdefault("OMP_NUM_THREADS", "1")

import kmamba_b200 as kb  # noqa: E402


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200)")


def _ensure_built():
    if not os.path.exists(kb.LIB_PATH):
        subprocess.run(["make", "-s", "-C", PKG], check=True)


@pytest.fixture(scope="session")
def lib():
    _ensure_built()
    return kb.load()


@pytest.fixture(scope="session")
def oracle():
    import oracle as o
    if not os.path.exists(o.ORACLE_SO):
        o.build()
    return o


@pytest.fixture(scope="session")
def golden():
    d = os.path.join(ROOT, "tests", "golden")

    def load(name):
        z = np.load(os.path.join(d, name))
        cases = {}
        for k in z.files:
            tag, field = k.split("/")
            cases.setdefault(tag, {})[field] = z[k]
        return cases
    return load


def rel_err(a, b):
    """max|a-b| / max(|b|, tau), tau = 1e-3 * rms(b): the per-tensor relative
    error used by every parity test (near-zero entries do not dominate)."""
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    if b.size == 0:
        return 0.0
    tau = 1e-3 * np.sqrt(np.mean(b * b)) + 1e-30
    return float(np.max(np.abs(a - b) / np.maximum(np.abs(b), tau)))


@pytest.fixture(scope="session")
def cuda():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch.device("cuda:0")
