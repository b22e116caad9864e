"""Shared test setup. GPU tests are marked `gpu` and need a CUDA device (a B200); everything else runs on CPU.
The oracle (oracle/) is only ever the checker here."""
import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

REFERENCE = "/root/reference"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200); run with -m gpu")
    config.addinivalue_line("markers", "reference: needs the reference sources or the compiled reference (oracle/_ref)")


@pytest.fixture(scope="session")
def libkx():
    """libkernix.so, built in-tree (the CUDA path; there is no fallback)."""
    from kernix_b200 import build, kx_abi
    build.build()
    return kx_abi.lib()


@pytest.fixture(scope="session")
def model_dir(tmp_path_factory):
    return str(tmp_path_factory.mktemp("models"))


def rel_err(got, want):
    """max |got - want| / max(1, max |want|), NaNs must match."""
    got = np.asarray(got, np.float64)
    want = np.asarray(want, np.float64)
    assert got.shape == want.shape, (got.shape, want.shape)
    gn, wn = np.isnan(got), np.isnan(want)
    assert np.array_equal(gn, wn), f"NaN pattern differs: {gn.sum()} vs {wn.sum()}"
    d = np.abs(np.where(gn, 0, got) - np.where(wn, 0, want))
    return float(d.max(initial=0.0) / max(1.0, float(np.abs(np.where(wn, 0, want)).max(initial=0.0))))
