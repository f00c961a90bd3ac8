"""Shared fixtures.  GPU tests carry @pytest.mark.gpu; everything else runs on CPU.

The oracle (oracle/) is the checker here and only here: tests compare the
CUDA library, called through its C ABI, against it.
"""
import pathlib
import sys

import numpy as np
import pytest

ROOT = pathlib.Path(__file__).resolve().parent.parent
for p in (ROOT / "google-classic_b200", ROOT / "oracle"):
    if str(p) not in sys.path:
        sys.path.insert(0, str(p))

import holo_b200 as hb  # noqa: E402
import holo_oracle  # noqa: E402

GOLDEN = ROOT / "tests" / "golden"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (runs the CUDA library)")


@pytest.fixture(scope="session")
def oracle():
    return holo_oracle.Oracle()


@pytest.fixture(scope="session")
def reference():
    try:
        return holo_oracle.Reference()
    except RuntimeError as e:  # neither prebuilt nor buildable here
        pytest.skip(str(e))


@pytest.fixture(scope="session")
def lib():
    return hb.load()


@pytest.fixture(scope="session")
def dev():
    d = hb.Device(0, 1)
    yield d


def rel_err(y, r):
    """max |y - r| / max |r|: the norm-wise relative error of the parity bar."""
    y = np.asarray(y, np.float64)
    r = np.asarray(r, np.float64)
    return float(np.abs(y - r).max() / max(np.abs(r).max(), 1e-30))
