import os
import sys

import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
for p in (REPO, os.path.join(REPO, "oracle"), os.path.join(REPO, "tests", "golden"),
          os.path.join(REPO, "ameva-forge_b200")):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200); parity tests proper")


@pytest.fixture(scope="session")
def golden():
    import numpy as np
    return np.load(os.path.join(REPO, "tests", "golden", "reference_golden.npz"))


@pytest.fixture(scope="session")
def ctx():
    """One device context for the GPU tests (the library's default)."""
    import forge_b200
    c = forge_b200.Context(device=0)
    yield c
    c.shutdown()


def max_rel_err(out, ref):
    """max |out - ref| / max |ref| -- the tolerance measure of the parity bar."""
    import numpy as np
    ref = np.asarray(ref, np.float64)
    return float(np.abs(np.asarray(out, np.float64) - ref).max() / max(np.abs(ref).max(), 1e-30))
