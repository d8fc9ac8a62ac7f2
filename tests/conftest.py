import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")


@pytest.fixture(scope="session")
def fla_golden():
    """The reference's float64 golden vectors (src/delta/tests/reference.rs)."""
    import json

    import numpy as np

    path = os.path.join(ROOT, "tests", "golden", "fla_naive_b2_t9_h2_k4_v6.json")
    fx = json.load(open(path))
    out = {k: np.array(v["data"], dtype=np.float64).reshape(v["shape"]) for k, v in fx["tensors"].items()}
    out["dims"] = fx["dims"]
    return out
