import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

GOLDEN = os.path.join(ROOT, "tests", "golden")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) GPU; the parity tests proper")


@pytest.fixture(scope="session")
def rms_golden():
    """{case: dict(x, w, r, eps, out, res)} from tests/golden/rms_norm_golden.npz."""
    g = np.load(os.path.join(GOLDEN, "rms_norm_golden.npz"))
    cases = {}
    for k in g.files:
        case, field = k.split("__")
        cases.setdefault(case, {})[field] = g[k]
    for c in cases.values():
        c["eps"] = float(c["eps"][0])
    return cases


@pytest.fixture(scope="session")
def relu_golden():
    g = np.load(os.path.join(GOLDEN, "relu_golden.npz"))
    return {dt: (g[f"{dt}__x"], g[f"{dt}__out"]) for dt in ("bf16", "fp16")}


@pytest.fixture(scope="session")
def cuda():
    """The CUDA device for -m gpu tests: fails (never skips) when there is none."""
    import torch

    assert torch.cuda.is_available(), "gpu tests need a CUDA device"
    cap = torch.cuda.get_device_capability()
    assert cap == (10, 0), f"gpu tests need an sm_100 device, got {cap}"
    return torch.device("cuda", torch.cuda.current_device())
