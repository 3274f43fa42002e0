import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

GOLDEN = os.path.join(ROOT, "tests", "golden")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) GPU")
    config.addinivalue_line("markers", "multigpu: needs two or more GPUs")


def golden(name: str):
    return np.load(os.path.join(GOLDEN, name))


@pytest.fixture(scope="session")
def cuda_dev():
    """Current CUDA device with the library's context created (GPU tests only)."""
    import torch

    if not torch.cuda.is_available():
        pytest.fail("GPU test collected on a host without CUDA; run `pytest -m 'not gpu'` here")
    from mruntime_b200 import capi

    torch.cuda.set_device(0)
    capi.init(0)
    return torch.device("cuda", 0)


def pytest_sessionfinish(session, exitstatus):
    """With MRT_ERR_LOG set, write every (case, device error, reference error)
    the tolerance checks saw, and the largest ratio, to that file."""
    path = os.environ.get("MRT_ERR_LOG")
    if not path or "gpu_util" not in sys.modules:
        return
    rows = sys.modules["gpu_util"].ERR_RATIOS
    with open(path, "w") as f:
        for what, err, ref in rows:
            f.write(f"{err / ref:.6f} {err:.6e} {ref:.6e} {what}\n")
        if rows:
            f.write(f"max ratio {max(e / r for _, e, r in rows):.6f} over {len(rows)} checks\n")
