"""CudaBackend (C++ mruntime::Backend) drop-in test on the GPU.

Runs tests/cpp/_build/cuda_backend_test, built by tests/cpp/Makefile against
the reference's headers and its CpuBackend (oracle/_ref); see that file for
what it checks."""
import os
import subprocess

import pytest

from conftest import ROOT

pytestmark = pytest.mark.gpu

BIN = os.path.join(ROOT, "tests", "cpp", "_build", "cuda_backend_test")


def test_cuda_backend_drop_in(cuda_dev):
    assert os.path.exists(BIN), f"{BIN} missing: run `make -C tests/cpp` (needs the reference headers)"
    r = subprocess.run([BIN], capture_output=True, text=True, timeout=600)
    print(r.stdout)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
    assert "All CudaBackend tests passed!" in r.stdout
