"""CudaBackend (C++ mruntime::Backend) drop-in tests on the GPU.

* tests/cpp/_build/cuda_backend_test (tests/cpp/cuda_backend_test.cpp): every
  Backend op against the reference's CpuBackend on the same seeded inputs.
* tests/cpp/_build/ref_engine_cuda (oracle/ref_shim/ref_engine.cpp built with
  -DREF_ENGINE_CUDA): the reference's own QwenModel + InferenceEngine driving
  CudaBackend, with and without the reference's ProfilingBackend around it,
  must pick the reference engine's greedy tokens on the tiny checkpoint
  (tests/golden/decode_tiny_greedy.json).  The 7B-width case is in
  test_golden_7b_gpu.py."""
import json
import os
import subprocess
import sys

import pytest

from conftest import GOLDEN, ROOT

sys.path.insert(0, GOLDEN)
import gen_decode_7b as G  # noqa: E402

pytestmark = pytest.mark.gpu

BIN = os.path.join(ROOT, "tests", "cpp", "_build", "cuda_backend_test")
ENGINE_CUDA = os.path.join(ROOT, "tests", "cpp", "_build", "ref_engine_cuda")


def test_cuda_backend_drop_in(cuda_dev):
    assert os.path.exists(BIN), f"{BIN} missing: run `make -C tests/cpp` (needs the reference headers)"
    r = subprocess.run([BIN], capture_output=True, text=True, timeout=600)
    print(r.stdout)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
    assert "All CudaBackend tests passed!" in r.stdout


@pytest.mark.parametrize("profile", [False, True], ids=["plain", "ProfilingBackend"])
def test_reference_engine_on_cuda_backend_tiny(cuda_dev, tmp_path, profile):
    assert os.path.exists(ENGINE_CUDA), f"{ENGINE_CUDA} missing: run `make -C tests/cpp engine_cuda`"
    with open(os.path.join(GOLDEN, "decode_tiny_greedy.json")) as f:
        g = json.load(f)
    paths = G.write_checkpoint(str(tmp_path), g["config"], g["seed"], g["prompt_len"])
    assert paths["weights_sha256"] == g["weights_sha256"]
    info = G.run_engine(ENGINE_CUDA, paths, g["max_new"], profile=profile, timeout=600, nice=False)
    print(info["backend"], info["tokens"], "margins", info.get("margins"))
    assert info["backend"] == "CudaBackend" + ("+ProfilingBackend" if profile else "")
    assert info["tokens"] == g["tokens"], f"CudaBackend engine {info['tokens']} != reference {g['tokens']}"
    if profile:
        layers = g["config"]["num_hidden_layers"]
        n_forward = g["prompt_len"] + g["max_new"]
        assert info["profile"]["gemm"]["calls"] == n_forward * (7 * layers + 1)
        assert info["profile"]["embedding_lookup"]["calls"] == n_forward
