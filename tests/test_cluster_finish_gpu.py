"""Swap-mode K-split finish inside thread-block clusters.

Few-token products (17 <= M <= 64) whose every weight tile is split into 2..8
K-slices, one slice per CTA, sum the slices through distributed shared memory
of a cluster instead of through global memory.  Both finishes add the slices
in slice order, so the cluster finish must reproduce the global-memory finish
(MRT_GEMM_CLUSTER=0, run in a child process) bit for bit, and both must meet
the oracle's tolerance.
"""
from __future__ import annotations

import os
import subprocess
import sys

import numpy as np
import pytest
import torch

from gpu_util import BF16, FP16, dev_u16, gemm, stream, upload
from mruntime_b200 import capi
from mruntime_b200 import workloads as W
from oracle import oracle as O

pytestmark = pytest.mark.gpu

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)

# (M, N, K, bias, fp32 output): the 7B projections q|k|v, o and down at 9..64
# tokens (tile widths 16, 32 and 64), token counts that leave a partial 16-column
# chunk, N not a multiple of 4 with K not a multiple of 64 (and unaligned
# output rows), the q/k/v bias and the FP32 output.
CASES = [
    (12, 4608, 3584, False, False),
    (16, 3584, 3584, False, False),
    (9, 3584, 3584, True, False),
    (17, 4608, 3584, False, False),
    (20, 3584, 3584, False, False),
    (32, 3584, 18944, False, False),
    (33, 4608, 3584, False, False),
    (47, 3584, 18944, False, False),
    (64, 3584, 3584, False, False),
    (18, 3581, 3576, False, False),
    (40, 3581, 3576, False, False),
    (24, 4608, 3584, True, False),
    (64, 4608, 3584, True, False),
    (36, 3584, 3584, False, True),
]


def _inputs(i: int, M: int, N: int, K: int):
    rng = np.random.default_rng(1000 + i)
    x = W.to_f16_bits(rng.standard_normal((M, K), dtype=np.float32))
    w = W.to_bf16_bits(rng.standard_normal((N, K), dtype=np.float32) * np.float32(0.02))
    b = W.to_bf16_bits(rng.standard_normal((N,), dtype=np.float32) * np.float32(0.5))
    return x, w, b


def _run(i: int, case) -> np.ndarray:
    """y (FP16 bits, or FP32) of case i through the C ABI on cuda:0."""
    M, N, K, bias, f32 = case
    x, w, b = _inputs(i, M, N, K)
    wt = upload(w, BF16)
    if bias:
        bd = dev_u16(b)
        wt.attach_bias(bd.data_ptr(), BF16, True, stream())
        torch.cuda.synchronize()
    if f32:
        xd = dev_u16(x)
        y = torch.empty((M, N), dtype=torch.float32, device="cuda")
        capi.gemm_f32(wt, xd.data_ptr(), K, y.data_ptr(), N, M, stream())
        capi.sync(stream())
        out = y.cpu().numpy()
    else:
        out = gemm(wt, x, bias=bias)
    wt.free()
    return out


def _child_outputs(tmp_path) -> dict:
    """Every case with the global-memory finish, in a child process."""
    out = tmp_path / "global_finish.npz"
    code = (
        "import sys, json, numpy as np\n"
        f"sys.path[:0] = [{HERE!r}, {ROOT!r}]\n"
        "import test_cluster_finish_gpu as T\n"
        "from mruntime_b200 import capi\n"
        "capi.init(0)\n"
        "res = {}\n"
        "for i, c in enumerate(T.CASES):\n"
        "    p = capi.gemm_plan(c[0], c[1], c[2])\n"
        "    assert not p['cluster'], p\n"
        "    res[f'y{i}'] = T._run(i, c)\n"
        f"np.savez({str(out)!r}, **res)\n"
    )
    env = dict(os.environ, MRT_GEMM_CLUSTER="0")
    r = subprocess.run([sys.executable, "-c", code], env=env, capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
    return dict(np.load(out))


def test_cluster_finish_matches_global_finish_and_oracle(cuda_dev, tmp_path):
    if os.environ.get("MRT_GEMM_CLUSTER") == "0":
        pytest.skip("cluster finish switched off in this process")
    ref = _child_outputs(tmp_path)
    for i, case in enumerate(CASES):
        M, N, K, bias, f32 = case
        p = capi.gemm_plan(M, N, K)
        assert p["kernel"] == "tcgen05-swap" and p["cluster"], (case, p)
        got = _run(i, case)
        want = ref[f"y{i}"]
        if f32:
            np.testing.assert_array_equal(got.view(np.uint32), want.view(np.uint32), err_msg=str(case))
        else:
            np.testing.assert_array_equal(got, want, err_msg=str(case))
        # Against the oracle (the reference's arithmetic) on a few rows.
        if not f32:
            x, w, b = _inputs(i, M, N, K)
            rows = np.unique(np.r_[0, M // 2, M - 1])
            y_or = O.gemm(x[rows], FP16, w, BF16, trans_b=True)
            if bias:  # qwen_model.cpp:130-155: bias added to the rounded product
                y_or = O.add_bias(y_or, W.bf16_to_f16_bits(b))
            same = float(np.mean(got[rows] == y_or))
            assert same > 0.9, (case, same)
