"""Failure detection on the GPU without a fault: a kernel wait that nothing
will ever satisfy must give up within its limit, report MRT_ERR_TIMEOUT
through mrt_sync, and leave the context usable for the next GEMM."""
import time

import numpy as np
import pytest

from gpu_util import BF16, FP16, REF_ERR_SLACK, gemm, stream, upload
from mruntime_b200 import capi
from mruntime_b200 import workloads as W
from oracle import oracle as O

pytestmark = pytest.mark.gpu


def test_bounded_wait_times_out_and_context_survives(cuda_dev):
    capi.sync(stream())
    t0 = time.perf_counter()
    capi.call("mrt_selftest_wait_timeout", 200, stream())
    with pytest.raises(capi.MrtError) as ei:
        capi.sync(stream())
    elapsed = time.perf_counter() - t0
    assert ei.value.code == capi.MRT_ERR_TIMEOUT
    assert "self-test" in str(ei.value)
    assert 0.15 < elapsed < 5.0
    capi.sync(stream())  # the flag was read and cleared
    rng = np.random.default_rng(9)
    x = W.to_f16_bits(rng.standard_normal((130, 256), dtype=np.float32))
    w = W.to_bf16_bits(rng.standard_normal((192, 256), dtype=np.float32) * np.float32(0.02))
    y = gemm(upload(w, BF16), x)  # a tcgen05 GEMM right after the timeout
    ref = O.gemm(x, O.FP16, w, O.BF16, trans_b=True)
    assert np.mean(y == ref) > 0.9
    assert O.rel_frobenius(y, O.gemm_f64(x, w, O.BF16)) <= O.rel_frobenius(ref, O.gemm_f64(x, w, O.BF16)) * REF_ERR_SLACK


def test_selftest_rejects_bad_limit(cuda_dev):
    with pytest.raises(capi.MrtError):
        capi.call("mrt_selftest_wait_timeout", 0, stream())
