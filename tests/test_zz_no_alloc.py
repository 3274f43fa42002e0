"""mrt_argmax_f16_noalloc: the greedy pick for callers that cannot allocate
device memory (a decode step captured in a CUDA graph cannot call cudaMalloc
or take the device-wide synchronisation of a cudaFree; serving runtimes may
own every byte of device memory through their own arenas).  Its partials
live in a fixed 96 KiB buffer inside the library.

Checks, through the C ABI: two calls in a row on different logits give
exactly the indices and values of the allocating entry point mrt_argmax_f16
(both use the same kernels; the tolerance for these integer and copied values
is zero), the second call changes no device memory usage, and a call beyond
the buffer's limit is refused.  Collected last (file name) so a failure here
never hides the other tests; it passes alone in a fresh process too."""
import ctypes as C

import numpy as np
import pytest
import torch

from mruntime_b200 import capi
from mruntime_b200 import workloads as W

pytestmark = pytest.mark.gpu


def _logits(seed: int, M: int, V: int) -> torch.Tensor:
    rng = np.random.default_rng(seed)
    h = W.to_f16_bits(rng.standard_normal((M, V), dtype=np.float32) * np.float32(4.0))
    h[:, 7] = 0x7E00            # NaN never wins
    h[0, 3] = h[0, V - 5] = 0x7BFF  # tie on the largest value: first index wins
    return torch.from_numpy(h.view(np.int16)).cuda()


def _pick(fn: str, logits: torch.Tensor, base: int):
    M, V = logits.shape
    idx = torch.full((M,), -1, dtype=torch.int64, device="cuda")
    val = torch.full((M,), float("nan"), dtype=torch.float32, device="cuda")
    s = torch.cuda.current_stream().cuda_stream
    capi.call(fn, logits.data_ptr(), M, V, V, base, idx.data_ptr(), val.data_ptr(), s)
    capi.sync(s)
    return idx.cpu().numpy(), val.cpu().numpy()


def test_noalloc_argmax_matches_allocating_entry_point(cuda_dev):
    cases = [(11, 8, 152064, 0), (12, 37, 151936, 1000)]  # two calls in a row, different shapes
    for n, (seed, M, V, base) in enumerate(cases):
        logits = _logits(seed, M, V)
        want_idx, want_val = _pick("mrt_argmax_f16", logits, base)
        torch.cuda.synchronize()
        free_before = torch.cuda.mem_get_info()[0]
        got_idx, got_val = _pick("mrt_argmax_f16_noalloc", logits, base)
        free_after = torch.cuda.mem_get_info()[0]
        np.testing.assert_array_equal(got_idx, want_idx)
        np.testing.assert_array_equal(got_val.view(np.uint32), want_val.view(np.uint32))
        assert got_idx[0] == base + 3
        if n > 0:  # the first call may load the library's device module; later calls allocate nothing
            assert free_after == free_before


def test_noalloc_argmax_rejects_oversized_calls(cuda_dev):
    logits = torch.zeros((432, 152064), dtype=torch.int16, device="cuda")  # 432 * 19 chunks > 8192 pairs
    idx = torch.empty(432, dtype=torch.int64, device="cuda")
    rc = capi.lib().mrt_argmax_f16_noalloc(logits.data_ptr(), 432, 152064, 152064, 0, idx.data_ptr(), None,
                                           C.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert rc == 2  # MRT_ERR_SHAPE
    assert b"static buffer" in capi.lib().mrt_last_error_string()
