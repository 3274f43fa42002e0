"""GPU parity of the SIMT GEMV (gemv.cu) for 1..4 tokens on tiled weights,
forced with MRT_GEMV=1 and every row-quad split (MRT_GEMV_RQ), against the
oracle (the reference's CpuBackend::gemm arithmetic) and the FP64 ground
truth; the bias, residual, SwiGLU and FP32-output epilogues against the reference's
own post-GEMM steps, bit for bit."""
import numpy as np
import pytest
import torch

from gpu_util import (BF16, FP16, abs_dot, check_close, dev_u16, f64_truth, gemm, host_u16, rel_frob, same_fraction,
                      stream, upload)
from mruntime_b200 import capi
from mruntime_b200 import workloads as W
from oracle import oracle as O

pytestmark = pytest.mark.gpu


def rand_f16(rng, shape, std=1.0):
    return W.to_f16_bits(rng.standard_normal(shape, dtype=np.float32) * np.float32(std))


def rand_w(rng, shape, dt):
    v = rng.standard_normal(shape, dtype=np.float32) * np.float32(0.02)
    return W.to_f16_bits(v) if dt == FP16 else W.to_bf16_bits(v)


@pytest.fixture
def gemv(monkeypatch):
    monkeypatch.setenv("MRT_GEMV", "1")
    return monkeypatch


# Ragged rows (N not a multiple of 4 or 32), K of one partial tile, K not a
# multiple of 64, the config-1 decode shape and a long K.
SHAPES = [(200, 64), (257, 136), (1000, 896), (4864, 896), (130, 72), (896, 4864)]


@pytest.mark.parametrize("rq", [1, 2, 4, 8, 0])
@pytest.mark.parametrize("NK", SHAPES)
@pytest.mark.parametrize("M", [1, 2, 3, 4])
def test_gemv_matches_oracle(cuda_dev, gemv, M, NK, rq):
    if rq:
        gemv.setenv("MRT_GEMV_RQ", str(rq))
    N, K = NK
    rng = np.random.default_rng(1000 + M * 31 + N + K + rq)
    x = rand_f16(rng, (M, K))
    w = rand_w(rng, (N, K), BF16)
    wt = upload(w, BF16)
    y = gemm(wt, x)
    y_or = O.gemm(x, FP16, w, BF16, trans_b=True)
    truth = f64_truth(x, w, BF16)
    check_close(y, truth, rel_frob(y_or, truth), f"gemv M={M} N={N} K={K} rq={rq}", absdot=abs_dot(x, w, BF16), K=K)
    assert same_fraction(y, y_or) > 0.9
    wt.free()


def test_gemv_is_deterministic_and_close_to_tensor_core_path(cuda_dev, monkeypatch):
    rng = np.random.default_rng(77)
    N, K = 4864, 896
    x = rand_f16(rng, (1, K))
    w = rand_w(rng, (N, K), FP16)
    wt = upload(w, FP16)
    monkeypatch.setenv("MRT_GEMV", "1")
    a, b = gemm(wt, x), gemm(wt, x)
    np.testing.assert_array_equal(a, b)
    monkeypatch.setenv("MRT_GEMV", "0")
    tc = gemm(wt, x)
    truth = f64_truth(x, w, FP16)
    assert rel_frob(a, truth) < 1e-3 and rel_frob(tc, truth) < 1e-3
    assert same_fraction(a, tc) > 0.95
    wt.free()


@pytest.mark.parametrize("M", [1, 4])
def test_gemv_bias_double_rounding(cuda_dev, gemv, M):
    rng = np.random.default_rng(50 + M)
    N, K = 1152, 896
    x = rand_f16(rng, (M, K))
    w = rand_w(rng, (N, K), BF16)
    b = rand_w(rng, (N,), BF16)
    wt = upload(w, BF16)
    bd = dev_u16(b)
    wt.attach_bias(bd.data_ptr(), BF16, True, stream())
    y_plain = gemm(wt, x)
    y_bias = gemm(wt, x, bias=True)
    np.testing.assert_array_equal(y_bias, O.add_bias(y_plain, W.bf16_to_f16_bits(b)))  # qwen_model.cpp:130-155
    wt.free()


@pytest.mark.parametrize("inplace", [False, True])
@pytest.mark.parametrize("M", [1, 3])
def test_gemv_residual(cuda_dev, gemv, M, inplace):
    rng = np.random.default_rng(60 + M)
    N, K = 896, 4864
    x = rand_f16(rng, (M, K))
    w = rand_w(rng, (N, K), BF16)
    res = rand_f16(rng, (M, N))
    wt = upload(w, BF16)
    want = O.add(res, gemm(wt, x))  # CpuBackend::add after the product (qwen_model.cpp:316, 324)
    xd = dev_u16(x)
    ld = N + (0 if inplace else 8)
    resd = torch.zeros((M, ld), dtype=torch.int16, device="cuda")
    resd[:, :N] = dev_u16(res)
    out = resd if inplace else torch.zeros((M, ld), dtype=torch.int16, device="cuda")
    capi.gemm_residual(wt, xd.data_ptr(), K, resd.data_ptr(), ld, out.data_ptr(), ld, M, False, stream())
    capi.sync(stream())
    np.testing.assert_array_equal(host_u16(out)[:, :N], want)
    wt.free()


@pytest.mark.parametrize("M", [1, 2])
def test_gemv_f32_output(cuda_dev, gemv, M):
    rng = np.random.default_rng(70 + M)
    N, K = 3584, 448
    x = rand_f16(rng, (M, K))
    w = rand_w(rng, (N, K), FP16)
    wt = upload(w, FP16)
    xd = dev_u16(x)
    y = torch.empty((M, N), dtype=torch.float32, device="cuda")
    capi.gemm_f32(wt, xd.data_ptr(), K, y.data_ptr(), N, M, stream())
    capi.sync(stream())
    truth = f64_truth(x, w, FP16)
    assert np.linalg.norm(y.cpu().numpy() - truth) / np.linalg.norm(truth) < 1e-5
    wt.free()


@pytest.mark.parametrize("MIK", [(1, 2304, 3584), (1, 448, 896), (2, 1000, 904), (4, 18944, 3584)])
def test_gemv_swiglu(cuda_dev, gemv, MIK):
    """mrt_gemm_swiglu through the GEMV's SwiGLU epilogue equals the GEMV's
    plain gate and up outputs put through the FP16 SiLU and the rounded
    multiply (qwen_model.cpp:278-285)."""
    from test_gemm_gpu import _silu_table_f16

    M, I, K = MIK
    rng = np.random.default_rng(M + I + K + 5)
    x = rand_f16(rng, (M, K))
    w = rand_w(rng, (2 * I, K), BF16)  # row 2j = gate j, row 2j + 1 = up j
    wt = upload(w, BF16)
    y = gemm(wt, x)
    xd = dev_u16(x)
    act = torch.empty((M, I), dtype=torch.int16, device="cuda")
    capi.gemm_swiglu(wt, xd.data_ptr(), K, act.data_ptr(), I, M, stream())
    capi.sync(stream())
    got = host_u16(act)
    lut = _silu_table_f16()
    want = W.to_f16_bits(W.f16_bits_to_f32(lut[y[:, 0::2]]).astype(np.float32) *
                         W.f16_bits_to_f32(y[:, 1::2]).astype(np.float32))
    same = got == want
    if not same.all():
        # only a SiLU input whose exp differs from the host's in the last bit
        diff = np.abs(got.astype(np.int32) - want.astype(np.int32))
        assert same.mean() > 0.9999 and diff.max() <= 1, (MIK, same.mean(), diff.max())
    wt.free()
