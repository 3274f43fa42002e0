"""The SM-pair GEMM (tcgen05.mma.cta_group::2, 256-row tiles over two SMs)
against the one-SM kernel and the oracle.

MRT_GEMM_PAIR=1 (read at every plan) makes the planner hand every eligible
normal-mode GEMM (M >= 256, K <= 4096, tiled weights) to the pair kernel and
MRT_GEMM_PAIR=0 none of them (without the variable the planner compares
costs).  Both accumulate every output over K in
the same 16-wide steps, so their outputs are compared bit for bit, and the
pair's against the reference's arithmetic within the suite's tolerance."""
import os

import numpy as np
import pytest
import torch

from gpu_util import BF16, FP16, abs_dot, check_close, dev_u16, f64_truth, host_u16, stream, upload
from mruntime_b200 import capi
from mruntime_b200 import workloads as W
from oracle import oracle as O

pytestmark = pytest.mark.gpu


def _rand(rng, shape, std):
    return W.to_f16_bits(rng.standard_normal(shape, dtype=np.float32) * np.float32(std))


def _run(wt, x, flags=0, out_f32=False, residual=None):
    M, K = x.shape
    xd = dev_u16(x)
    if out_f32:
        y = torch.empty((M, wt.n), dtype=torch.float32, device="cuda")
        capi.gemm_f32(wt, xd.data_ptr(), K, y.data_ptr(), wt.n, M, stream())
        capi.sync(stream())
        return y.cpu().numpy()
    y = torch.empty((M, wt.n), dtype=torch.int16, device="cuda")
    if residual is not None:
        rd = dev_u16(residual)
        capi.gemm_residual(wt, xd.data_ptr(), K, rd.data_ptr(), wt.n, y.data_ptr(), wt.n, M, bool(flags), stream())
    else:
        capi.gemm(wt, xd.data_ptr(), K, y.data_ptr(), wt.n, M, bool(flags), stream())
    capi.sync(stream())
    return host_u16(y)


def _both(fn):
    os.environ["MRT_GEMM_PAIR"] = "0"
    one = fn()
    os.environ["MRT_GEMM_PAIR"] = "1"
    try:
        two = fn()
    finally:
        os.environ.pop("MRT_GEMM_PAIR", None)
    return one, two


# (M, N, K): ragged M and N, K of one k-block, K not a multiple of 64, the
# 7B q|k|v and gate+up widths; then K longer than 64 k-blocks (segmented
# accumulation in the pair kernel), the 7B down projection among them.
SHAPES = [(256, 256, 64), (300, 1000, 904), (512, 4608, 3584), (2048, 2304, 3584), (257, 37888, 896),
          (512, 1000, 8192), (300, 3584, 18944), (2048, 512, 18944)]


@pytest.mark.parametrize("MNK", SHAPES)
def test_pair_matches_one_sm_and_oracle(cuda_dev, MNK):
    M, N, K = MNK
    rng = np.random.default_rng(M + N + K)
    x = _rand(rng, (M, K), 1.0)
    w = W.to_bf16_bits(rng.standard_normal((N, K), dtype=np.float32) * np.float32(0.02))
    wt = upload(w, BF16)
    os.environ["MRT_GEMM_PAIR"] = "1"
    p = capi.gemm_plan(M, N, K)
    os.environ.pop("MRT_GEMM_PAIR", None)
    assert p["pair"], p
    one, two = _both(lambda: _run(wt, x))
    if K <= 64 * 64:
        # same 16-wide steps in the same order: bit for bit
        np.testing.assert_array_equal(two, one)
    else:
        # 64-k-block segments summed in registers (the one-SM plan may cut K
        # into slices instead): both within the tolerance below
        assert np.mean(two == one) > 0.9
    rows = np.unique(np.r_[0:4, M // 2, M - 4:M])
    xs = x[rows]
    truth = f64_truth(xs, w, BF16)
    ref = O.gemm(xs, FP16, w, BF16, trans_b=True)
    check_close(two[rows], truth, O.rel_frobenius(ref, truth), f"pair {MNK}", absdot=abs_dot(xs, w, BF16), K=K)


def test_pair_epilogues(cuda_dev):
    """Bias (double rounding), FP32 output and the residual add through the
    pair kernel equal the one-SM kernel's."""
    rng = np.random.default_rng(77)
    M, N, K = 384, 1152, 896
    x = _rand(rng, (M, K), 1.0)
    w = W.to_bf16_bits(rng.standard_normal((N, K), dtype=np.float32) * np.float32(0.02))
    b = W.to_bf16_bits(rng.standard_normal(N, dtype=np.float32) * np.float32(0.02))
    res = _rand(rng, (M, N), 1.0)
    wt = upload(w, BF16)
    bd = dev_u16(b)
    wt.attach_bias(bd.data_ptr(), BF16, True, stream())
    for kw in ({"flags": 1}, {"out_f32": True}, {"residual": res}):
        one, two = _both(lambda: _run(wt, x, **kw))
        if kw.get("out_f32"):
            np.testing.assert_array_equal(two.view(np.uint32), one.view(np.uint32))
        else:
            np.testing.assert_array_equal(two, one)


def _forced_splits(n, fn):
    os.environ["MRT_GEMM_PAIR_SPLITS"] = str(n)
    try:
        return fn()
    finally:
        os.environ.pop("MRT_GEMM_PAIR_SPLITS", None)


# (M, N, K, slices): K-split tails on SM pairs -- whole waves of 74 pairs over
# the whole K and the last partial wave's tiles cut into K-slices, or (fewer
# tiles than pairs) every tile cut; slices of one k-block, ragged last slices,
# and slices longer than 64 k-blocks (segmented accumulation), the 7B o and
# down projections at M = 2048 among them.
TAIL_SHAPES = [(2048, 3584, 3584, 3), (2048, 3584, 18944, 2), (2048, 3584, 18944, 7), (300, 1000, 904, 3),
               (257, 640, 128, 2), (512, 1000, 8192, 5), (2304, 2304, 1000, 16)]


@pytest.mark.parametrize("MNKS", TAIL_SHAPES)
def test_pair_k_split_tails(cuda_dev, MNKS):
    """Pair plans with K-split tails: within the reference's error bars on
    sampled rows (tail tiles included), close to the whole-K pair plan, and
    repeatable bit for bit (slices are summed in slice order)."""
    M, N, K, n = MNKS
    rng = np.random.default_rng(M * 7 + N + K + n)
    x = _rand(rng, (M, K), 1.0)
    w = W.to_bf16_bits(rng.standard_normal((N, K), dtype=np.float32) * np.float32(0.02))
    wt = upload(w, BF16)
    p = _forced_splits(n, lambda: capi.gemm_plan(M, N, K, 148))
    tiles = -(-M // 256) * -(-N // 256)
    assert p["pair"] and p["full_tiles"] == (tiles // 74) * 74 and p["tail_splits"] >= 2, p
    if torch.cuda.get_device_properties(0).multi_processor_count != 148:
        pytest.skip("the forced plan is laid out for 148 SMs")
    got = _forced_splits(n, lambda: _run(wt, x))
    again = _forced_splits(n, lambda: _run(wt, x))
    np.testing.assert_array_equal(got, again)
    os.environ["MRT_GEMM_PAIR"] = "1"
    try:
        whole = _run(wt, x)
    finally:
        os.environ.pop("MRT_GEMM_PAIR", None)
    assert np.mean(got == whole) > 0.8
    # rows of the first m-tiles and the last (tail tiles are the last in
    # m-fastest order: every m-tile of the last n-tiles)
    rows = np.unique(np.r_[0:4, 130:132, M // 2, M - 4:M])
    xs = x[rows]
    truth = f64_truth(xs, w, BF16)
    ref = O.gemm(xs, FP16, w, BF16, trans_b=True)
    check_close(got[rows], truth, O.rel_frobenius(ref, truth), f"pair tails {MNKS}", absdot=abs_dot(xs, w, BF16),
                K=K)


def test_pair_k_split_tail_epilogues(cuda_dev):
    """Bias (double rounding), FP32 output and the residual add of tail
    tiles come from the tail reduction: each equals the reference's
    operation applied to the same plan's plain output."""
    if torch.cuda.get_device_properties(0).multi_processor_count != 148:
        pytest.skip("the forced plan is laid out for 148 SMs")
    rng = np.random.default_rng(78)
    M, N, K = 384, 1152, 896
    x = _rand(rng, (M, K), 1.0)
    w = W.to_bf16_bits(rng.standard_normal((N, K), dtype=np.float32) * np.float32(0.02))
    b = W.to_bf16_bits(rng.standard_normal(N, dtype=np.float32) * np.float32(0.02))
    res = _rand(rng, (M, N), 1.0)
    wt = upload(w, BF16)
    bd = dev_u16(b)
    wt.attach_bias(bd.data_ptr(), BF16, True, stream())
    plain = _forced_splits(3, lambda: _run(wt, x))
    with_bias = _forced_splits(3, lambda: _run(wt, x, flags=1))
    np.testing.assert_array_equal(with_bias, O.add_bias(plain, W.bf16_to_f16_bits(b)))
    y32 = _forced_splits(3, lambda: _run(wt, x, out_f32=True))
    np.testing.assert_array_equal(O.f32_to_f16(y32), plain)
    with_res = _forced_splits(3, lambda: _run(wt, x, residual=res))
    np.testing.assert_array_equal(with_res, O.add(res, plain))


def test_pair_no_timeout(cuda_dev):
    capi.sync(stream())
