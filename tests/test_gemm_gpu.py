"""GPU parity of the linear-layer path, through the C ABI, against the oracle
(the reference's arithmetic, pinned by tests/test_oracle.py) and the FP64
ground truth, on seeded inputs."""
import numpy as np
import pytest
import torch

from conftest import golden
from gpu_util import (BF16, FP16, FP32, abs_dot, check_close, dev_u16, f64_truth, gemm, host_u16, rel_frob,
                      same_fraction, stream, upload)
from mruntime_b200 import capi
from mruntime_b200 import workloads as W
from oracle import oracle as O

pytestmark = pytest.mark.gpu


def rand_f16(rng, shape, std=1.0):
    return W.to_f16_bits(rng.standard_normal(shape, dtype=np.float32) * np.float32(std))


def rand_w(rng, shape, dt):
    v = rng.standard_normal(shape, dtype=np.float32) * np.float32(0.02)
    return W.to_f16_bits(v) if dt == FP16 else W.to_bf16_bits(v)


# ------------------------------------------------------------------ general contract (bit-exact)

def test_known_answer_backend_test(cuda_dev):
    g = golden("kat_backend_test.npz")
    a, b = dev_u16(g["a"]), dev_u16(g["b"])
    c = torch.zeros((2, 4), dtype=torch.int16, device="cuda")
    capi.gemm_general(a.data_ptr(), FP16, (2, 3), b.data_ptr(), FP16, (3, 4), c.data_ptr(), FP16, stream=stream())
    capi.sync(stream())
    np.testing.assert_array_equal(host_u16(c), g["c"])


def _dev_any(a, dt):
    if dt == FP32:
        return torch.from_numpy(np.ascontiguousarray(a, np.float32)).cuda()
    return dev_u16(a)


def _host_any(t, dt):
    return t.cpu().numpy() if dt == FP32 else host_u16(t)


def test_general_gemm_bitexact_with_reference(cuda_dev):
    g = golden("gemm_small.npz")
    for i in range(int(g["n_cases"])):
        M, N, K, adt, bdt, cdt, ta, tb = (int(v) for v in g[f"c{i}_spec"])
        alpha, beta = (float(v) for v in g[f"c{i}_ab"])
        A, B, C0 = g[f"c{i}_A"], g[f"c{i}_B"], g[f"c{i}_C0"]
        a, b, c = _dev_any(A, adt), _dev_any(B, bdt), _dev_any(C0, cdt)
        capi.gemm_general(a.data_ptr(), adt, A.shape, b.data_ptr(), bdt, B.shape, c.data_ptr(), cdt, alpha, beta,
                          bool(ta), bool(tb), stream())
        capi.sync(stream())
        got = _host_any(c, cdt)
        np.testing.assert_array_equal(got.view(np.uint32) if cdt == FP32 else got,
                                      g[f"c{i}_C"].view(np.uint32) if cdt == FP32 else g[f"c{i}_C"],
                                      err_msg=f"case {i}")


def test_convert_bitexact_with_reference(cuda_dev):
    g = golden("convert.npz")
    src = torch.from_numpy(g["f32_bits"].view(np.float32)).cuda()
    n = src.numel()
    out16 = torch.empty(n, dtype=torch.int16, device="cuda")
    capi.convert(src.data_ptr(), FP32, out16.data_ptr(), FP16, n, stream())
    outb = torch.empty(n, dtype=torch.int16, device="cuda")
    capi.convert(src.data_ptr(), FP32, outb.data_ptr(), BF16, n, stream())
    h = dev_u16(np.arange(65536, dtype=np.uint32).astype(np.uint16))
    out32 = torch.empty(65536, dtype=torch.float32, device="cuda")
    capi.convert(h.data_ptr(), FP16, out32.data_ptr(), FP32, 65536, stream())
    capi.sync(stream())
    np.testing.assert_array_equal(host_u16(out16), g["f16_of_f32"])
    np.testing.assert_array_equal(host_u16(outb), g["bf16_of_f32"])
    got = out32.cpu().numpy()
    want = g["f32_of_f16"].view(np.float32)
    nan = np.isnan(want)
    np.testing.assert_array_equal(np.isnan(got), nan)
    np.testing.assert_array_equal(got[~nan].view(np.uint32), want[~nan].view(np.uint32))


# ------------------------------------------------------------------ weight upload

def weight_fp16(wt) -> np.ndarray:
    """Read back the library-owned FP16 weight as row-major [n, k]."""
    buf = torch.empty((wt.n, wt.k), dtype=torch.int16, device="cuda")
    wt.read(buf.data_ptr(), stream=stream())
    capi.sync(stream())
    return host_u16(buf)


def test_tiled_layout_is_the_swizzled_tile_order(cuda_dev):
    # 128 x 64 tiles, 16-byte chunk c of row r stored at chunk c ^ (r % 8)
    rng = np.random.default_rng(12)
    N, K = 300, 200
    w = W.to_f16_bits(rng.standard_normal((N, K), dtype=np.float32))
    wt = upload(w, FP16)
    assert wt.tiled()
    k_tiles = (K + 63) // 64
    n_pad = (N + 255) // 256 * 256
    raw = torch.empty(n_pad * k_tiles * 64, dtype=torch.int16, device="cuda")
    capi.convert(wt.data_ptr(), FP16, raw.data_ptr(), FP16, raw.numel(), stream())
    capi.sync(stream())
    raw = host_u16(raw)
    r = np.arange(N)[:, None]
    k = np.arange(K)[None, :]
    off = (((r >> 7) * k_tiles + (k >> 6)) << 13) + ((r & 127) << 6) + ((((k & 63) >> 3) ^ (r & 7)) << 3) + (k & 7)
    np.testing.assert_array_equal(raw[off], w)
    pad = np.ones(raw.size, bool)
    pad[off.reshape(-1)] = False
    assert not raw[pad].any()  # padding rows and columns are zero
    np.testing.assert_array_equal(weight_fp16(wt), w)


@pytest.mark.parametrize("M", [3, 70])
def test_general_kernel_reads_tiled_weight(cuda_dev, M):
    # an odd row stride of x sends the call to the general kernel, which reads
    # the weight through the tiled layout; same k-order arithmetic: bit-exact
    rng = np.random.default_rng(M)
    N, K = 130, 96
    x = rand_f16(rng, (M, K))
    w = rand_w(rng, (N, K), FP16)
    wt = upload(w, FP16)
    xs = np.zeros((M, K + 3), np.uint16)
    xs[:, :K] = x
    xd = dev_u16(xs)
    y = torch.empty((M, N), dtype=torch.int16, device="cuda")
    capi.gemm(wt, xd.data_ptr(), K + 3, y.data_ptr(), N, M, False, stream())
    capi.sync(stream())
    np.testing.assert_array_equal(host_u16(y), O.gemm(x, FP16, w, FP16, trans_b=True))


@pytest.mark.parametrize("on_device", [True, False])
@pytest.mark.parametrize("dt", [FP16, BF16, FP32])
def test_upload_rounds_like_reference_packing(cuda_dev, on_device, dt):
    rng = np.random.default_rng(5)
    v = rng.standard_normal((300, 72), dtype=np.float32) * np.float32(0.05)
    v[0, :4] = [1e-7, -3e-9, 70000.0, 2.0 ** -20]
    src = {FP16: W.to_f16_bits(v), BF16: W.to_bf16_bits(v), FP32: v}[dt]
    wt = upload(src, dt, on_device=on_device)
    got = weight_fp16(wt)
    want = {FP16: src, BF16: O.bf16_to_f16(src), FP32: O.f32_to_f16(v)}[dt]
    np.testing.assert_array_equal(got, want)


def test_upload_shards_select_rows_and_columns(cuda_dev):
    rng = np.random.default_rng(6)
    w = rand_w(rng, (96, 64), BF16)
    full = O.bf16_to_f16(w)
    wt = upload(w, BF16, row_ranges=[(8, 24), (48, 56)], k_range=(16, 48))
    assert (wt.n, wt.k) == (24, 32)
    want = np.concatenate([full[8:24, 16:48], full[48:56, 16:48]])
    np.testing.assert_array_equal(weight_fp16(wt), want)


# ------------------------------------------------------------------ fast kernels vs oracle

def _check_against_oracle(x, w, wdt, y, rows=None, what=""):
    idx = np.arange(x.shape[0]) if rows is None else np.asarray(rows)
    xs = x[idx]
    y_or = O.gemm(xs, FP16, w, wdt, trans_b=True)
    truth = f64_truth(xs, w, wdt)
    ref_err = rel_frob(y_or, truth)
    err = check_close(y[idx], truth, ref_err, what, absdot=abs_dot(xs, w, wdt), K=x.shape[1])
    return err, ref_err, same_fraction(y[idx], y_or)


@pytest.mark.parametrize("M", [1, 2, 3, 4, 7, 8, 9, 15, 16, 17, 31, 32, 33, 48, 63, 64])
@pytest.mark.parametrize("NK", [(200, 64), (257, 136), (1000, 896)])
def test_skinny_kernel(cuda_dev, monkeypatch, M, NK):
    monkeypatch.setenv("MRT_GEMV", "0")  # the swap-mode tcgen05 kernel (the GEMV has tests of its own)
    N, K = NK
    rng = np.random.default_rng(M * 7 + N)
    x = rand_f16(rng, (M, K))
    w = rand_w(rng, (N, K), BF16)
    wt = upload(w, BF16)
    y = gemm(wt, x)
    _, _, same = _check_against_oracle(x, w, BF16, y, what=f"skinny M={M} N={N} K={K}")
    assert same > 0.9


@pytest.mark.parametrize("M", [65, 100, 128, 129, 256, 300, 512])
@pytest.mark.parametrize("NK", [(64, 64), (200, 72), (256, 896), (1000, 1000 - 1000 % 8), (4864, 896)])
def test_tensor_core_kernel(cuda_dev, M, NK):
    N, K = NK
    rng = np.random.default_rng(M * 13 + N)
    x = rand_f16(rng, (M, K))
    w = rand_w(rng, (N, K), FP16)
    wt = upload(w, FP16)
    y = gemm(wt, x)
    rows = None if M * N * K <= 300 * 1000 * 1000 else np.r_[0:8, M // 2, M - 8:M]
    _, _, same = _check_against_oracle(x, w, FP16, y, rows, what=f"tc M={M} N={N} K={K}")
    assert same > 0.9


# One shape per tcgen05 plan kind the planner can pick: mode (X or W as the
# 128-row operand) x bn x (every tile over the whole K | whole waves + K-split
# tail (normal mode) | every tile split).  Swap mode's whole-tile plans run
# one or two CTAs per SM (20000 rows: 157 tiles on 157 CTAs).  256-column
# normal-mode tiles need two 128-row m-tiles (single m-tile plans use 128 or
# 64 columns).
PLAN_SHAPES = {
    ("tcgen05", 64, "full"): (65, 64, 64), ("tcgen05", 64, "uniform"): (65, 64, 896),
    ("tcgen05", 128, "full"): (200, 4864, 64), ("tcgen05", 128, "hybrid"): (65, 20000, 2048),
    ("tcgen05", 128, "uniform"): (700, 200, 2048), ("tcgen05", 256, "full"): (129, 40000, 136),
    ("tcgen05", 256, "hybrid"): (129, 20000, 512), ("tcgen05", 256, "uniform"): (129, 4864, 2048),
    ("tcgen05-swap", 16, "full"): (1, 20000, 896), ("tcgen05-swap", 16, "uniform"): (1, 64, 896),
    ("tcgen05-swap", 32, "full"): (17, 20000, 896), ("tcgen05-swap", 32, "uniform"): (17, 64, 896),
    ("tcgen05-swap", 64, "full"): (40, 20000, 896), ("tcgen05-swap", 64, "uniform"): (40, 640, 896),
}


@pytest.mark.parametrize("key", sorted(PLAN_SHAPES))
def test_tensor_core_plan_kinds(cuda_dev, monkeypatch, key):
    monkeypatch.setenv("MRT_GEMV", "0")
    M, N, K = PLAN_SHAPES[key]
    p = capi.gemm_plan(M, N, K)
    tiles = -(-N // 128) if p["kernel"] == "tcgen05-swap" else -(-M // 128) * -(-N // p["bn"])
    kind = "full" if p["full_tiles"] == tiles else ("uniform" if p["full_tiles"] == 0 else "hybrid")
    assert (p["kernel"], p["bn"], kind) == key, p
    rng = np.random.default_rng(M + N + K)
    x = rand_f16(rng, (M, K))
    w = rand_w(rng, (N, K), BF16)
    wt = upload(w, BF16)
    y = gemm(wt, x)
    rows = None if M * N * K <= 100 * 1000 * 1000 else np.r_[0:4, M // 2, M - 4:M]
    _, _, same = _check_against_oracle(x, w, BF16, y, rows, what=f"plan {key} M={M} N={N} K={K}")
    assert same > 0.9


@pytest.mark.parametrize("M", [1, 5, 40, 130])
def test_unaligned_k_uses_general_kernel(cuda_dev, M):
    rng = np.random.default_rng(M)
    K, N = 13, 37
    x = rand_f16(rng, (M, K))
    w = rand_w(rng, (N, K), FP16)
    wt = upload(w, FP16)
    y = gemm(wt, x)
    np.testing.assert_array_equal(y, O.gemm(x, FP16, w, FP16, trans_b=True))  # same sum order: bit-exact


@pytest.mark.parametrize("M", [1, 16, 64, 200])
def test_bias_double_rounding(cuda_dev, M):
    rng = np.random.default_rng(40 + M)
    N, K = 136, 128
    x = rand_f16(rng, (M, K))
    w = rand_w(rng, (N, K), BF16)
    b = rand_w(rng, (N,), BF16)
    wt = upload(w, BF16)
    bd = dev_u16(b)
    wt.attach_bias(bd.data_ptr(), BF16, True, stream())
    y_plain = gemm(wt, x)
    y_bias = gemm(wt, x, bias=True)
    b16 = W.bf16_to_f16_bits(b)
    np.testing.assert_array_equal(y_bias, O.add_bias(y_plain, b16))  # qwen_model.cpp:130-155 exactly
    truth = f64_truth(x, w, BF16, bias=b)
    y_or = O.add_bias(O.gemm(x, FP16, w, BF16, trans_b=True), b16)
    check_close(y_bias, truth, rel_frob(y_or, truth), f"bias M={M}", absdot=abs_dot(x, w, BF16), K=K,
                pre_round=f64_truth(x, w, BF16))


@pytest.mark.parametrize("M", [1, 33, 130, 512])
def test_f32_output(cuda_dev, M):
    rng = np.random.default_rng(90 + M)
    N, K = 264, 512
    x = rand_f16(rng, (M, K))
    w = rand_w(rng, (N, K), FP16)
    wt = upload(w, FP16)
    xd = dev_u16(x)
    y = torch.empty((M, N), dtype=torch.float32, device="cuda")
    capi.gemm_f32(wt, xd.data_ptr(), K, y.data_ptr(), N, M, stream())
    capi.sync(stream())
    truth = f64_truth(x, w, FP16)
    err = np.linalg.norm(y.cpu().numpy() - truth) / np.linalg.norm(truth)
    assert err < 1e-5


def test_zero_rows_is_a_no_op(cuda_dev):
    wt = upload(np.zeros((16, 64), np.uint16), FP16)
    capi.gemm(wt, 0, 64, 0, 16, 0, False, stream())
    capi.sync(stream())


def test_host_buffer_call_matches_device_call(cuda_dev):
    rng = np.random.default_rng(77)
    for M in (1, 300):
        x = rand_f16(rng, (M, 896))
        w = rand_w(rng, (640, 896), BF16)
        wt = upload(w, BF16)
        y_dev = gemm(wt, x)
        y_host = np.empty((M, 640), np.uint16)
        xh = np.ascontiguousarray(x)
        capi.gemm_host(wt, xh.ctypes.data, y_host.ctypes.data, M, False, stream())
        np.testing.assert_array_equal(y_host, y_dev)


@pytest.mark.parametrize("M,N,K,bias", [(256, 640, 896, False), (300, 4608, 3584, True), (1000, 1000, 904, False),
                                        (2048, 3584, 18944, False), (2049, 640, 896, True)])
def test_pinned_host_call_pipelines_row_chunks(cuda_dev, M, N, K, bias):
    """Pinned host buffers take the chunked path (copy in, multiply and copy
    out of different row chunks overlap on three streams), including a ragged
    last chunk and the bias.  Each chunk is its own GEMM, whose plan (and so
    its K-split summation order) may differ from a one-piece call's: the
    result meets the same error bars as the device call, agrees with it on
    the large majority of outputs, and repeats bit for bit."""
    rng = np.random.default_rng(M + N)
    x = rand_f16(rng, (M, K))
    w = rand_w(rng, (N, K), BF16)
    wt = upload(w, BF16)
    bvec = None
    if bias:
        bvec = W.to_bf16_bits(rng.standard_normal(N, dtype=np.float32) * np.float32(0.02))
        b = dev_u16(bvec)
        wt.attach_bias(b.data_ptr(), BF16, True, stream())
    xd = dev_u16(x)
    y_dev = torch.empty((M, N), dtype=torch.int16, device="cuda")
    capi.gemm(wt, xd.data_ptr(), K, y_dev.data_ptr(), N, M, bias, stream())
    capi.sync(stream())
    yd = host_u16(y_dev)
    xh = torch.from_numpy(np.ascontiguousarray(x).view(np.int16)).pin_memory()
    yh = torch.full((M, N), -1, dtype=torch.int16).pin_memory()
    capi.gemm_host(wt, xh.data_ptr(), yh.data_ptr(), M, bias, stream())
    first = yh.numpy().view(np.uint16).copy()
    yh.fill_(-1)
    capi.gemm_host(wt, xh.data_ptr(), yh.data_ptr(), M, bias, stream())  # reuses staging buffers and events
    np.testing.assert_array_equal(yh.numpy().view(np.uint16), first)
    rows = np.unique(np.linspace(0, M - 1, 24).astype(np.int64))
    truth = f64_truth(x[rows], w, BF16, bias=bvec)
    pre = f64_truth(x[rows], w, BF16) if bias else None
    ad = abs_dot(x[rows], w, BF16)
    dev_err = check_close(yd[rows], truth, None, "device call", absdot=ad, K=K, pre_round=pre)
    host_err = check_close(first[rows], truth, None, "pinned host call", absdot=ad, K=K, pre_round=pre)
    assert host_err <= dev_err * 1.01, f"host call error {host_err:.4e} vs device call {dev_err:.4e}"
    assert same_fraction(first, yd) > 0.9


# ------------------------------------------------------------------ argmax

def test_argmax_edge_cases_match_reference(cuda_dev):
    g = golden("bias_argmax.npz")
    for key, am in (("rows", "am_rows"), ("rand", "am_rand")):
        rows = g[key]
        M, V = rows.shape
        d = dev_u16(rows)
        idx = torch.empty(M, dtype=torch.int64, device="cuda")
        capi.argmax_f16(d.data_ptr(), M, V, V, 0, idx.data_ptr(), None, stream())
        capi.sync(stream())
        np.testing.assert_array_equal(idx.cpu().numpy(), g[am])
    # index_base shifts the result (vocabulary shard)
    d = dev_u16(g["rand"][:1])
    idx = torch.empty(1, dtype=torch.int64, device="cuda")
    capi.argmax_f16(d.data_ptr(), 1, g["rand"].shape[1], g["rand"].shape[1], 1000, idx.data_ptr(), None, stream())
    capi.sync(stream())
    assert int(idx.item()) == int(g["am_rand"][0]) + 1000


def test_no_kernel_timed_out(cuda_dev):
    capi.sync(stream())  # raises MrtError(MRT_ERR_TIMEOUT) if any bounded wait gave up


# ------------------------------------------------------------------ gate|up with SwiGLU

def _silu_table_f16() -> np.ndarray:
    """The reference's FP16 SiLU of every FP16 input (qwen_model.cpp:281-283:
    x / (1 + exp(-x)) in FP32, rounded to FP16); exp correctly rounded."""
    x = W.f16_bits_to_f32(np.arange(65536, dtype=np.uint32).astype(np.uint16)).astype(np.float32)
    with np.errstate(over="ignore", invalid="ignore"):
        e = np.exp(-x.astype(np.float64)).astype(np.float32)
        y = x / (np.float32(1.0) + e)
    return W.to_f16_bits(y)


# (M, I, K): fused in the swap epilogue (16-, 64-token tiles), fused in the
# normal-mode epilogue, and K-split plans (global and cluster finish, normal
# mode with a split tail) that take the product-then-pairs route.
SWIGLU_SHAPES = [(1, 18944, 3584), (16, 18944, 3584), (40, 18944, 3584), (300, 18944, 3584),
                 (1, 2304, 3584), (33, 2304, 3584), (65, 10000, 2048)]


@pytest.mark.parametrize("MIK", SWIGLU_SHAPES)
def test_gemm_swiglu(cuda_dev, MIK):
    """mrt_gemm_swiglu on interleaved gate|up rows equals the plain product's
    gate and up outputs put through the FP16 SiLU and the rounded multiply."""
    M, I, K = MIK
    rng = np.random.default_rng(M + I + K)
    x = rand_f16(rng, (M, K))
    w = rand_w(rng, (2 * I, K), BF16)  # row 2j = gate j, row 2j + 1 = up j
    wt = upload(w, BF16)
    p = capi.gemm_plan(M, 2 * I, K)
    if p["kernel"] == "gemv":
        tiles = 0  # the GEMV runs SwiGLU in its own epilogue
    elif p["pair"]:
        tiles = -(-M // 256) * -(-2 * I // 256)  # SM pairs: 256-row tiles, always the whole K
    else:
        tiles = -(-2 * I // 128) if p["kernel"] == "tcgen05-swap" else -(-M // 128) * -(-2 * I // p["bn"])
    fused = p["full_tiles"] == tiles
    if p["kernel"] != "gemv":
        assert fused == (I in (18944,)), p  # the shapes above cover both routes
    y = gemm(wt, x)  # same plan: the same FP16 gate and up values
    xd = dev_u16(x)
    act = torch.empty((M, I), dtype=torch.int16, device="cuda")
    capi.gemm_swiglu(wt, xd.data_ptr(), K, act.data_ptr(), I, M, stream())
    capi.sync(stream())
    got = host_u16(act)
    g, u = y[:, 0::2], y[:, 1::2]
    lut = _silu_table_f16()
    prod = W.f16_bits_to_f32(lut[g]).astype(np.float32) * W.f16_bits_to_f32(u).astype(np.float32)
    want = W.to_f16_bits(prod)
    same = got == want
    if not same.all():
        # Only a SiLU input whose exp differs from the host's expf in the last
        # bit may move one FP16 ulp.
        diff = np.abs(got.astype(np.int32) - want.astype(np.int32))
        assert same.mean() > 0.9999 and diff.max() <= 1, (MIK, same.mean(), diff.max())
    # And the product itself is the oracle's within tolerance (rows sampled).
    rows = np.unique(np.r_[0, M // 2, M - 1])
    _, _, s2 = _check_against_oracle(x, w, BF16, y, rows, what=f"swiglu product {MIK}")
    assert s2 > 0.9


# ------------------------------------------------------------------ residual epilogue

# (M, N, K, bias): swap mode with whole tiles, K-split global and cluster
# finishes, normal mode with whole tiles, a K-split tail and segmented
# accumulation (K > 4096), and the general kernel (K not a multiple of 8).
RESIDUAL_SHAPES = [(1, 896, 896, False), (1, 3584, 18944, False), (16, 3584, 3584, True), (40, 896, 4864, False),
                   (200, 896, 896, True), (300, 3584, 18944, False), (65, 20000, 2048, False), (3, 200, 68, False)]


@pytest.mark.parametrize("MNKB", RESIDUAL_SHAPES)
@pytest.mark.parametrize("inplace", [False, True])
def test_gemm_residual(cuda_dev, MNKB, inplace):
    """mrt_gemm_residual equals mrt_gemm followed by the reference's add
    (CpuBackend::add, cpu_backend.cpp:430-455, as qwen_model.cpp:316/324 use
    it) applied to that product, bit for bit; in place and with strided
    residual / output rows."""
    M, N, K, bias = MNKB
    rng = np.random.default_rng(M * 3 + N + K)
    x = rand_f16(rng, (M, K))
    w = rand_w(rng, (N, K), BF16)
    res = rand_f16(rng, (M, N))
    wt = upload(w, BF16)
    if bias:
        b = W.to_bf16_bits(rng.standard_normal(N, dtype=np.float32) * np.float32(0.02))
        bd = dev_u16(b)
        wt.attach_bias(bd.data_ptr(), BF16, True, stream())
    y = gemm(wt, x, bias)
    want = O.add(res, y)
    xd = dev_u16(x)
    ld = N + (0 if inplace else 8)  # strided rows when not in place
    resd = torch.zeros((M, ld), dtype=torch.int16, device="cuda")
    resd[:, :N] = dev_u16(res)
    out = resd if inplace else torch.zeros((M, ld), dtype=torch.int16, device="cuda")
    capi.gemm_residual(wt, xd.data_ptr(), K, resd.data_ptr(), ld, out.data_ptr(), ld, M, bias, stream())
    capi.sync(stream())
    got = host_u16(out)[:, :N]
    np.testing.assert_array_equal(got, want)


def test_gemm_residual_rejects_bad_arguments(cuda_dev):
    rng = np.random.default_rng(2)
    wt = upload(rand_w(rng, (64, 64), FP16), FP16)
    x = dev_u16(rand_f16(rng, (2, 64)))
    y = torch.zeros((2, 64), dtype=torch.int16, device="cuda")
    with pytest.raises(capi.MrtError):
        capi.gemm_residual(wt, x.data_ptr(), 64, 0, 64, y.data_ptr(), 64, 2, False, stream())
    with pytest.raises(capi.MrtError):
        capi.gemm_residual(wt, x.data_ptr(), 64, y.data_ptr(), 32, y.data_ptr(), 64, 2, False, stream())


# ------------------------------------------------------------------ lm_head with the pick in the epilogue

# (M, V, K, index_base): the tied 0.5B head, ragged vocabularies (partial last
# tile), a vocabulary shard of the 7B head, 17..64-token tiles.
LM_SHAPES = [(1, 151936, 896, 0), (7, 5000, 896, 0), (16, 152064 // 8, 3584, 3 * (152064 // 8)),
             (33, 1000, 896, 0), (64, 20000, 896, 7)]


@pytest.mark.parametrize("MVKB", LM_SHAPES)
@pytest.mark.parametrize("with_logits", [True, False])
def test_lm_head_fused_pick(cuda_dev, MVKB, with_logits):
    """For M <= 64 mrt_lm_head_argmax picks in the GEMM's epilogue; the
    picks (and values) must equal the reference's greedy rule
    (inference_engine.cpp:84-95) over the logits mrt_gemm produces, and the
    logits, when requested, those same logits."""
    M, V, K, base = MVKB
    rng = np.random.default_rng(M + V + K)
    x = rand_f16(rng, (M, K))
    w = rand_w(rng, (V, K), FP16)
    wt = upload(w, FP16)
    logits = gemm(wt, x)
    want = np.array([O.argmax(r) for r in logits]) + base
    xd = dev_u16(x)
    lg = torch.zeros((M, V), dtype=torch.int16, device="cuda") if with_logits else None
    idx = torch.full((M,), -1, dtype=torch.int64, device="cuda")
    val = torch.zeros((M,), dtype=torch.float32, device="cuda")
    capi.lm_head_argmax(wt, xd.data_ptr(), K, M, lg.data_ptr() if lg is not None else None, base, idx.data_ptr(),
                        val.data_ptr(), stream())
    capi.sync(stream())
    np.testing.assert_array_equal(idx.cpu().numpy(), want)
    vals = W.f16_bits_to_f32(logits[np.arange(M), want - base])
    np.testing.assert_array_equal(val.cpu().numpy(), vals)
    if with_logits:
        np.testing.assert_array_equal(host_u16(lg), logits)


def test_lm_head_fused_pick_edge_cases(cuda_dev):
    """The reference's rule on crafted logit rows (ties, NaN, +-inf, signed
    zeros; tests/golden/bias_argmax.npz, picks from the reference build): a
    one-hot x selects column 0 of a weight holding the row, so the GEMM's
    logits are the crafted values exactly."""
    g = golden("bias_argmax.npz")
    K = 64
    x = np.zeros((1, K), np.uint16)
    x[0, 0] = 0x3C00  # 1.0
    xd = dev_u16(x)
    for row, want in zip(g["rows"], g["am_rows"]):
        V = row.size
        w = np.zeros((V, K), np.uint16)
        w[:, 0] = row
        wt = upload(w, FP16)
        idx = torch.full((1,), -1, dtype=torch.int64, device="cuda")
        capi.lm_head_argmax(wt, xd.data_ptr(), K, 1, None, 0, idx.data_ptr(), None, stream())
        capi.sync(stream())
        assert int(idx.item()) == int(want), (row, want)
        wt.free()


# ------------------------------------------------------------------ segmented accumulation (long K)

@pytest.mark.parametrize("MNK", [(256, 1000, 8192), (130, 3584, 18944), (700, 200, 8200), (2048, 512, 18944)])
def test_long_k_accumulates_in_segments(cuda_dev, MNK):
    """Normal-mode GEMMs whose units run over more than 64 k-blocks take the
    segmented-accumulation kernel; their error against FP64 must stay within
    the reference's own (the tensor cores' round-toward-zero accumulation over
    ~300 k-blocks alone is ~0.9 % worse)."""
    M, N, K = MNK
    rng = np.random.default_rng(M + N + K)
    x = rand_f16(rng, (M, K))
    w = rand_w(rng, (N, K), BF16)
    wt = upload(w, BF16)
    y = gemm(wt, x)
    rows = np.unique(np.r_[0:16, M // 2, M - 16:M])
    _, _, same = _check_against_oracle(x, w, BF16, y, rows, what=f"segmented M={M} N={N} K={K}")
    assert same > 0.9


def test_host_async_matches_host_call(cuda_dev):
    """mrt_gemm_host_async: several products queued on pinned buffers (the two
    staging sets in turn, different weights and sizes), one wait; each equals
    the synchronous mrt_gemm_host call bit for bit (same row chunks).
    Pageable buffers are refused."""
    rng = np.random.default_rng(31)
    cases = [(2048, 3584, 896), (300, 4608, 3584), (64, 896, 896), (1024, 3584, 3584)]
    ws, xs, ys, want = [], [], [], []
    for M, N, K in cases:
        w = rand_w(rng, (N, K), BF16)
        wt = upload(w, BF16)
        x = torch.from_numpy(rand_f16(rng, (M, K)).view(np.int16)).pin_memory()
        y_sync = torch.empty((M, N), dtype=torch.int16).pin_memory()
        capi.gemm_host(wt, x.data_ptr(), y_sync.data_ptr(), M, False, stream())
        ws.append(wt)
        xs.append(x)
        ys.append(torch.zeros((M, N), dtype=torch.int16).pin_memory())
        want.append(y_sync.numpy().copy())
    for _ in range(2):
        for wt, x, y, (M, N, K) in zip(ws, xs, ys, cases):
            capi.gemm_host_async(wt, x.data_ptr(), y.data_ptr(), M, False, stream())
        capi.sync(stream())
        for y, w_ in zip(ys, want):
            np.testing.assert_array_equal(y.numpy(), w_)
    pageable = np.zeros((64, 896), np.uint16)
    out = np.zeros((64, 896), np.uint16)
    with pytest.raises(capi.MrtError):
        capi.gemm_host_async(ws[2], pageable.ctypes.data, out.ctypes.data, 64, False, stream())
