"""Pins the oracle (oracle/mrt_oracle.c) to the reference.

Two independent anchors: the golden vectors in tests/golden/ (generated from
the reference's own CpuBackend compiled from source, by
tests/golden/gen_golden.py) and, where this host has the reference build in
oracle/_ref/, a live bit-for-bit comparison.  CPU only.
"""
import numpy as np
import pytest

from conftest import golden
from mruntime_b200 import workloads as W
from oracle import oracle as O

FP16, BF16, FP32 = O.FP16, O.BF16, O.FP32


def test_known_answer_backend_test():
    # reference test/backend_test.cpp:11-29: C[0,0] = 38, C[0,1] = 44 (+-0.05)
    g = golden("kat_backend_test.npz")
    c = O.gemm(g["a"], FP16, g["b"], FP16)
    np.testing.assert_array_equal(c, g["c"])
    f = O.f16_to_f32(c)
    assert abs(f[0, 0] - 38.0) < 0.05 and abs(f[0, 1] - 44.0) < 0.05


def test_converters_match_golden():
    g = golden("convert.npz")
    f32 = g["f32_bits"].view(np.float32)
    np.testing.assert_array_equal(O.f32_to_f16(f32), g["f16_of_f32"])
    np.testing.assert_array_equal(O.f16_to_f32(np.arange(65536, dtype=np.uint32).astype(np.uint16)).view(np.uint32),
                                  g["f32_of_f16"])
    np.testing.assert_array_equal(O.f32_to_bf16(f32), g["bf16_of_f32"])


def test_workload_rounding_matches_reference_converters():
    # the input generator's numpy roundings must be the reference's converters
    rng = np.random.default_rng(7)
    x = rng.standard_normal(200000, dtype=np.float32) * np.float32(30.0)
    x[:4] = [65519.0, 65520.0, 1e-8, -3e-6]
    np.testing.assert_array_equal(W.to_f16_bits(x), O.f32_to_f16(x))
    np.testing.assert_array_equal(W.to_bf16_bits(x), O.f32_to_bf16(x))
    b = W.to_bf16_bits(x)
    np.testing.assert_array_equal(W.bf16_to_f16_bits(b), O.bf16_to_f16(b))


def test_gemm_small_matches_golden():
    g = golden("gemm_small.npz")
    for i in range(int(g["n_cases"])):
        M, N, K, adt, bdt, cdt, ta, tb = (int(v) for v in g[f"c{i}_spec"])
        alpha, beta = (float(v) for v in g[f"c{i}_ab"])
        c = O.gemm(g[f"c{i}_A"], adt, g[f"c{i}_B"], bdt, cdt, alpha=alpha, beta=beta, trans_a=bool(ta),
                   trans_b=bool(tb), C0=g[f"c{i}_C0"])
        np.testing.assert_array_equal(c, g[f"c{i}_C"], err_msg=f"case {i}")


def test_bias_and_argmax_match_golden():
    g = golden("bias_argmax.npz")
    np.testing.assert_array_equal(O.add_bias(g["acc"], g["bias"]), g["biased"])
    assert [O.argmax(r) for r in g["rows"]] == list(g["am_rows"])
    assert [O.argmax(r) for r in g["rand"]] == list(g["am_rand"])


def test_decode_gemv_matches_golden():
    g = golden("decode_gemv.npz")
    d = W.decode_gemv()
    y = O.gemm(d["x"], FP16, d["w"], FP16, trans_b=True)
    np.testing.assert_array_equal(y, g["y_ref"])
    err = O.rel_frobenius(y, g["y_f64"])
    assert err == pytest.approx(float(g["ref_err"]), rel=1e-9)
    assert err <= 1e-3


def test_empty_gemm_is_a_no_op():
    # cpu_backend.cpp:124-126: M == 0 or N == 0 returns without touching C
    c = O.gemm(np.zeros((0, 8), np.uint16), FP16, np.zeros((4, 8), np.uint16), FP16, trans_b=True)
    assert c.shape == (0, 4)


def test_shape_mismatch_rejected():
    with pytest.raises(ValueError):
        O.gemm(np.zeros((2, 3), np.uint16), FP16, np.zeros((4, 5), np.uint16), FP16, trans_b=True)


@pytest.mark.skipif(not O.ref_available(), reason="reference build oracle/_ref absent")
class TestLiveReference:
    def test_converters_exhaustive_f16(self):
        h = np.arange(65536, dtype=np.uint32).astype(np.uint16)
        np.testing.assert_array_equal(O.f16_to_f32(h).view(np.uint32), O.ref_f16_to_f32(h).view(np.uint32))

    def test_converters_random_f32(self):
        rng = np.random.default_rng(11)
        bits = rng.integers(0, 2**32, size=1 << 20, dtype=np.uint64).astype(np.uint32)
        f = bits.view(np.float32)
        np.testing.assert_array_equal(O.f32_to_f16(f), O.ref_f32_to_f16(f))
        np.testing.assert_array_equal(O.f32_to_bf16(f), O.ref_f32_to_bf16(f))

    @pytest.mark.parametrize("shape", [(1, 4864, 896), (3, 129, 72), (17, 31, 40)])
    @pytest.mark.parametrize("wdt", [FP16, BF16])
    def test_gemm_bitexact(self, shape, wdt):
        M, N, K = shape
        rng = np.random.default_rng(M * 1000 + N)
        x = W.to_f16_bits(rng.standard_normal((M, K), dtype=np.float32))
        wv = rng.standard_normal((N, K), dtype=np.float32) * np.float32(0.02)
        w = W.to_f16_bits(wv) if wdt == FP16 else W.to_bf16_bits(wv)
        rb = O.RefBackend(4)
        np.testing.assert_array_equal(O.gemm(x, FP16, w, wdt, trans_b=True), rb.gemm(x, FP16, w, wdt, trans_b=True))
        rb.close()

    def test_bias_and_argmax(self):
        rng = np.random.default_rng(3)
        acc = W.to_f16_bits(rng.standard_normal((16, 300), dtype=np.float32) * 8)
        bias = W.to_f16_bits(rng.standard_normal(300, dtype=np.float32))
        np.testing.assert_array_equal(O.add_bias(acc, bias), O.ref_add_bias(acc, bias))
        for row in acc:
            assert O.argmax(row) == O.ref_argmax(row)

    def test_add_matches_cpu_backend_add(self):
        """orc_add_f16 against CpuBackend::add (cpu_backend.cpp:430-455): random
        values of every magnitude, overflow to inf, inf + -inf, NaN, signed
        zeros and subnormals."""
        rng = np.random.default_rng(21)
        a = rng.integers(0, 65536, size=1 << 18, dtype=np.uint32).astype(np.uint16)
        b = rng.integers(0, 65536, size=1 << 18, dtype=np.uint32).astype(np.uint16)
        edge = np.array([0x0000, 0x8000, 0x7BFF, 0xFBFF, 0x7C00, 0xFC00, 0x7E00, 0x0001, 0x8001, 0x3C00], np.uint16)
        a = np.r_[a, np.repeat(edge, edge.size)]
        b = np.r_[b, np.tile(edge, edge.size)]
        np.testing.assert_array_equal(O.add(a, b), O.ref_add(a, b))
