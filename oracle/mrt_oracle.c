/*
 * mrt_oracle.c -- CPU restatement of mruntime's linear-layer arithmetic.
 *
 * TEST INFRASTRUCTURE ONLY (the checker, never the thing measured or shipped).
 * Parity of this file with the reference is pinned two ways:
 *   1. tests/test_oracle.py compares it bit-for-bit with the reference's own
 *      CpuBackend::gemm and dtype converters, compiled from the reference
 *      sources into oracle/_ref/libmrt_ref.so by oracle/Makefile;
 *   2. the same test checks it against the golden vectors in tests/golden/,
 *      which tests/golden/gen_golden.py produced from that reference build,
 *      and against the reference's known-answer test (test/backend_test.cpp:11-29).
 *
 * Build with -ffp-contract=off: the reference's scalar loop
 * (cpu_backend.cpp:152-156) is a separate multiply and add in FP32, and a
 * fused multiply-add would change the rounding.
 */
#include "mrt_oracle.h"

#include <math.h>
#include <string.h>

static inline uint32_t f32_bits(float f) { uint32_t u; memcpy(&u, &f, 4); return u; }
static inline float bits_f32(uint32_t u) { float f; memcpy(&f, &u, 4); return f; }

/* include/mruntime/dtype.h:39-119.  The reference walks the cases one by one;
 * here the normal and subnormal results share one rounding step: the 24-bit
 * significand is shifted right by the number of bits FP16 cannot hold (13 for
 * normals, 14 - e for subnormals), rounded to nearest-even, and the rounded
 * significand is added onto the exponent field so that a carry out of the
 * mantissa bumps the exponent (and, at the top, lands on infinity). */
uint16_t orc_f32_to_f16(float f) {
    const uint32_t x = f32_bits(f);
    const uint16_t sign = (uint16_t)((x >> 16) & 0x8000u);
    const uint32_t e = (x >> 23) & 0xFFu;
    const uint32_t m = x & 0x7FFFFFu;
    if (e == 0xFFu) {
        if (m == 0) return (uint16_t)(sign | 0x7C00u);
        uint32_t payload = m >> 13;
        if ((payload & 0x3FFu) == 0) payload = 1;
        return (uint16_t)(sign | 0x7C00u | payload);
    }
    if (e == 0) return sign; /* zero and FP32 denormals -> signed zero */
    const int32_t he = (int32_t)e - 112; /* FP16 biased exponent */
    if (he >= 31) return (uint16_t)(sign | 0x7C00u);
    if (he < -10) return sign;
    const uint32_t sig = m | 0x800000u;
    const int shift = he > 0 ? 13 : 14 - he;
    uint32_t q = sig >> shift;
    const uint32_t rem = sig & ((1u << shift) - 1u);
    const uint32_t half = 1u << (shift - 1);
    if (rem > half || (rem == half && (q & 1u))) ++q;
    if (he > 0) return (uint16_t)(sign | (((uint32_t)(he - 1) << 10) + q));
    return (uint16_t)(sign | q); /* q == 0x400 is the smallest normal */
}

/* include/mruntime/dtype.h:121-148: exact widening; NaN -> +quiet NaN. */
float orc_f16_to_f32(uint16_t h) {
    const uint32_t sign = ((uint32_t)h & 0x8000u) << 16;
    const uint32_t e = (h >> 10) & 0x1Fu;
    uint32_t m = h & 0x3FFu;
    if (e == 0x1Fu) {
        if (m != 0) return bits_f32(0x7FC00000u);
        return bits_f32(sign | 0x7F800000u);
    }
    if (e == 0) {
        if (m == 0) return bits_f32(sign);
        int lead = 0; /* normalise the subnormal significand */
        while ((m & 0x400u) == 0) { m <<= 1; ++lead; }
        return bits_f32(sign | ((uint32_t)(113 - lead) << 23) | ((m & 0x3FFu) << 13));
    }
    return bits_f32(sign | ((e + 112u) << 23) | (m << 13));
}

/* include/mruntime/dtype.h:153-160 (same rounding trick, including its
 * behaviour on NaN inputs, which the reference does not special-case). */
uint16_t orc_f32_to_bf16(float f) {
    uint32_t x = f32_bits(f);
    x += 0x7FFFu + ((x >> 16) & 1u);
    return (uint16_t)(x >> 16);
}

/* include/mruntime/dtype.h:162-167. */
float orc_bf16_to_f32(uint16_t b) { return bits_f32((uint32_t)b << 16); }

void orc_f32_to_f16_n(const float* src, uint16_t* dst, size_t n) {
    for (size_t i = 0; i < n; ++i) dst[i] = orc_f32_to_f16(src[i]);
}
void orc_f16_to_f32_n(const uint16_t* src, float* dst, size_t n) {
    for (size_t i = 0; i < n; ++i) dst[i] = orc_f16_to_f32(src[i]);
}
void orc_f32_to_bf16_n(const float* src, uint16_t* dst, size_t n) {
    for (size_t i = 0; i < n; ++i) dst[i] = orc_f32_to_bf16(src[i]);
}
/* BF16 -> FP16 as the reference's packing step does it: widen exactly, then
 * round with the FP16 converter (src/core/cpu_backend.cpp:48-55). */
void orc_bf16_to_f16_n(const uint16_t* src, uint16_t* dst, size_t n) {
    for (size_t i = 0; i < n; ++i) dst[i] = orc_f32_to_f16(orc_bf16_to_f32(src[i]));
}

/* load_scalar_as_fp32 / store_scalar_from_fp32 (include/mruntime/dtype.h:169-194). */
static inline float load_as_f32(const void* p, int dt, size_t i) {
    switch (dt) {
        case ORC_FP32: return ((const float*)p)[i];
        case ORC_BF16: return orc_bf16_to_f32(((const uint16_t*)p)[i]);
        default: return orc_f16_to_f32(((const uint16_t*)p)[i]);
    }
}
static inline void store_from_f32(void* p, int dt, size_t i, float v) {
    switch (dt) {
        case ORC_FP32: ((float*)p)[i] = v; return;
        case ORC_BF16: ((uint16_t*)p)[i] = orc_f32_to_bf16(v); return;
        default: ((uint16_t*)p)[i] = orc_f32_to_f16(v); return;
    }
}

/* src/core/cpu_backend.cpp:72-169 on its portable path (the KleidiAI branch
 * at 104-122 only exists on Arm64 with FP16 vector arithmetic). */
int orc_gemm(const void* A, int a_dtype, size_t a_rows0, size_t a_cols0,
             const void* B, int b_dtype, size_t b_rows0, size_t b_cols0,
             void* C, int c_dtype, size_t c_rows, size_t c_cols,
             float alpha, float beta, int trans_a, int trans_b,
             size_t m0, size_t m1) {
    const size_t M = trans_a ? a_cols0 : a_rows0;
    const size_t K = trans_a ? a_rows0 : a_cols0;
    const size_t N = trans_b ? b_rows0 : b_cols0;
    if ((trans_b ? b_cols0 : b_rows0) != K) return -1;
    if (c_rows != M || c_cols != N) return -1;
    if (m1 > M) m1 = M;
    for (size_t m = m0; m < m1; ++m) {
        for (size_t n = 0; n < N; ++n) {
            float acc = 0.0f;
            if (alpha != 0.0f) {
                for (size_t k = 0; k < K; ++k) {
                    const size_t ai = trans_a ? (k * a_cols0 + m) : (m * a_cols0 + k);
                    const size_t bi = trans_b ? (n * b_cols0 + k) : (k * b_cols0 + n);
                    const float prod = load_as_f32(A, a_dtype, ai) * load_as_f32(B, b_dtype, bi);
                    acc += prod;
                }
                acc *= alpha;
            }
            float out = acc;
            if (beta != 0.0f) out += beta * load_as_f32(C, c_dtype, m * N + n);
            store_from_f32(C, c_dtype, m * N + n, out);
        }
    }
    return 0;
}

void orc_gemm_f64(const uint16_t* X, size_t M, size_t K,
                  const void* W, int w_dtype, size_t N, double* Y) {
    for (size_t m = 0; m < M; ++m) {
        for (size_t n = 0; n < N; ++n) {
            double acc = 0.0;
            for (size_t k = 0; k < K; ++k)
                acc += (double)orc_f16_to_f32(X[m * K + k]) * (double)load_as_f32(W, w_dtype, n * K + k);
            Y[m * N + n] = acc;
        }
    }
}

/* src/models/qwen/qwen_model.cpp:130-155 (the add_bias lambda). */
void orc_add_bias_f16(uint16_t* out, const uint16_t* bias, size_t rows, size_t n) {
    for (size_t r = 0; r < rows; ++r)
        for (size_t i = 0; i < n; ++i) {
            float v = orc_f16_to_f32(out[r * n + i]);
            v += orc_f16_to_f32(bias[i]);
            out[r * n + i] = orc_f32_to_f16(v);
        }
}

/* CpuBackend::add (src/core/cpu_backend.cpp:430-455) on FP16 operands: each
 * element widened exactly, one FP32 add, the reference's FP16 rounding. */
void orc_add_f16(const uint16_t* a, const uint16_t* b, uint16_t* out, size_t n) {
    for (size_t i = 0; i < n; ++i) out[i] = orc_f32_to_f16(orc_f16_to_f32(a[i]) + orc_f16_to_f32(b[i]));
}

/* src/engine/inference_engine.cpp:84-95. */
int64_t orc_argmax_f16(const uint16_t* logits, size_t n) {
    float best = -INFINITY;
    int64_t best_idx = 0;
    for (size_t i = 0; i < n; ++i) {
        const float v = orc_f16_to_f32(logits[i]);
        if (v > best) { best = v; best_idx = (int64_t)i; }
    }
    return best_idx;
}

double orc_rel_frobenius_f16(const uint16_t* got, const double* want, size_t n) {
    double num = 0.0, den = 0.0;
    for (size_t i = 0; i < n; ++i) {
        const double d = (double)orc_f16_to_f32(got[i]) - want[i];
        num += d * d;
        den += want[i] * want[i];
    }
    return den > 0.0 ? sqrt(num / den) : sqrt(num);
}
