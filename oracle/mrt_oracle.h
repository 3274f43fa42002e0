/*
 * mrt_oracle.h -- CPU restatement of mruntime's linear-layer arithmetic.
 *
 * TEST INFRASTRUCTURE ONLY.  This library is the checker for the CUDA path:
 * only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline leg may
 * load it.  The product library (mruntime_b200) never links or calls it.
 *
 * Every function restates one piece of the reference (kabu1204/mruntime) and
 * cites the file:line it follows.  It is pinned bit-for-bit against the
 * reference's own code compiled from source (oracle/_ref, see Makefile) and
 * against the committed golden vectors in tests/golden/.
 */
#ifndef MRT_ORACLE_H
#define MRT_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Same numbering as mruntime::DType (include/mruntime/dtype.h:12-16). */
enum { ORC_FP16 = 0, ORC_BF16 = 1, ORC_FP32 = 2 };

/* FP32 -> FP16 bits, round-to-nearest-even, FP32 denormals flushed to signed
 * zero, NaN payload = top 10 mantissa bits forced non-zero
 * (include/mruntime/dtype.h:39-119). */
uint16_t orc_f32_to_f16(float f);
/* FP16 bits -> FP32, exact; every NaN becomes the positive quiet NaN
 * (include/mruntime/dtype.h:121-148). */
float orc_f16_to_f32(uint16_t h);
/* FP32 -> BF16 bits by the add-0x7FFF-plus-lsb rounding trick, no NaN special
 * case (include/mruntime/dtype.h:153-160). */
uint16_t orc_f32_to_bf16(float f);
/* BF16 bits -> FP32, exact (include/mruntime/dtype.h:162-167). */
float orc_bf16_to_f32(uint16_t b);

/* Vector forms of the converters above. */
void orc_f32_to_f16_n(const float* src, uint16_t* dst, size_t n);
void orc_f16_to_f32_n(const uint16_t* src, float* dst, size_t n);
void orc_f32_to_bf16_n(const float* src, uint16_t* dst, size_t n);
void orc_bf16_to_f16_n(const uint16_t* src, uint16_t* dst, size_t n);

/*
 * Portable CpuBackend::gemm (src/core/cpu_backend.cpp:72-169, scalar path
 * 124-168).  A is [a_rows0, a_cols0] (3-D A flattened to rows, line 87), B is
 * [b_rows0, b_cols0]; C is [M, N] row-major.  Only output rows [m0, m1) are
 * computed, which is exact because every output row depends only on its own
 * row of A (cpu_backend.cpp:143-166).  Returns 0, or -1 on a shape mismatch
 * (the reference asserts at cpu_backend.cpp:95-98).
 */
int orc_gemm(const void* A, int a_dtype, size_t a_rows0, size_t a_cols0,
             const void* B, int b_dtype, size_t b_rows0, size_t b_cols0,
             void* C, int c_dtype, size_t c_rows, size_t c_cols,
             float alpha, float beta, int trans_a, int trans_b,
             size_t m0, size_t m1);

/* FP64 ground truth of Y = X * W^T for FP16 X [M,K] and W [N,K] given in any
 * of the three dtypes; output FP64 [M,N].  Not a reference function: it is
 * the exact-arithmetic yardstick the tolerance is measured against. */
void orc_gemm_f64(const uint16_t* X, size_t M, size_t K,
                  const void* W, int w_dtype, size_t N, double* Y);

/* Bias add after the q/k/v projections: out = fp16(fp32(out) + fp32(bias)),
 * applied in place to every row (src/models/qwen/qwen_model.cpp:130-155). */
void orc_add_bias_f16(uint16_t* out, const uint16_t* bias, size_t rows, size_t n);
void orc_add_f16(const uint16_t* a, const uint16_t* b, uint16_t* out, size_t n);

/* Greedy argmax over one row of FP16 logits: first index whose value is
 * strictly greater than every earlier one, starting from -inf, so NaN never
 * wins and an all -inf/NaN row yields 0 (src/engine/inference_engine.cpp:84-95). */
int64_t orc_argmax_f16(const uint16_t* logits, size_t n);

/* Relative Frobenius error ||got - want||_F / ||want||_F with got in FP16. */
double orc_rel_frobenius_f16(const uint16_t* got, const double* want, size_t n);

#ifdef __cplusplus
}
#endif
#endif
