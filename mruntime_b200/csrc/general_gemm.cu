// general_gemm.cu -- the whole Backend::gemm contract on the device.
//
// The model only ever calls gemm(x, W, y, 1, 0, false, true) with FP16 x/y
// and FP16/BF16 W; those calls take the skinny or tcgen05 kernels.  Every
// other call pattern the interface allows (FP32 operands, trans_a, B given as
// [K, N], alpha != 1, beta != 0, K not a multiple of 8, unaligned rows) lands
// here.  One thread owns one output and sums its k terms in order with
// separately rounded multiply and add (__fmul_rn/__fadd_rn, so the compiler
// cannot fuse them), then applies alpha, beta*C and the reference's store
// rounding -- the arithmetic of src/core/cpu_backend.cpp:149-165, so results
// match the reference bit for bit.  Operand tiles are staged through shared
// memory to keep global loads coalesced.
#include "common.cuh"
#include "kernels.h"

namespace mrt {
namespace {

constexpr int kT = 16;  // 16x16 outputs per block, 16-wide k tiles

__device__ __forceinline__ float ld_f32(const void* p, int dt, int64_t i) {
    if (dt == 2) return static_cast<const float*>(p)[i];
    const uint16_t v = static_cast<const uint16_t*>(p)[i];
    return dt == 1 ? bf16_bits_to_f32(v) : f16_bits_to_f32(v);
}

__global__ void general_gemm_kernel(const GeneralGemmArgs a) {
    __shared__ float sa[kT][kT + 1];  // sa[m][k]
    __shared__ float sb[kT][kT + 1];  // sb[k][n]
    const int tx = threadIdx.x;        // n within tile
    const int ty = threadIdx.y;        // m within tile
    const int64_t m = static_cast<int64_t>(blockIdx.y) * kT + ty;
    const int64_t n = static_cast<int64_t>(blockIdx.x) * kT + tx;
    float acc = 0.0f;
    if (a.alpha != 0.0f) {
        for (int64_t k0 = 0; k0 < a.K; k0 += kT) {
            // A element (mm, kk): trans_a ? A[kk, mm] : A[mm, kk]
            {
                const int64_t mm = static_cast<int64_t>(blockIdx.y) * kT + ty;
                const int64_t kk = k0 + tx;
                float v = 0.0f;
                if (mm < a.M && kk < a.K) {
                    const int64_t idx = a.trans_a ? kk * a.a_cols0 + mm : mm * a.a_cols0 + kk;
                    v = ld_f32(a.a, a.a_dtype, idx);
                }
                sa[ty][tx] = v;
            }
            // B element (kk, nn): trans_b ? B[nn, kk] : B[kk, nn]
            {
                const int64_t kk = k0 + ty;
                const int64_t nn = static_cast<int64_t>(blockIdx.x) * kT + tx;
                float v = 0.0f;
                if (nn < a.N && kk < a.K) {
                    const int64_t idx = a.b_k_tiles > 0 ? tiled_offset(nn, kk, a.b_k_tiles)
                                                        : (a.trans_b ? nn * a.b_cols0 + kk : kk * a.b_cols0 + nn);
                    v = ld_f32(a.b, a.b_dtype, idx);
                }
                sb[ty][tx] = v;
            }
            __syncthreads();
            const int kend = static_cast<int>(a.K - k0 < kT ? a.K - k0 : kT);
            for (int kk = 0; kk < kend; ++kk) acc = __fadd_rn(acc, __fmul_rn(sa[ty][kk], sb[kk][tx]));
            __syncthreads();
        }
        acc = __fmul_rn(acc, a.alpha);
    }
    if (m >= a.M || n >= a.N) return;
    float out = acc;
    const int64_t ci = m * a.ldc + n;
    if (a.beta != 0.0f) out = __fadd_rn(out, __fmul_rn(a.beta, ld_f32(a.c, a.c_dtype, ci)));
    if (a.c_dtype == 2) {
        static_cast<float*>(a.c)[ci] = out;
    } else if (a.c_dtype == 1) {
        static_cast<uint16_t*>(a.c)[ci] = f32_to_bf16_bits(out);
    } else {
        static_cast<uint16_t*>(a.c)[ci] = add_residual(round_out(out, a.bias, n), a.residual, m * a.ldr + n);
    }
}

}  // namespace

cudaError_t launch_general_gemm(const GeneralGemmArgs& a, cudaStream_t s) {
    if (a.M <= 0 || a.N <= 0) return cudaSuccess;
    dim3 block(kT, kT);
    dim3 grid(static_cast<unsigned>((a.N + kT - 1) / kT), static_cast<unsigned>((a.M + kT - 1) / kT));
    if (grid.y > 65535u) return cudaErrorInvalidValue;
    general_gemm_kernel<<<grid, block, 0, s>>>(a);
    note_launches(1);
    return cudaGetLastError();
}

}  // namespace mrt
