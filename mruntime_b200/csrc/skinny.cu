// skinny.cu -- decode-shape GEMM, Y[M,N] = X[M,K] * W[N,K]^T for M <= 64.
//
// Decode is bound by streaming W once from HBM (2*N*K bytes; x and y are tiny).
// Each CTA owns 8*RN consecutive weight rows; its 8 warps split K and every
// warp streams its share of those rows with 16-byte non-allocating loads.
// The products run on mma.sync m16n8k16 (FP16 in, FP32 accumulate) so M up to
// 64 costs no more issue slots than M = 1 -- the FP32 CUDA-core FMA rate
// would cap M = 16 below the HBM roofline.
//
// Operand trick: the sum over k does not care in which order the 16 k values
// of one MMA are visited, as long as A and B use the same order.  Thread
// (g = lane/4, t = lane%4) loads 8 consecutive halves W[n0+g][kb+8t .. +7]
// with one 16-byte load and x rows g and g+8 the same way; halves 0-3 feed the
// k-slots {2t,2t+1,2t+8,2t+9} of a first MMA and halves 4-7 those of a second
// MMA.  That covers k = kb .. kb+31 exactly once with fully vectorised loads
// and no shared-memory staging.
//
// Partial sums of the 8 warps are added in a fixed order through shared
// memory, then rounded with the reference's converter (and the q/k/v bias
// double rounding when a bias is given).
#include "common.cuh"
#include "kernels.h"

namespace mrt {
namespace {

constexpr int kWarps = 8;

__device__ __forceinline__ void mma_16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                          uint32_t a3, uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 "
        "{%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, {%0, %1, %2, %3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// MT: 16-row tiles of x (M <= 16*MT).  RN: 8-row tiles of W per CTA.
// U: 32-wide k steps each warp loads before it multiplies.
template <int MT, int RN, int U>
__global__ void __launch_bounds__(kWarps * 32) skinny_kernel(const SkinnyArgs a) {
    __shared__ float red[kWarps][MT * 16][RN * 8];

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int g = lane >> 2;
    const int t = lane & 3;
    const int64_t K = a.K;
    const int64_t n_base = static_cast<int64_t>(blockIdx.x) * (8 * RN);

    const uint16_t* wrow[RN];
    bool wok[RN];
#pragma unroll
    for (int r = 0; r < RN; ++r) {
        const int64_t n = n_base + r * 8 + g;
        wok[r] = n < a.N;
        wrow[r] = a.w + (wok[r] ? n : 0) * K;
    }
    const uint16_t* xrow[MT][2];
    bool xok[MT][2];
#pragma unroll
    for (int mt = 0; mt < MT; ++mt)
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            const int m = mt * 16 + g + 8 * h;
            xok[mt][h] = m < a.M;
            xrow[mt][h] = a.x + (xok[mt][h] ? m : 0) * a.ldx;
        }

    float acc[MT][RN][4];
#pragma unroll
    for (int mt = 0; mt < MT; ++mt)
#pragma unroll
        for (int r = 0; r < RN; ++r)
#pragma unroll
            for (int i = 0; i < 4; ++i) acc[mt][r][i] = 0.0f;

    const int ksteps = static_cast<int>((K + 31) / 32);
    const uint4 zero = make_uint4(0u, 0u, 0u, 0u);
    for (int s0 = warp * U; s0 < ksteps; s0 += kWarps * U) {
        uint4 wv[U][RN];
        uint4 xv[U][MT][2];
#pragma unroll
        for (int u = 0; u < U; ++u) {
            const int64_t k = static_cast<int64_t>(s0 + u) * 32 + t * 8;
            const bool kin = (s0 + u) < ksteps && k < K;
#pragma unroll
            for (int r = 0; r < RN; ++r) wv[u][r] = (kin && wok[r]) ? ld_stream_16B(wrow[r] + k) : zero;
#pragma unroll
            for (int mt = 0; mt < MT; ++mt)
#pragma unroll
                for (int h = 0; h < 2; ++h)
                    xv[u][mt][h] = (kin && xok[mt][h])
                                       ? __ldg(reinterpret_cast<const uint4*>(xrow[mt][h] + k))
                                       : zero;
        }
#pragma unroll
        for (int u = 0; u < U; ++u)
#pragma unroll
            for (int r = 0; r < RN; ++r)
#pragma unroll
                for (int mt = 0; mt < MT; ++mt) {
                    const uint4& x0 = xv[u][mt][0];
                    const uint4& x1 = xv[u][mt][1];
                    const uint4& w = wv[u][r];
                    mma_16816(acc[mt][r], x0.x, x1.x, x0.y, x1.y, w.x, w.y);
                    mma_16816(acc[mt][r], x0.z, x1.z, x0.w, x1.w, w.z, w.w);
                }
    }

    // Accumulator fragment: c0,c1 at (row g, cols 2t, 2t+1), c2,c3 at row g+8.
#pragma unroll
    for (int mt = 0; mt < MT; ++mt)
#pragma unroll
        for (int r = 0; r < RN; ++r) {
            red[warp][mt * 16 + g][r * 8 + 2 * t] = acc[mt][r][0];
            red[warp][mt * 16 + g][r * 8 + 2 * t + 1] = acc[mt][r][1];
            red[warp][mt * 16 + g + 8][r * 8 + 2 * t] = acc[mt][r][2];
            red[warp][mt * 16 + g + 8][r * 8 + 2 * t + 1] = acc[mt][r][3];
        }
    __syncthreads();

    constexpr int kOut = MT * 16 * RN * 8;
    for (int e = threadIdx.x; e < kOut; e += kWarps * 32) {
        const int m = e / (RN * 8);
        const int nl = e % (RN * 8);
        const int64_t n = n_base + nl;
        if (m >= a.M || n >= a.N) continue;
        float s = 0.0f;
#pragma unroll
        for (int w = 0; w < kWarps; ++w) s += red[w][m][nl];
        if (a.out_f32) {
            static_cast<float*>(a.y)[m * a.ldy + n] = s;
        } else {
            static_cast<uint16_t*>(a.y)[m * a.ldy + n] = round_out(s, a.bias, n);
        }
    }
}

template <int MT, int RN, int U>
cudaError_t launch_one(const SkinnyArgs& a, cudaStream_t s) {
    const int64_t blocks = (static_cast<int64_t>(a.N) + 8 * RN - 1) / (8 * RN);
    if (blocks <= 0) return cudaSuccess;
    skinny_kernel<MT, RN, U><<<static_cast<unsigned>(blocks), kWarps * 32, 0, s>>>(a);
    note_launches(1);
    return cudaGetLastError();
}

}  // namespace

// rn: weight rows per CTA in units of 8 (1, 2 or 4).
cudaError_t launch_skinny(const SkinnyArgs& a, int rn, cudaStream_t s) {
    if (a.M <= 0 || a.N <= 0) return cudaSuccess;
    if (a.M > 16) return cudaErrorInvalidValue;  // larger M runs on the tcgen05 kernel
    if (rn >= 4) return launch_one<1, 4, 4>(a, s);
    if (rn == 2) return launch_one<1, 2, 4>(a, s);
    return launch_one<1, 1, 4>(a, s);
}

}  // namespace mrt
