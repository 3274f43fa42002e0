// gemm_tc.cu -- prefill GEMM on the 5th-generation tensor cores (sm_100a).
//
// Y[M,N] = X[M,K] * W[N,K]^T, FP16 operands, FP32 accumulation in tensor
// memory (TMEM), FP16 (or FP32) output.
//
// One persistent CTA per SM walks a static list of work units
// (m-tile, n-tile, k-split); m varies fastest so the CTAs running at the same
// time share weight tiles in L2.  Warp roles:
//   warp 0    TMA producer: one lane streams 128x64 X tiles and BNx64 W tiles
//             (128-byte swizzle) into a STAGES-deep shared-memory ring,
//             completion counted on a "full" mbarrier per stage;
//   warp 1    allocates TMEM (2*BN columns = two accumulators) and one lane
//             issues tcgen05.mma (M=128, N=BN, K=16; four per stage) and
//             tcgen05.commit to release ring stages and to publish a finished
//             accumulator;
//   warps 2-5 epilogue: tcgen05.ld of their 32 TMEM lanes (= tile rows),
//             rounding with the reference's FP16 converter (plus the q/k/v
//             bias double rounding), 16-byte stores; the second accumulator
//             lets the next tile's MMAs overlap this drain.
// Every mbarrier wait is bounded (common.cuh); on a timeout the kernel
// records an error code, waits (bounded) for its own copies and MMAs in flight
// and frees its TMEM before returning.
//
// TMA loads here never use cluster-wide broadcast and every operand is memory
// of this GPU.
#include "common.cuh"
#include "kernels.h"

namespace mrt {
namespace {

constexpr int kBM = 128;
constexpr int kBK = 64;
constexpr int kThreadsTc = 192;
constexpr int kEpiThreads = 128;
// Segmented accumulation (normal mode, units longer than kSegMinKb k-blocks):
// every kSegKb k-blocks the MMAs move to the other TMEM accumulator and 8
// epilogue warps add the finished segment into FP32 registers with IEEE
// round-to-nearest.  The tensor cores' own accumulation rounds toward zero;
// over ~1200 MMAs (K = 18944) that bias makes the result ~0.4-0.9 % less
// accurate than the reference's sequential FP32 loop (cpu_backend.cpp:143-166),
// and segments of kSegKb k-blocks bring it back to the reference's error.
constexpr int kThreadsSeg = 64 + 256;

template <bool SEG>
constexpr int threads_of() { return SEG ? kThreadsSeg : kThreadsTc; }

template <int BN, bool SWAP>
struct TcCfg {
    static constexpr int kABytes = kBM * kBK * 2;
    static constexpr int kBBytes = BN * kBK * 2;
    static constexpr int kStageBytes = kABytes + kBBytes;
    // Normal mode: as many ring stages as fit in ~200 KB (4 for BN = 256, 8
    // for BN = 64).  Swap mode (weight streaming): ~108 KB (6 stages for
    // BN = 16, 4 for BN = 64), so two CTAs fit on an SM -- the next GEMM's CTA
    // streams its weights beside this one's epilogue and K-split fix-up.
    static constexpr int kRingBudget = SWAP ? 108 * 1024 : 200 * 1024;
    static constexpr int kStages = kRingBudget / kStageBytes > 12 ? 12 : kRingBudget / kStageBytes;
    // Two accumulators of BN FP32 columns, rounded up to a power of two >= 32.
    static constexpr uint32_t kTmemCols = 2 * BN <= 32 ? 32 : (2 * BN <= 64 ? 64 : (2 * BN <= 128 ? 128 : (2 * BN <= 256 ? 256 : 512)));
    // full[S], empty[S], tfull[2], tempty[2], drain, cl_ready, cl_done; TMEM slot.
    static constexpr int kBarBytes = (2 * kStages + 7) * 8 + 16;
    static constexpr size_t kSmem = static_cast<size_t>(kStages) * kStageBytes + kBarBytes + 1024;
};

// One work unit: an output tile and the k-blocks it covers.  `slot` is -1
// for a full-K tile (stored directly) or the partials slot of a tail slice.
struct Unit {
    int mt, nt, kb0, kb1, slot, ti;  // ti: index among the tail tiles (-1 for a full-K tile)
};

__device__ __forceinline__ Unit decode_unit(const TcGemmArgs& a, int u, int num_m, int n_tail, int num_kb) {
    Unit w;
    int t;
    if (u < a.full_tiles) {
        t = u;
        w.kb0 = 0;
        w.kb1 = num_kb;
        w.slot = -1;
        w.ti = -1;
    } else if (a.cluster_k > 1) {
        // One slice per CTA; the slices of tail tile ti are CTAs
        // ti * cluster_k .. + cluster_k - 1, one cluster.
        const int ti = u / a.cluster_k;
        const int sp = u % a.cluster_k;
        t = ti;
        w.kb0 = sp * a.kb_per;
        w.kb1 = min(w.kb0 + a.kb_per, num_kb);
        w.slot = sp;
        w.ti = ti;
    } else {
        const int v = u - a.full_tiles;
        const int ti = v % n_tail;
        const int sp = v / n_tail;
        t = a.full_tiles + ti;
        w.kb0 = sp * a.kb_per;
        w.kb1 = min(w.kb0 + a.kb_per, num_kb);
        w.slot = sp * n_tail + ti;
        w.ti = ti;
    }
    w.mt = t % num_m;
    w.nt = t / num_m;
    return w;
}

__device__ __forceinline__ uint32_t pack_h2(uint16_t lo, uint16_t hi) {
    return static_cast<uint32_t>(lo) | (static_cast<uint32_t>(hi) << 16);
}

// Store 32 FP32 accumulator columns of one tile row into a tail slot
// (tile-local layout [tile_rows][bn]; always in bounds and 16-byte aligned).
__device__ __forceinline__ void store_partial_chunk(const TcGemmArgs& a, const uint32_t (&r)[32], int slot,
                                                   int row_in_tile, int col_in_tile, int bn, int tile_rows = kBM) {
    float* dst = a.partials + (static_cast<int64_t>(slot) * tile_rows + row_in_tile) * bn + col_in_tile;
    if ((reinterpret_cast<uintptr_t>(dst) & 31) == 0) {
        // whole 32-byte sectors: a partial-sector write costs the memory
        // system a read-modify-write of the sector
#pragma unroll
        for (int j = 0; j < 32; j += 8)
            st_global_v8(dst + j, r[j], r[j + 1], r[j + 2], r[j + 3], r[j + 4], r[j + 5], r[j + 6], r[j + 7]);
    } else {
#pragma unroll
        for (int j = 0; j < 32; j += 4)
            *reinterpret_cast<uint4*>(dst + j) = make_uint4(r[j], r[j + 1], r[j + 2], r[j + 3]);
    }
}

// Store 32 accumulator columns of one output row.
__device__ __forceinline__ void store_row_chunk(const TcGemmArgs& a, const uint32_t (&r)[32],
                                                int64_t row, int64_t col0) {
    if (a.out_f32) {
        float* dst = static_cast<float*>(a.y) + row * a.ldy + col0;
        const bool vec = col0 + 32 <= a.N && ((reinterpret_cast<uintptr_t>(dst) & 15) == 0);
        if (vec && (reinterpret_cast<uintptr_t>(dst) & 31) == 0) {
#pragma unroll
            for (int j = 0; j < 32; j += 8)
                st_global_v8(dst + j, r[j], r[j + 1], r[j + 2], r[j + 3], r[j + 4], r[j + 5], r[j + 6], r[j + 7]);
        } else if (vec) {
#pragma unroll
            for (int j = 0; j < 32; j += 4)
                *reinterpret_cast<uint4*>(dst + j) = make_uint4(r[j], r[j + 1], r[j + 2], r[j + 3]);
        } else {
#pragma unroll
            for (int j = 0; j < 32; ++j)
                if (col0 + j < a.N) dst[j] = __uint_as_float(r[j]);
        }
        return;
    }
    uint16_t* dst = static_cast<uint16_t*>(a.y) + row * a.ldy + col0;
    const uint16_t* res = a.residual != nullptr ? a.residual + row * a.ldr + col0 : nullptr;
    const bool vec = col0 + 32 <= a.N && ((reinterpret_cast<uintptr_t>(dst) & 15) == 0) &&
                     ((reinterpret_cast<uintptr_t>(res) & 15) == 0);
    if (vec) {
        uint32_t h[16];
#pragma unroll
        for (int j = 0; j < 16; ++j)
            h[j] = pack_h2(round_out(__uint_as_float(r[2 * j]), a.bias, col0 + 2 * j),
                           round_out(__uint_as_float(r[2 * j + 1]), a.bias, col0 + 2 * j + 1));
        if (res != nullptr) {
            // The residual row chunk is read whole before any output is
            // written (y may be the residual buffer itself).
            uint4 q[4];
#pragma unroll
            for (int j = 0; j < 4; ++j) q[j] = *reinterpret_cast<const uint4*>(res + 8 * j);
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const uint32_t w[4] = {q[j].x, q[j].y, q[j].z, q[j].w};
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    const uint32_t o = h[4 * j + i];
                    h[4 * j + i] = pack_h2(add_f16(static_cast<uint16_t>(w[i] & 0xFFFFu), static_cast<uint16_t>(o & 0xFFFFu)),
                                           add_f16(static_cast<uint16_t>(w[i] >> 16), static_cast<uint16_t>(o >> 16)));
                }
            }
        }
        if ((reinterpret_cast<uintptr_t>(dst) & 31) == 0) {
            // whole 32-byte sectors (see store_partial_chunk)
            st_global_v8(dst, h[0], h[1], h[2], h[3], h[4], h[5], h[6], h[7]);
            st_global_v8(dst + 16, h[8], h[9], h[10], h[11], h[12], h[13], h[14], h[15]);
        } else {
#pragma unroll
            for (int j = 0; j < 16; j += 4)
                *reinterpret_cast<uint4*>(dst + 2 * j) = make_uint4(h[j], h[j + 1], h[j + 2], h[j + 3]);
        }
    } else {
#pragma unroll
        for (int j = 0; j < 32; ++j)
            if (col0 + j < a.N) dst[j] = add_residual(round_out(__uint_as_float(r[j]), a.bias, col0 + j), res, j);
    }
}

// Swap mode: 16 accumulator columns (tokens) of one weight row; each column
// is one token's output at weight row `n`, so a warp's 32 lanes write 32
// consecutive outputs of that token.
//
// With greedy-pick partials (a.am_val) every lane of the warp must call this:
// the warp's 32 rows (one chunk) are reduced to their best (value, index)
// per token by shuffles.
__device__ __forceinline__ void store_swap_chunk(const TcGemmArgs& a, const uint32_t (&r)[16], int64_t n,
                                                 int64_t m0) {
    const bool in = n < a.N;
#pragma unroll
    for (int j = 0; j < 16; ++j) {
        const int64_t m = m0 + j;
        if (m >= a.M) break;  // uniform over the warp
        if (a.out_f32) {
            if (in) static_cast<float*>(a.y)[m * a.ldy + n] = __uint_as_float(r[j]);
            continue;
        }
        const uint16_t h = in ? add_residual(round_out(__uint_as_float(r[j]), a.bias, n), a.residual, m * a.ldr + n) : 0;
        if (in && a.y != nullptr) static_cast<uint16_t*>(a.y)[m * a.ldy + n] = h;
        if (a.am_val != nullptr) {
            const ArgBest b = warp_arg_best(in ? ArgBest{nan_to_ninf(f16_bits_to_f32(h)), n} : ArgBest{-INFINITY, INT64_MAX});
            if ((threadIdx.x & 31) == 0) {
                const int64_t at = m * a.am_chunks + (n >> 5);
                a.am_val[at] = b.v;
                a.am_idx[at] = b.i;
            }
        }
    }
}

// SwiGLU epilogue, swap mode: lane = weight row n, r[j] = token m0 + j.  Even
// rows are gate rows, odd rows the matching up rows (the partner lane n ^ 1);
// the even lane stores fp16(silu(gate) * up) for its pair n / 2
// (qwen_model.cpp:278-285: gate and up rounded to FP16, SiLU from the FP16
// table, the product rounded).  Every lane reaches the shuffles.
__device__ __forceinline__ void store_swap_chunk_swiglu(const TcGemmArgs& a, const uint32_t (&r)[16], int64_t n,
                                                        int64_t m0) {
    uint16_t* y = static_cast<uint16_t*>(a.y);
#pragma unroll
    for (int j = 0; j < 16; ++j) {
        const int64_t m = m0 + j;
        if (m >= a.M) break;  // uniform over the warp
        const uint32_t h = f32_to_f16_bits(__uint_as_float(r[j]));
        const uint32_t up = __shfl_xor_sync(0xFFFFFFFFu, h, 1);
        if ((n & 1) == 0 && n < a.N) {
            const float sg = f16_bits_to_f32(a.swiglu_lut[h]);
            y[m * a.ldy + (n >> 1)] = f32_to_f16_bits(__fmul_rn(sg, f16_bits_to_f32(static_cast<uint16_t>(up))));
        }
    }
}

// SwiGLU epilogue, normal mode: lane = token row, r[j] = weight row col0 + j
// (col0 even), so pairs are (r[2i], r[2i+1]) -> y[row][col0 / 2 + i].
__device__ __forceinline__ void store_row_chunk_swiglu(const TcGemmArgs& a, const uint32_t (&r)[32], int64_t row,
                                                       int64_t col0) {
    uint16_t h[16];
#pragma unroll
    for (int i = 0; i < 16; ++i) {
        const uint16_t g = f32_to_f16_bits(__uint_as_float(r[2 * i]));
        const uint16_t u = f32_to_f16_bits(__uint_as_float(r[2 * i + 1]));
        h[i] = f32_to_f16_bits(__fmul_rn(f16_bits_to_f32(a.swiglu_lut[g]), f16_bits_to_f32(u)));
    }
    uint16_t* dst = static_cast<uint16_t*>(a.y) + row * a.ldy + (col0 >> 1);
    if (col0 + 32 <= a.N && (reinterpret_cast<uintptr_t>(dst) & 15) == 0) {
        *reinterpret_cast<uint4*>(dst) = make_uint4(pack_h2(h[0], h[1]), pack_h2(h[2], h[3]), pack_h2(h[4], h[5]),
                                                    pack_h2(h[6], h[7]));
        *reinterpret_cast<uint4*>(dst + 8) = make_uint4(pack_h2(h[8], h[9]), pack_h2(h[10], h[11]),
                                                        pack_h2(h[12], h[13]), pack_h2(h[14], h[15]));
    } else {
#pragma unroll
        for (int i = 0; i < 16; ++i)
            if (col0 + 2 * i + 1 < a.N) dst[i] = h[i];
    }
}

// Swap mode: up to 16 FP32 columns (tokens) into a tail slot, laid out as
// [bn / 4 token groups][128 rows][4 tokens] so that one float4 per lane of a
// warp (32 consecutive rows) is one contiguous 512-byte run.  Only the
// `groups` float4 groups holding real tokens are written (columns past the
// last token are never read back).
__device__ __forceinline__ void store_partial_chunk16(const TcGemmArgs& a, const uint32_t (&r)[16], int slot,
                                                     int row_in_tile, int col_in_tile, int bn, int groups) {
    float* dst = a.partials + static_cast<int64_t>(slot) * kBM * bn + (col_in_tile / 4) * (kBM * 4) + row_in_tile * 4;
#pragma unroll
    for (int g = 0; g < 4; ++g)
        if (g < groups)
            *reinterpret_cast<uint4*>(dst + g * (kBM * 4)) =
                make_uint4(r[4 * g], r[4 * g + 1], r[4 * g + 2], r[4 * g + 3]);
}

__device__ __forceinline__ void add4(float4& s, const float4& p) {
    s.x += p.x;
    s.y += p.y;
    s.z += p.z;
    s.w += p.w;
}

// Sum of `splits` partial slices (slice order) of `ng` float4 groups starting
// at token column c0 of one weight row (layout of store_partial_chunk16);
// KB slices x KG groups of loads are issued before any of them is added.
template <int KB, int KG>
__device__ __forceinline__ void sum_slices(const float* base, int64_t slice, int splits, int c0, int ng,
                                           float4 (&sum)[4]) {
#pragma unroll 1
    for (int sp0 = 0; sp0 < splits; sp0 += KB) {
        float4 p[KB][KG];
#pragma unroll
        for (int b = 0; b < KB; ++b)
#pragma unroll
            for (int g = 0; g < KG; ++g)
                if (sp0 + b < splits && g < ng)
                    p[b][g] = __ldcg(reinterpret_cast<const float4*>(base + (sp0 + b) * slice + (c0 / 4 + g) * (kBM * 4)));
#pragma unroll
        for (int b = 0; b < KB; ++b)
#pragma unroll
            for (int g = 0; g < KG; ++g)
                if (sp0 + b < splits && g < ng) {
                    if (sp0 + b == 0)
                        sum[g] = p[b][g];
                    else
                        add4(sum[g], p[b][g]);
                }
    }
}

// Swap-mode K-split finish for one 32-row quadrant of a tail tile, run by the
// whole epilogue warp that just stored its partial rows.  The warp counts
// itself in; only the warp that completes the count (the last of the
// tail_splits slices to arrive) sums all slices in slice order -- so the
// result does not depend on arrival order -- stores the output and resets the
// counter.  Nobody waits for anybody, so a slice lost to an error cannot hang
// the kernel; it only leaves its tile unfinished.
//
// The sum is latency-bound (a few KB per warp from L2), so each lane reads
// only its weight row's real token columns and keeps up to 4 slices x 16
// tokens (or 8 slices x 4 tokens) of loads in flight before adding them in
// order.
template <int BN>
__device__ __forceinline__ void swap_tail_fixup(const TcGemmArgs& a, const Unit& w, int n_tail, int quad, int lane) {
    // The warp's partial rows are ordered before lane 0's arrival (__syncwarp),
    // which releases them with one acquire-release atomic; the last arrival's
    // acquire makes every slice's rows visible to the warp after the shuffle.
    __syncwarp();
    int last = 0;
    if (lane == 0) {
        int* cnt = a.tile_counters + w.ti * 4 + quad;
        int old;
        asm volatile("atom.add.acq_rel.gpu.global.s32 %0, [%1], 1;" : "=r"(old) : "l"(cnt) : "memory");
        last = old == a.tail_splits - 1;
        if (last) *cnt = 0;
    }
    last = __shfl_sync(0xFFFFFFFFu, last, 0);
    if (!last) return;
    const int r = quad * 32 + lane;
    const int64_t n = static_cast<int64_t>(w.mt) * kBM + r;  // weight row = output column
    const int cols = min(BN, a.M - w.nt * BN);                 // tokens in this tile
    const int64_t slice = static_cast<int64_t>(n_tail) * kBM * BN;
    const float* base = a.partials + static_cast<int64_t>(w.ti) * kBM * BN + r * 4;  // slice 0, token group 0
    constexpr int kG = 4;  // float4 groups (16 tokens) per pass
#pragma unroll 1
    for (int c0 = 0; c0 < cols; c0 += 16) {
        const int ng = min(kG, (cols - c0 + 3) / 4);
        float4 sum[kG];
        // One batch of loads covers up to 8 slices of one group (<= 4
        // tokens, 16-token tiles) or 4 slices of 2..4 groups (more would
        // spill registers).
        if (BN == 16 && ng == 1)
            sum_slices<8, 1>(base, slice, a.tail_splits, c0, ng, sum);
        else
            sum_slices<4, kG>(base, slice, a.tail_splits, c0, ng, sum);
        uint32_t bits[16] = {};
#pragma unroll
        for (int g = 0; g < kG; ++g)
            if (g < ng) {
                bits[4 * g] = __float_as_uint(sum[g].x);
                bits[4 * g + 1] = __float_as_uint(sum[g].y);
                bits[4 * g + 2] = __float_as_uint(sum[g].z);
                bits[4 * g + 3] = __float_as_uint(sum[g].w);
            }
        store_swap_chunk(a, bits, n, static_cast<int64_t>(w.nt) * BN + c0);
    }
}

// ------------------------------------------------ cluster K-split (swap mode)

__device__ __forceinline__ uint32_t cluster_rank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}

__device__ __forceinline__ uint32_t cluster_size() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_nctarank;" : "=r"(r));
    return r;
}

// Hardware cluster barrier, split: every thread arrives once right after the
// barriers are initialised (nothing before that can fail or return), and
// waits once later; the wait therefore always completes.
__device__ __forceinline__ void cluster_arrive() {
    asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory");
}

__device__ __forceinline__ void cluster_wait() {
    asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory");
}

// Address of the same shared-memory location in CTA `rank` of the cluster.
__device__ __forceinline__ uint32_t cluster_map(uint32_t smem_addr, uint32_t rank) {
    uint32_t r;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(smem_addr), "r"(rank));
    return r;
}

// Arrive on mbarrier `bar` of CTA `rank`, releasing this thread's (and,
// through the preceding CTA barrier, its CTA's) shared-memory writes to the
// cluster.
__device__ __forceinline__ void mbar_arrive_cluster(uint64_t* bar, uint32_t rank) {
    asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_map(smem_u32(bar), rank))
                 : "memory");
}

__device__ __forceinline__ bool mbar_try_wait_cluster(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.b32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

// Bounded wait with cluster-scope acquire.  With give_up_on_error it also
// stops as soon as any thread of the grid has raised an error; without it
// only the time limit ends the wait (used where the caller's shared memory
// may still be read by another CTA of the cluster).
__device__ __forceinline__ bool mbar_wait_cluster(uint64_t* bar, uint32_t parity, int* flag, int code,
                                                  bool give_up_on_error) {
    if (mbar_try_wait_cluster(bar, parity)) return true;
    const uint64_t t0 = globaltimer_ns();
    for (uint32_t it = 1;; ++it) {
        if (mbar_try_wait_cluster(bar, parity)) return true;
        if ((it & 255u) == 0) {
            if (give_up_on_error && error_raised(flag)) return false;
            if (globaltimer_ns() - t0 > kWaitLimitNs) {
                raise_error(flag, code);
                return false;
            }
        }
    }
}

__device__ __forceinline__ float4 ld_cluster_f4(uint32_t addr) {
    float4 v;
    asm volatile("ld.shared::cluster.v4.f32 {%0, %1, %2, %3}, [%4];"
                 : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
                 : "r"(addr)
                 : "memory");
    return v;
}

// Named barrier of the 128 epilogue threads (id 1); returns whether `pred`
// held on all of them.
__device__ __forceinline__ bool epi_bar_and(bool pred) {
    uint32_t r;
    asm volatile(
        "{\n\t.reg .pred p, q;\n\t"
        "setp.ne.u32 p, %1, 0;\n\t"
        "bar.red.and.pred q, 1, 128, p;\n\t"
        "selp.u32 %0, 1, 0, q;\n\t}"
        : "=r"(r)
        : "r"(pred ? 1u : 0u)
        : "memory");
    return r != 0;
}

__device__ __forceinline__ void epi_bar_sync() { asm volatile("bar.sync 1, 128;" ::: "memory"); }

// The same over the N epilogue threads of a kernel (named barrier 1).
template <int N>
__device__ __forceinline__ bool epi_bar_and_n(bool pred) {
    uint32_t r;
    asm volatile(
        "{\n\t.reg .pred p, q;\n\t"
        "setp.ne.u32 p, %1, 0;\n\t"
        "bar.red.and.pred q, 1, %2, p;\n\t"
        "selp.u32 %0, 1, 0, q;\n\t}"
        : "=r"(r)
        : "r"(pred ? 1u : 0u), "n"(N)
        : "memory");
    return r != 0;
}

template <int N>
__device__ __forceinline__ void epi_bar_sync_n() {
    asm volatile("bar.sync 1, %0;" ::"n"(N) : "memory");
}

// Four consecutive outputs n..n+3 of one token (swap mode: consecutive weight
// rows), rounded like every other store of this kernel.
__device__ __forceinline__ void store_swap_rows4(const TcGemmArgs& a, const float4& s, int64_t n, int64_t token) {
    if (n >= a.N) return;
    const float v[4] = {s.x, s.y, s.z, s.w};
    const bool whole = n + 4 <= a.N;
    if (a.out_f32) {
        float* dst = static_cast<float*>(a.y) + token * a.ldy + n;
        if (whole && (reinterpret_cast<uintptr_t>(dst) & 15) == 0) {
            *reinterpret_cast<float4*>(dst) = s;
        } else {
            for (int i = 0; i < 4 && n + i < a.N; ++i) dst[i] = v[i];
        }
        return;
    }
    uint16_t* dst = static_cast<uint16_t*>(a.y) + token * a.ldy + n;
    const int64_t ri = token * a.ldr + n;
    if (whole && (reinterpret_cast<uintptr_t>(dst) & 7) == 0) {
        uint16_t h[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) h[i] = add_residual(round_out(v[i], a.bias, n + i), a.residual, ri + i);
        *reinterpret_cast<uint2*>(dst) = make_uint2(pack_h2(h[0], h[1]), pack_h2(h[2], h[3]));
    } else {
        for (int i = 0; i < 4 && n + i < a.N; ++i)
            dst[i] = add_residual(round_out(v[i], a.bias, n + i), a.residual, ri + i);
    }
}

// Cluster K-split finish, run by the 128 epilogue threads of every CTA of the
// cluster (one K-slice each).  Each CTA copies its FP32 accumulator (real
// token columns only) into its own shared memory -- the operand ring, idle
// once the last MMA has completed -- as [token][128 rows], and arrives on
// every CTA's `ready` barrier.  CTA r then sums rows [128 r / S, 128 (r+1) / S)
// (in 4-row groups) over the S slices, in slice order like the global-memory
// finish, reading the other CTAs' copies through distributed shared memory,
// and stores them.  A CTA leaves only after all S CTAs arrived on its `done`
// barrier (they have finished reading its copy).  Every wait is bounded; a
// slice that never arrives leaves its tile unwritten with an error raised.
template <int BN>
__device__ __forceinline__ void swap_cluster_finish(const TcGemmArgs& a, uint8_t* smem, uint32_t tmem_base,
                                                    uint64_t* tfull, uint64_t* ready, uint64_t* done, int num_m,
                                                    int n_tail, int num_kb, int quad, int lane, int et) {
    const uint32_t S = static_cast<uint32_t>(a.cluster_k);
    const uint32_t rank = cluster_rank();
    const Unit w = decode_unit(a, blockIdx.x, num_m, n_tail, num_kb);
    const int cols = min(BN, a.M - w.nt * BN);
    float* stg = reinterpret_cast<float*>(smem);
    // The launch's cluster shape must match the slice numbering (the host
    // guarantees it); otherwise no CTA of the cluster is addressed at all.
    if (cluster_size() != S || rank != static_cast<uint32_t>(w.slot)) {
        if (et == 0) raise_error(a.err_flag, kErrEpiWait);
        cluster_wait();
        return;
    }
    int ok = 1;
    if (lane == 0) ok = mbar_wait(&tfull[0], 0, a.err_flag, kErrEpiWait) ? 1 : 0;
    ok = __shfl_sync(0xFFFFFFFFu, ok, 0);
    if (ok) {
        tc_fence_after();
        const uint32_t t_row = tmem_base + (static_cast<uint32_t>(quad * 32) << 16);
        const int r = quad * 32 + lane;
#pragma unroll 1
        for (int c = 0; c * 16 < cols; ++c) {
            uint32_t v[16];
            __syncwarp();
            tmem_ld_16cols(t_row + c * 16, v);
#pragma unroll
            for (int j = 0; j < 16; ++j)
                if (c * 16 + j < cols) stg[(c * 16 + j) * kBM + r] = __uint_as_float(v[j]);
        }
    }
    const bool staged = epi_bar_and(ok != 0);
    cluster_wait();  // every CTA of the cluster has initialised its barriers
    if (staged && et == 0)
        for (uint32_t p = 0; p < S; ++p) mbar_arrive_cluster(ready, p);
    const bool go = staged && mbar_wait_cluster(ready, 0, a.err_flag, kErrEpiWait, true);
    if (go) {
        const int g0 = static_cast<int>(32u * rank / S);
        const int G = static_cast<int>(32u * (rank + 1) / S) - g0;
        const uint32_t base = smem_u32(stg);
        uint32_t peer[8];
#pragma unroll
        for (int p = 0; p < 8; ++p) peer[p] = p < static_cast<int>(S) ? cluster_map(base, p) : 0u;
#pragma unroll 1
        for (int e = et; e < G * cols; e += kEpiThreads) {
            const int m = e / G;
            const int nl = (g0 + e - m * G) * 4;  // row within the tile
            const uint32_t off = static_cast<uint32_t>(m * kBM + nl) * 4u;
            float4 v[8];
#pragma unroll
            for (int p = 0; p < 8; ++p)
                if (p < static_cast<int>(S)) v[p] = ld_cluster_f4(peer[p] + off);
            float4 sum = v[0];
#pragma unroll
            for (int p = 1; p < 8; ++p)
                if (p < static_cast<int>(S)) add4(sum, v[p]);
            store_swap_rows4(a, sum, static_cast<int64_t>(w.mt) * kBM + nl, static_cast<int64_t>(w.nt) * BN + m);
        }
    }
    epi_bar_sync();  // this CTA's reads of the cluster's copies are complete
    if (et == 0) {
        for (uint32_t p = 0; p < S; ++p) mbar_arrive_cluster(done, p);
        // Stay resident (shared memory valid) until every CTA has read this
        // one's copy; only the time limit ends this wait.
        mbar_wait_cluster(done, 0, a.err_flag, kErrEpiWait, false);
    }
}

template <int BN, bool SWAP, bool SEG>
__global__ void __launch_bounds__(threads_of<SEG>(), SWAP ? 2 : 1)
    tc_gemm_kernel(const TcGemmArgs a, const __grid_constant__ CUtensorMap tma,
                   const __grid_constant__ CUtensorMap tmb) {
    static_assert(!(SEG && SWAP), "segmented accumulation is a normal-mode variant");
    using Cfg = TcCfg<BN, SWAP>;
    constexpr int kEpi = SEG ? 256 : kEpiThreads;         // epilogue threads
    const int kSegLen = SEG ? max(1, a.seg_kb) : (1 << 30);  // k-blocks per accumulator segment
    constexpr int S = Cfg::kStages;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* sA = smem;
    uint8_t* sB = smem + S * Cfg::kABytes;
    uint64_t* bars = reinterpret_cast<uint64_t*>(sB + S * Cfg::kBBytes);
    uint64_t* full = bars;
    uint64_t* empty = bars + S;
    uint64_t* tfull = bars + 2 * S;
    uint64_t* tempty = tfull + 2;
    uint64_t* drain = tempty + 2;
    uint64_t* cl_ready = drain + 1;  // cluster K-split finish (swap mode)
    uint64_t* cl_done = drain + 2;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 3);
    const bool clustered = SWAP && a.cluster_k > 1;

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;

    if (threadIdx.x == 0) {
        for (int s = 0; s < S; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        for (int i = 0; i < 2; ++i) {
            mbar_init(&tfull[i], 1);
            mbar_init(&tempty[i], kEpi);
        }
        mbar_init(drain, 1);
        if (clustered) {
            mbar_init(cl_ready, static_cast<uint32_t>(a.cluster_k));
            mbar_init(cl_done, static_cast<uint32_t>(a.cluster_k));
        }
        fence_barrier_init();
    }
    if (warp == 1) {
        tmem_alloc(tmem_slot, Cfg::kTmemCols);
        tmem_relinquish();
    }
    if (warp == 0 && lane == 0) {
        prefetch_tmap(&tma);
        prefetch_tmap(&tmb);
    }
    // The next launch (if it has a programmatic edge) may start its own
    // prologue and weight stream while this grid works.
    griddep_launch_dependents();
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (clustered) cluster_arrive();  // barriers initialised; every thread, once
    const uint32_t tmem_base = *tmem_slot;

    // A tiles (128 rows) vary fastest; in swap mode A is W and B is X.
    const int num_m = SWAP ? (a.N + kBM - 1) / kBM : (a.M + kBM - 1) / kBM;
    const int num_n = SWAP ? (a.M + BN - 1) / BN : (a.N + BN - 1) / BN;
    const int num_kb = (a.K + kBK - 1) / kBK;
    const int n_tail = num_m * num_n - a.full_tiles;
    const int total = a.full_tiles + n_tail * a.tail_splits;

    if (warp == 0) {
        if (lane == 0) {
            int stage = 0;
            uint32_t phase = 0;
            uint32_t issued = 0, issued_parity = 0;
            bool ok = true;
            // The weight half of one ring stage (tiled weights only).  Decode
            // (swap mode) reads each weight byte once per step: it streams with
            // an evict-first L2 policy so the KV cache and activations stay cached.
            const uint64_t stream_policy = l2_policy_evict_first();
            auto load_w = [&](const Unit& w, int kb, int st) {
                if constexpr (SWAP) {
                    // W is A: one contiguous, already swizzled 128 x 64 tile.
                    bulk_load_hint(sA + st * Cfg::kABytes,
                                   a.w_tiled + tiled_offset(static_cast<int64_t>(w.mt) * kBM, static_cast<int64_t>(kb) * kBK, a.w_k_tiles),
                                   Cfg::kABytes, &full[st], stream_policy);
                } else {
                    // W is B: BN rows = BN/128 whole tiles, or half of one for BN = 64.
                    constexpr int kPieces = BN >= 128 ? BN / 128 : 1;
                    constexpr uint32_t kPieceBytes = (BN >= 128 ? 128 : BN) * kBK * 2;
#pragma unroll
                    for (int h = 0; h < kPieces; ++h)
                        bulk_load(sB + st * Cfg::kBBytes + h * kPieceBytes,
                                  a.w_tiled + tiled_offset(static_cast<int64_t>(w.nt) * BN + h * 128,
                                                           static_cast<int64_t>(kb) * kBK, a.w_k_tiles),
                                  kPieceBytes, &full[st]);
                }
            };
            // The activation half (always through its tensor map).
            auto load_x = [&](const Unit& w, int kb, int st) {
                if constexpr (SWAP) {
                    tma_load_2d(sB + st * Cfg::kBBytes, &tmb, &full[st], kb * kBK, w.nt * BN);
                } else {
                    tma_load_2d(sA + st * Cfg::kABytes, &tma, &full[st], kb * kBK, w.mt * kBM);
                }
            };
            // This CTA's (unit, k-block) sequence.
            int u = blockIdx.x, kb = 0;
            Unit w{};
            if (u < total) {
                w = decode_unit(a, u, num_m, n_tail, num_kb);
                kb = w.kb0;
            }
            auto advance = [&](int& uu, int& kk, Unit& ww) {
                if (++kk == ww.kb1) {
                    uu += gridDim.x;
                    if (uu < total) {
                        ww = decode_unit(a, uu, num_m, n_tail, num_kb);
                        kk = ww.kb0;
                    }
                }
            };
            auto claim = [&](int st) {
                mbar_arrive_expect_tx(&full[st], Cfg::kStageBytes);
                issued |= 1u << st;
                issued_parity = (issued_parity & ~(1u << st)) | (phase << st);
            };
            // A tiled weight is complete before its upload returns and is never
            // written again, so the first ring pass of weight tiles is requested
            // before waiting for the kernel this one overlaps; the activations,
            // and every global write, come after the wait.
            int pre = 0;
            if (a.w_prefetch && a.w_tiled != nullptr) {
                for (; pre < S && u < total; ++pre) {
                    claim(stage);  // a fresh ring: no stage to wait for
                    load_w(w, kb, stage);
                    advance(u, kb, w);
                    if (++stage == S) {
                        stage = 0;
                        phase ^= 1u;
                    }
                }
            }
            griddep_wait();
            {
                int u2 = blockIdx.x, kb2 = 0;
                Unit w2{};
                if (pre > 0) {
                    w2 = decode_unit(a, u2, num_m, n_tail, num_kb);
                    kb2 = w2.kb0;
                }
                for (int i = 0; i < pre; ++i) {
                    load_x(w2, kb2, i);
                    advance(u2, kb2, w2);
                }
            }
            for (; u < total; advance(u, kb, w)) {
                if (!mbar_wait(&empty[stage], phase ^ 1u, a.err_flag, kErrTmaWait)) {
                    ok = false;
                    break;
                }
                claim(stage);
                if (a.w_tiled == nullptr) {
                    tma_load_2d(sA + stage * Cfg::kABytes, &tma, &full[stage], kb * kBK, w.mt * kBM);
                    tma_load_2d(sB + stage * Cfg::kBBytes, &tmb, &full[stage], kb * kBK, w.nt * BN);
                } else {
                    load_w(w, kb, stage);
                    load_x(w, kb, stage);
                }
                if (++stage == S) {
                    stage = 0;
                    phase ^= 1u;
                }
            }
            if (!ok) {
                // Leave no copy in flight into shared memory we are about to give up.
                for (int s = 0; s < S; ++s)
                    if (issued & (1u << s)) mbar_wait(&full[s], (issued_parity >> s) & 1u, nullptr, kErrDrainWait);
            }
        }
    } else if (warp == 1) {
        // Bounded waits start only once the kernel this one may overlap is done.
        griddep_wait();
        if (lane == 0) {
            const uint32_t idesc = idesc_f16_f32(kBM, BN);
            int stage = 0;
            uint32_t phase = 0;
            int acc = 0;
            uint32_t acc_phase = 0;
            bool any = false;
            bool ok = true;
            for (int u = blockIdx.x; u < total && ok; u += gridDim.x) {
                const Unit w = decode_unit(a, u, num_m, n_tail, num_kb);
                // One accumulator per segment of the unit's k-blocks (one
                // segment unless SEG), alternating between the two.
                for (int s0 = w.kb0; s0 < w.kb1 && ok; s0 += kSegLen) {
                    const int s1 = min(s0 + kSegLen, w.kb1);
                    if (!mbar_wait(&tempty[acc], acc_phase ^ 1u, a.err_flag, kErrMmaWait)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(acc * BN);
                    for (int kb = s0; kb < s1; ++kb) {
                        if (!mbar_wait(&full[stage], phase, a.err_flag, kErrMmaWait)) {
                            ok = false;
                            break;
                        }
                        tc_fence_after();
                        const uint32_t a_addr = smem_u32(sA + stage * Cfg::kABytes);
                        const uint32_t b_addr = smem_u32(sB + stage * Cfg::kBBytes);
#pragma unroll
                        for (int k = 0; k < kBK / 16; ++k) {
                            tc_mma_f16(d_tmem, smem_desc_k128(a_addr + k * 32), smem_desc_k128(b_addr + k * 32),
                                       idesc, (kb > s0 || k > 0) ? 1u : 0u);
                        }
                        tc_commit(&empty[stage]);
                        any = true;
                        if (++stage == S) {
                            stage = 0;
                            phase ^= 1u;
                        }
                    }
                    if (!ok) break;
                    tc_commit(&tfull[acc]);
                    acc ^= 1;
                    if (acc == 0) acc_phase ^= 1u;
                }
            }
            if (any) {
                // Every MMA this thread issued must finish before TMEM is freed.
                tc_commit(drain);
                mbar_wait(drain, 0, nullptr, kErrDrainWait);
            }
        }
    } else if constexpr (SEG) {
        // 8 epilogue warps: warp w reads TMEM lanes 32 (w mod 4) .. +31 (its
        // rows) and columns [half * BN/2, (half + 1) * BN/2) of each segment's
        // accumulator and keeps their running sums in registers.  The last
        // segment's sums are written back into its accumulator (which this
        // thread still owns) and stored from there 32 columns at a time, so
        // the store code never holds every sum at once.
        constexpr int HB = BN / 2;
        const int quad = warp & 3;
        const int half = (warp - 2) >> 2;
        griddep_wait();  // before any bounded wait and any global write
        int acc = 0;
        uint32_t acc_phase = 0;
        for (int u = blockIdx.x; u < total; u += gridDim.x) {
            const Unit w = decode_unit(a, u, num_m, n_tail, num_kb);
            float sum[HB];
            bool ok = true;
            uint32_t t_row = 0;
            for (int s0 = w.kb0; s0 < w.kb1; s0 += kSegLen) {
                int got = 1;
                if (lane == 0) got = mbar_wait(&tfull[acc], acc_phase, a.err_flag, kErrEpiWait) ? 1 : 0;
                got = __shfl_sync(0xFFFFFFFFu, got, 0);
                if (!got) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                t_row = tmem_base + (static_cast<uint32_t>(quad * 32) << 16) + static_cast<uint32_t>(acc * BN + half * HB);
                const bool last = s0 + kSegLen >= w.kb1;
                // 16 columns per load keeps the running sums and one load's
                // registers within the 168 a thread has at 10 warps per CTA.
#pragma unroll
                for (int c = 0; c < HB / 16; ++c) {
                    uint32_t r[16];
                    __syncwarp();
                    tmem_ld_16cols(t_row + c * 16, r);
#pragma unroll
                    for (int j = 0; j < 16; ++j)
                        sum[c * 16 + j] = s0 == w.kb0 ? __uint_as_float(r[j]) : __fadd_rn(sum[c * 16 + j], __uint_as_float(r[j]));
                    if (last) {
#pragma unroll
                        for (int j = 0; j < 16; ++j) r[j] = __float_as_uint(sum[c * 16 + j]);
                        tmem_st_16cols(t_row + c * 16, r);
                    }
                }
                if (last) break;  // the accumulator stays owned until the stores below
                tc_fence_before();
                mbar_arrive(&tempty[acc]);
                acc ^= 1;
                if (acc == 0) acc_phase ^= 1u;
            }
            if (!ok) break;
            const int row_in_tile = quad * 32 + lane;
            const int64_t row = static_cast<int64_t>(w.mt) * kBM + row_in_tile;
#pragma unroll 1
            for (int c = 0; c < HB / 32; ++c) {
                uint32_t r[32];
                __syncwarp();
                tmem_ld_32cols(t_row + c * 32, r);
                const int col_in_tile = half * HB + c * 32;
                const int64_t col0 = static_cast<int64_t>(w.nt) * BN + col_in_tile;
                if (w.slot >= 0) {
                    store_partial_chunk(a, r, w.slot, row_in_tile, col_in_tile, BN);
                } else if (row < a.M && col0 < a.N) {
                    if (a.swiglu_lut != nullptr)
                        store_row_chunk_swiglu(a, r, row, col0);
                    else
                        store_row_chunk(a, r, row, col0);
                }
            }
            tc_fence_before();
            mbar_arrive(&tempty[acc]);
            acc ^= 1;
            if (acc == 0) acc_phase ^= 1u;
        }
    } else if (clustered) {
        griddep_wait();  // before any bounded wait and any global write
        if constexpr (SWAP)
            swap_cluster_finish<BN>(a, smem, tmem_base, tfull, cl_ready, cl_done, num_m, n_tail, num_kb, warp & 3,
                                    lane, threadIdx.x - 64);
    } else {
        const int quad = warp & 3;  // TMEM lanes this warp may read: 32*quad .. +31
        griddep_wait();  // before any bounded wait and any global write
        int acc = 0;
        uint32_t acc_phase = 0;
        for (int u = blockIdx.x; u < total; u += gridDim.x) {
            const Unit w = decode_unit(a, u, num_m, n_tail, num_kb);
            // One lane waits; the verdict is shared so the warp stays
            // converged for the .sync.aligned TMEM loads below.
            int ok = 1;
            if (lane == 0) ok = mbar_wait(&tfull[acc], acc_phase, a.err_flag, kErrEpiWait) ? 1 : 0;
            ok = __shfl_sync(0xFFFFFFFFu, ok, 0);
            if (!ok) break;
            tc_fence_after();
            // TMEM lane = A row of the tile (x row, or weight row in swap mode).
            const int64_t row = static_cast<int64_t>(w.mt) * kBM + quad * 32 + lane;
            const uint32_t t_row = tmem_base + (static_cast<uint32_t>(quad * 32) << 16) +
                                   static_cast<uint32_t>(acc * BN);
            if constexpr (SWAP) {
                // Only the chunks holding real tokens (warp-uniform bound).
                const int cols = min(BN, a.M - w.nt * BN);
#pragma unroll 1
                for (int c = 0; c * 16 < cols; ++c) {
                    uint32_t r[16];
                    __syncwarp();
                    tmem_ld_16cols(t_row + c * 16, r);
                    if (w.slot >= 0) {
                        store_partial_chunk16(a, r, w.slot, quad * 32 + lane, c * 16, BN, min(4, (cols - c * 16 + 3) / 4));
                    } else if (a.swiglu_lut != nullptr) {
                        store_swap_chunk_swiglu(a, r, row, static_cast<int64_t>(w.nt) * BN + c * 16);
                    } else {
                        store_swap_chunk(a, r, row, static_cast<int64_t>(w.nt) * BN + c * 16);
                    }
                }
            } else {
#pragma unroll 1
                for (int c = 0; c < BN / 32; ++c) {
                    uint32_t r[32];
                    __syncwarp();
                    tmem_ld_32cols(t_row + c * 32, r);
                    const int64_t col0 = static_cast<int64_t>(w.nt) * BN + c * 32;
                    if (w.slot >= 0) {
                        store_partial_chunk(a, r, w.slot, quad * 32 + lane, c * 32, BN);
                    } else if (row < a.M && col0 < a.N) {
                        if (a.swiglu_lut != nullptr)
                            store_row_chunk_swiglu(a, r, row, col0);
                        else
                            store_row_chunk(a, r, row, col0);
                    }
                }
            }
            tc_fence_before();
            mbar_arrive(&tempty[acc]);  // the accumulator is free; the fix-up reads global memory only
            if constexpr (SWAP) {
                if (w.slot >= 0) swap_tail_fixup<BN>(a, w, n_tail, quad, lane);
            }
            acc ^= 1;
            if (acc == 0) acc_phase ^= 1u;
        }
    }

    if (clustered && warp < 2) {
        __syncwarp();
        cluster_wait();  // pairs with the arrive above (the epilogue warps wait in the finish)
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        __syncwarp();
        tc_fence_after();
        tmem_dealloc(tmem_base, Cfg::kTmemCols);
    }
}

// Kernel attributes, once per device.
template <int BN, bool SWAP, bool SEG>
cudaError_t prepare_bn() {
    static bool attr_set[64] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
    if (!attr_set[dev]) {
        cudaError_t e = cudaFuncSetAttribute(tc_gemm_kernel<BN, SWAP, SEG>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             static_cast<int>(TcCfg<BN, SWAP>::kSmem));
        if (e != cudaSuccess) return e;
        // All shared memory, no L1 carve-out: every instance then runs under one
        // SM configuration, so two swap-mode CTAs (of one GEMM and the next)
        // can share an SM.
        e = cudaFuncSetAttribute(tc_gemm_kernel<BN, SWAP, SEG>, cudaFuncAttributePreferredSharedMemoryCarveout,
                                 cudaSharedmemCarveoutMaxShared);
        if (e != cudaSuccess) return e;
        attr_set[dev] = true;
    }
    return cudaSuccess;
}

template <int BN, bool SWAP, bool SEG = false>
cudaError_t launch_bn(const TcGemmArgs& a, const CUtensorMap& ta, const CUtensorMap& tb, cudaStream_t s) {
    cudaError_t e = prepare_bn<BN, SWAP, SEG>();
    if (e != cudaSuccess) return e;
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(static_cast<unsigned>(a.grid));
    cfg.blockDim = dim3(threads_of<SEG>());
    cfg.dynamicSmemBytes = TcCfg<BN, SWAP>::kSmem;
    cfg.stream = s;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    int n_attr = 1;
    if (SWAP && a.cluster_k > 1) {
        attr[1].id = cudaLaunchAttributeClusterDimension;
        attr[1].val.clusterDim.x = static_cast<unsigned>(a.cluster_k);
        attr[1].val.clusterDim.y = 1;
        attr[1].val.clusterDim.z = 1;
        n_attr = 2;
    }
    cfg.attrs = attr;
    cfg.numAttrs = n_attr;
    e = cudaLaunchKernelEx(&cfg, tc_gemm_kernel<BN, SWAP, SEG>, a, ta, tb);
    if (e != cudaSuccess) return e;
    note_launches(1);
    return cudaGetLastError();
}

// Whether clusters of k swap-mode CTAs of width BN can be resident at all.
template <int BN>
bool cluster_fits(int k) {
    if (prepare_bn<BN, true, false>() != cudaSuccess) return false;
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(static_cast<unsigned>(k));
    cfg.blockDim = dim3(kThreadsTc);
    cfg.dynamicSmemBytes = TcCfg<BN, true>::kSmem;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = static_cast<unsigned>(k);
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    int n = 0;
    const cudaError_t e = cudaOccupancyMaxActiveClusters(&n, tc_gemm_kernel<BN, true, false>, &cfg);
    if (e != cudaSuccess) {
        (void)cudaGetLastError();
        return false;
    }
    return n > 0;
}


// ------------------------------------------------ 2-SM pairs (cta_group::2)
//
// Normal mode, whole-K tiles of 256 X rows x BN W rows computed by a cluster
// of two CTAs on two SMs with tcgen05.mma.cta_group::2 (M = 256).  CTA r of
// the pair holds X rows [256 mt + 128 r, +128) and W rows [BN nt + BN/2 r,
// +BN/2) in its shared memory; the MMA, issued by CTA 0 alone, reads both
// CTAs' halves and leaves rows 128 r .. of the 256 x BN product in CTA r's
// tensor memory.  Per k-block each CTA loads 16 KB of X and BN/2 x 128 B of W
// (32 KB at BN = 256) instead of 48 KB, so six ring stages fit where the
// one-SM kernel has four, and every W byte crosses L2 -> SM once per pair.
//
// Both CTAs' copies are counted on CTA 0's `full` barrier (the copy's
// mbarrier operand is CTA 0's, addressed through mapa); CTA 0's commits
// arrive on both CTAs' `empty`, `tfull` and `drain` barriers (multicast to
// the pair).  CTA 1's epilogue tells CTA 0's `tempty` by one remote arrival
// after its 128 threads are done with the accumulator.  Copies use the
// cta_group::2 form of the tensor copy; none broadcasts to several CTAs.
// Every wait is bounded; the two hardware cluster barriers (after set-up,
// before TMEM is freed) are reached by every thread unconditionally.

template <int BN>
struct PairCfg {
    static constexpr int kABytes = kBM * kBK * 2;         // 128 X rows
    static constexpr int kBBytes = (BN / 2) * kBK * 2;    // BN / 2 W rows
    static constexpr int kStageBytes = kABytes + kBBytes;
    static constexpr int kStages = (200 * 1024) / kStageBytes > 12 ? 12 : (200 * 1024) / kStageBytes;
    static constexpr uint32_t kTmemCols = 2 * BN <= 256 ? 256 : 512;
    // full[S], empty[S], tfull[2], tempty[2], drain; TMEM slot.
    static constexpr int kBarBytes = (2 * kStages + 5) * 8 + 16;
    static constexpr size_t kSmem = static_cast<size_t>(kStages) * kStageBytes + kBarBytes + 1024;
};

__device__ __forceinline__ void tmem_alloc_pair(uint32_t* dst_smem, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst_smem)),
                 "r"(ncols)
                 : "memory");
}

__device__ __forceinline__ void tmem_relinquish_pair() {
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_dealloc_pair(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}

__device__ __forceinline__ void tc_mma_f16_pair(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                                uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
}

// Arrive once on `bar` in both CTAs of the pair when every tcgen05 operation
// this thread issued so far has completed.
__device__ __forceinline__ void tc_commit_pair(uint64_t* bar) {
    const uint16_t both = 3;
    asm volatile(
        "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;" ::"r"(
            smem_u32(bar)),
        "h"(both)
        : "memory");
}

// 2-D tensor copy into this CTA's shared memory whose completion is counted
// on the mbarrier at shared::cluster address `bar_cluster` (CTA 0's barrier).
__device__ __forceinline__ void tma_load_2d_pair(void* smem_dst, const void* tmap, uint32_t bar_cluster, int32_t c0,
                                                 int32_t c1) {
    asm volatile(
        "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%2, %3}], [%4];" ::"r"(smem_u32(smem_dst)),
        "l"(reinterpret_cast<uint64_t>(tmap)), "r"(c0), "r"(c1), "r"(bar_cluster)
        : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx_local(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes) : "memory");
}

// tma: X map (box 64 x 128 rows, 128-byte swizzle); tmw: the tiled weight as
// rows of 64 (box 64 x 128, no swizzle: each box is one pre-swizzled tile).
template <int BN, bool SEG>
__global__ void __launch_bounds__(threads_of<SEG>(), 1)
    tc_pair_kernel(const TcGemmArgs a, const __grid_constant__ CUtensorMap tma, const __grid_constant__ CUtensorMap tmw) {
    using Cfg = PairCfg<BN>;
    constexpr int S = Cfg::kStages;
    constexpr int kEpi = SEG ? 256 : kEpiThreads;               // epilogue threads per CTA
    const int kSegLen = SEG ? max(1, a.seg_kb) : (1 << 30);     // k-blocks per accumulator segment
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* sA = smem;
    uint8_t* sB = smem + S * Cfg::kABytes;
    uint64_t* bars = reinterpret_cast<uint64_t*>(sB + S * Cfg::kBBytes);
    uint64_t* full = bars;
    uint64_t* empty = bars + S;
    uint64_t* tfull = bars + 2 * S;
    uint64_t* tempty = tfull + 2;
    uint64_t* drain = tempty + 2;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const uint32_t rank = cluster_rank();
    const bool leader = rank == 0;

    if (threadIdx.x == 0) {
        for (int s = 0; s < S; ++s) {
            mbar_init(&full[s], 1);   // CTA 0: its producer's arrive.expect_tx (+ both CTAs' bytes)
            mbar_init(&empty[s], 1);  // one multicast commit
        }
        for (int i = 0; i < 2; ++i) {
            mbar_init(&tfull[i], 1);
            mbar_init(&tempty[i], kEpi + 1);  // CTA 0: its epilogue threads + CTA 1's one arrival
        }
        mbar_init(drain, 1);
        fence_barrier_init();
    }
    if (warp == 1) {
        tmem_alloc_pair(tmem_slot, Cfg::kTmemCols);
        tmem_relinquish_pair();
    }
    if (warp == 0 && lane == 0) {
        prefetch_tmap(&tma);
        prefetch_tmap(&tmw);
    }
    griddep_launch_dependents();
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    // Both CTAs' barriers are initialised before anything addresses the other's.
    cluster_arrive();
    cluster_wait();
    const uint32_t tmem_base = *tmem_slot;

    // Units as in the one-SM kernel (decode_unit with 256-row m-tiles):
    // whole-K tiles, then the K-slices of the tail tiles.
    const int num_m2 = (a.M + 2 * kBM - 1) / (2 * kBM);
    const int num_n = (a.N + BN - 1) / BN;
    const int n_tail = num_m2 * num_n - a.full_tiles;
    const int total = a.full_tiles + n_tail * a.tail_splits;
    const int pair = blockIdx.x >> 1;
    const int npairs = gridDim.x >> 1;
    const int num_kb = (a.K + kBK - 1) / kBK;

    if (warp == 0) {
        if (lane == 0) {
            const uint32_t full0 = cluster_map(smem_u32(full), 0);  // CTA 0's full[0]
            int stage = 0;
            uint32_t phase = 0;
            uint32_t issued = 0, issued_parity = 0;
            bool ok = true;
            auto load_w = [&](const Unit& w, int kb, int st) {
                // this CTA's BN / 2 W rows = BN / 256 whole 128-row tiles (BN = 256: one)
                const int64_t wtile = (static_cast<int64_t>(w.nt) * BN + rank * (BN / 2)) / kBM;
#pragma unroll
                for (int h = 0; h < BN / 256; ++h)
                    tma_load_2d_pair(sB + st * Cfg::kBBytes + h * (kBM * kBK * 2), &tmw, full0 + st * 8, 0,
                                     static_cast<int32_t>(((wtile + h) * a.w_k_tiles + kb) * kBM));
            };
            auto load_x = [&](const Unit& w, int kb, int st) {
                tma_load_2d_pair(sA + st * Cfg::kABytes, &tma, full0 + st * 8, kb * kBK,
                                 w.mt * 2 * kBM + static_cast<int>(rank) * kBM);
            };
            auto claim = [&](int st) {
                if (leader) mbar_arrive_expect_tx_local(&full[st], 2 * Cfg::kStageBytes);
                issued |= 1u << st;
                issued_parity = (issued_parity & ~(1u << st)) | (phase << st);
            };
            // Next k-block of this pair's unit sequence.
            auto advance = [&](int& uu, Unit& ww, int& kk) {
                if (++kk == ww.kb1) {
                    uu += npairs;
                    if (uu < total) ww = decode_unit(a, uu, num_m2, n_tail, num_kb);
                    kk = ww.kb0;
                }
            };
            int u = pair;
            Unit w = decode_unit(a, u, num_m2, n_tail, num_kb);
            int kb = w.kb0;
            // First ring pass of weight tiles before waiting for the kernel
            // this one overlaps (weights are never written by it).
            int pre = 0;
            if (a.w_prefetch) {
                int uu = u, kk = kb;
                Unit ww = w;
                for (; pre < S && uu < total; ++pre) {
                    claim(stage);
                    load_w(ww, kk, stage);
                    advance(uu, ww, kk);
                    if (++stage == S) {
                        stage = 0;
                        phase ^= 1u;
                    }
                }
            }
            griddep_wait();
            for (int i = 0; i < pre; ++i) {
                load_x(w, kb, i);
                advance(u, w, kb);
            }
            for (; u < total;) {
                if (!mbar_wait(&empty[stage], phase ^ 1u, a.err_flag, kErrTmaWait)) {
                    ok = false;
                    break;
                }
                claim(stage);
                load_w(w, kb, stage);
                load_x(w, kb, stage);
                if (++stage == S) {
                    stage = 0;
                    phase ^= 1u;
                }
                advance(u, w, kb);
            }
            if (!ok) {
                // Copies still in flight land in this CTA's shared memory: wait
                // (bounded) for the stages this thread filled last.
                for (int s2 = 0; s2 < S; ++s2)
                    if ((issued & (1u << s2)) && leader) mbar_wait(&full[s2], (issued_parity >> s2) & 1u, nullptr, kErrDrainWait);
            }
        }
    } else if (warp == 1) {
        griddep_wait();
        if (lane == 0) {
            if (leader) {
                const uint32_t idesc = idesc_f16_f32(2 * kBM, BN);
                int stage = 0;
                uint32_t phase = 0;
                int acc = 0;
                uint32_t acc_phase = 0;
                bool ok = true;
                for (int u = pair; u < total && ok; u += npairs) {
                    const Unit w = decode_unit(a, u, num_m2, n_tail, num_kb);
                    for (int s0 = w.kb0; s0 < w.kb1 && ok; s0 += kSegLen) {
                        const int s1 = min(s0 + kSegLen, w.kb1);
                        if (!mbar_wait(&tempty[acc], acc_phase ^ 1u, a.err_flag, kErrMmaWait)) {
                            ok = false;
                            break;
                        }
                        tc_fence_after();
                        const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(acc * BN);
                        for (int kb = s0; kb < s1; ++kb) {
                            if (!mbar_wait(&full[stage], phase, a.err_flag, kErrMmaWait)) {
                                ok = false;
                                break;
                            }
                            tc_fence_after();
                            const uint32_t a_addr = smem_u32(sA + stage * Cfg::kABytes);
                            const uint32_t b_addr = smem_u32(sB + stage * Cfg::kBBytes);
#pragma unroll
                            for (int k = 0; k < kBK / 16; ++k)
                                tc_mma_f16_pair(d_tmem, smem_desc_k128(a_addr + k * 32), smem_desc_k128(b_addr + k * 32),
                                                idesc, (kb > s0 || k > 0) ? 1u : 0u);
                            tc_commit_pair(&empty[stage]);
                            if (++stage == S) {
                                stage = 0;
                                phase ^= 1u;
                            }
                        }
                        if (!ok) break;
                        tc_commit_pair(&tfull[acc]);
                        acc ^= 1;
                        if (acc == 0) acc_phase ^= 1u;
                    }
                }
                // Both CTAs learn when every MMA (reading both CTAs' shared
                // memory, writing both CTAs' TMEM) has completed.
                tc_commit_pair(drain);
            }
            mbar_wait(drain, 0, nullptr, kErrDrainWait);
        }
    } else if constexpr (SEG) {
        // As the one-SM kernel's segmented epilogue: 8 warps, warp w reads
        // TMEM lanes 32 (w mod 4) .. +31 and half the columns, keeps running
        // sums of the segments in FP32 registers (round to nearest), writes
        // the last segment's sums back and stores from there.
        constexpr int HB = BN / 2;
        const int quad = warp & 3;
        const int half = (warp - 2) >> 2;
        const int et = threadIdx.x - 64;
        griddep_wait();
        int acc = 0;
        uint32_t acc_phase = 0;
        bool go = true;
        for (int u = pair; u < total && go; u += npairs) {
            const Unit w = decode_unit(a, u, num_m2, n_tail, num_kb);
            float sum[HB];
            uint32_t t_row = 0;
            for (int s0 = w.kb0; s0 < w.kb1; s0 += kSegLen) {
                int ok = 1;
                if (lane == 0) ok = mbar_wait(&tfull[acc], acc_phase, a.err_flag, kErrEpiWait) ? 1 : 0;
                ok = __shfl_sync(0xFFFFFFFFu, ok, 0);
                if (!epi_bar_and_n<kEpi>(ok != 0)) {
                    go = false;
                    break;
                }
                tc_fence_after();
                t_row = tmem_base + (static_cast<uint32_t>(quad * 32) << 16) + static_cast<uint32_t>(acc * BN + half * HB);
                const bool last = s0 + kSegLen >= w.kb1;
                const bool first = s0 == w.kb0;
#pragma unroll
                for (int c = 0; c < HB / 16; ++c) {
                    uint32_t r[16];
                    __syncwarp();
                    tmem_ld_16cols(t_row + c * 16, r);
#pragma unroll
                    for (int j = 0; j < 16; ++j)
                        sum[c * 16 + j] = first ? __uint_as_float(r[j]) : __fadd_rn(sum[c * 16 + j], __uint_as_float(r[j]));
                    if (last) {
#pragma unroll
                        for (int j = 0; j < 16; ++j) r[j] = __float_as_uint(sum[c * 16 + j]);
                        tmem_st_16cols(t_row + c * 16, r);
                    }
                }
                if (last) break;  // the accumulator stays owned until the stores below
                tc_fence_before();
                if (leader) {
                    mbar_arrive(&tempty[acc]);
                } else {
                    epi_bar_sync_n<kEpi>();
                    if (et == 0) mbar_arrive_cluster(&tempty[acc], 0);
                }
                acc ^= 1;
                if (acc == 0) acc_phase ^= 1u;
            }
            if (!go) break;
            const int row_in_tile = static_cast<int>(rank) * kBM + quad * 32 + lane;
            const int64_t row = static_cast<int64_t>(w.mt) * 2 * kBM + row_in_tile;
#pragma unroll 1
            for (int c = 0; c < HB / 32; ++c) {
                uint32_t r[32];
                __syncwarp();
                tmem_ld_32cols(t_row + c * 32, r);
                const int64_t col0 = static_cast<int64_t>(w.nt) * BN + half * HB + c * 32;
                if (w.slot >= 0) {
                    store_partial_chunk(a, r, w.slot, row_in_tile, half * HB + c * 32, BN, 2 * kBM);
                } else if (row < a.M && col0 < a.N) {
                    if (a.swiglu_lut != nullptr)
                        store_row_chunk_swiglu(a, r, row, col0);
                    else
                        store_row_chunk(a, r, row, col0);
                }
            }
            tc_fence_before();
            if (leader) {
                mbar_arrive(&tempty[acc]);
            } else {
                epi_bar_sync_n<kEpi>();
                if (et == 0) mbar_arrive_cluster(&tempty[acc], 0);
            }
            acc ^= 1;
            if (acc == 0) acc_phase ^= 1u;
        }
    } else {
        const int quad = warp & 3;
        const int et = threadIdx.x - 64;
        griddep_wait();
        int acc = 0;
        uint32_t acc_phase = 0;
        for (int u = pair; u < total; u += npairs) {
            const Unit w = decode_unit(a, u, num_m2, n_tail, num_kb);
            int ok = 1;
            if (lane == 0) ok = mbar_wait(&tfull[acc], acc_phase, a.err_flag, kErrEpiWait) ? 1 : 0;
            ok = __shfl_sync(0xFFFFFFFFu, ok, 0);
            // The four warps leave together (the named barrier below needs all 128).
            if (!epi_bar_and(ok != 0)) break;
            tc_fence_after();
            const int row_in_tile = static_cast<int>(rank) * kBM + quad * 32 + lane;
            const int64_t row = static_cast<int64_t>(w.mt) * 2 * kBM + row_in_tile;
            const uint32_t t_row = tmem_base + (static_cast<uint32_t>(quad * 32) << 16) + static_cast<uint32_t>(acc * BN);
#pragma unroll 1
            for (int c = 0; c < BN / 32; ++c) {
                uint32_t r[32];
                __syncwarp();
                tmem_ld_32cols(t_row + c * 32, r);
                const int64_t col0 = static_cast<int64_t>(w.nt) * BN + c * 32;
                if (w.slot >= 0) {
                    store_partial_chunk(a, r, w.slot, row_in_tile, c * 32, BN, 2 * kBM);
                } else if (row < a.M && col0 < a.N) {
                    if (a.swiglu_lut != nullptr)
                        store_row_chunk_swiglu(a, r, row, col0);
                    else
                        store_row_chunk(a, r, row, col0);
                }
            }
            tc_fence_before();
            if (leader) {
                mbar_arrive(&tempty[acc]);
            } else {
                epi_bar_sync();  // this CTA's 128 threads are done with the accumulator
                if (et == 0) mbar_arrive_cluster(&tempty[acc], 0);
            }
            acc ^= 1;
            if (acc == 0) acc_phase ^= 1u;
        }
    }

    tc_fence_before();
    __syncthreads();
    // The other CTA is done too (its remote arrivals and its MMA operands).
    cluster_arrive();
    cluster_wait();
    if (warp == 1) {
        __syncwarp();
        tc_fence_after();
        tmem_dealloc_pair(tmem_base, Cfg::kTmemCols);
    }
}

template <int BN, bool SEG>
cudaError_t launch_pair_bn(const TcGemmArgs& a, const CUtensorMap& tx, const CUtensorMap& tw, cudaStream_t s) {
    static bool attr_set[64] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
    if (!attr_set[dev]) {
        cudaError_t e = cudaFuncSetAttribute(tc_pair_kernel<BN, SEG>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             static_cast<int>(PairCfg<BN>::kSmem));
        if (e != cudaSuccess) return e;
        attr_set[dev] = true;
    }
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(static_cast<unsigned>(a.grid));
    cfg.blockDim = dim3(threads_of<SEG>());
    cfg.dynamicSmemBytes = PairCfg<BN>::kSmem;
    cfg.stream = s;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    attr[1].id = cudaLaunchAttributeClusterDimension;
    attr[1].val.clusterDim.x = 2;
    attr[1].val.clusterDim.y = 1;
    attr[1].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 2;
    cudaError_t e = cudaLaunchKernelEx(&cfg, tc_pair_kernel<BN, SEG>, a, tx, tw);
    if (e != cudaSuccess) return e;
    note_launches(1);
    return cudaGetLastError();
}

}  // namespace

bool tc_cluster_ok(int bn, int k) {
    if (k < 2 || k > 8) return false;
    const int slot = bn == 16 ? 0 : (bn == 32 ? 1 : (bn == 64 ? 2 : -1));
    if (slot < 0) return false;
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return false;
    // 0 unknown, 1 no, 2 yes
    static signed char known[64][3][9] = {};
    signed char& v = known[dev][slot][k];
    if (v == 0) {
        const bool ok = slot == 0 ? cluster_fits<16>(k) : (slot == 1 ? cluster_fits<32>(k) : cluster_fits<64>(k));
        v = ok ? 2 : 1;
    }
    return v == 2;
}

bool tc_gemm_segmented(const TcGemmArgs& a) {
    if (a.swap) return false;
    const int num_kb = (a.K + kBK - 1) / kBK;
    const bool long_full = a.full_tiles > 0 && num_kb > kSegMinKb;
    const bool long_tail = a.full_tiles < tc_gemm_tiles(a) && a.kb_per > kSegMinKb;
    return long_full || long_tail;
}

cudaError_t launch_tc_pair(const TcGemmArgs& a, const CUtensorMap& tmap_x, const CUtensorMap& tmap_w_rows,
                           cudaStream_t s) {
    if (a.M <= 0 || a.N <= 0) return cudaSuccess;
    // Tiles of 256 x BN, an even persistent grid of at most one pair per
    // unit, FP16 or FP32 output (no greedy-pick partials); every tail slice
    // owns at least one k-block and stores into `partials`.
    if (!a.pair || a.swap || a.K <= 0 || a.w_tiled == nullptr || a.grid < 2 || (a.grid & 1) != 0 ||
        a.tail_splits <= 0 || a.am_val != nullptr || a.cluster_k != 0)
        return cudaErrorInvalidValue;
    const int tiles = tc_gemm_tiles(a);
    const int num_kb = (a.K + kBK - 1) / kBK;
    if (a.full_tiles < 0 || a.full_tiles > tiles) return cudaErrorInvalidValue;
    const bool tail = a.full_tiles < tiles;
    if (tail && (a.kb_per <= 0 || (a.tail_splits - 1) * a.kb_per >= num_kb || a.tail_splits * a.kb_per < num_kb ||
                 a.partials == nullptr || a.swiglu_lut != nullptr))
        return cudaErrorInvalidValue;
    const int64_t units = a.full_tiles + static_cast<int64_t>(tiles - a.full_tiles) * (tail ? a.tail_splits : 0);
    if (a.grid > 2 * units) return cudaErrorInvalidValue;
    const bool seg = (a.full_tiles > 0 && num_kb > kSegMinKb) || (tail && a.kb_per > kSegMinKb);
    if (a.bn == 256) return seg ? launch_pair_bn<256, true>(a, tmap_x, tmap_w_rows, s)
                                : launch_pair_bn<256, false>(a, tmap_x, tmap_w_rows, s);
    return cudaErrorInvalidValue;
}

int tc_gemm_tiles(const TcGemmArgs& a) {
    if (a.pair) return ((a.M + 2 * kBM - 1) / (2 * kBM)) * ((a.N + a.bn - 1) / a.bn);
    return a.swap ? ((a.N + kBM - 1) / kBM) * ((a.M + a.bn - 1) / a.bn)
                  : ((a.M + kBM - 1) / kBM) * ((a.N + a.bn - 1) / a.bn);
}

// tmap_x must have a box of 128 rows (normal mode) or bn rows (swap mode);
// tmap_w the other one.
cudaError_t launch_tc_gemm(const TcGemmArgs& a, const CUtensorMap& tmap_x, const CUtensorMap& tmap_w,
                           cudaStream_t s) {
    if (a.M <= 0 || a.N <= 0) return cudaSuccess;
    const int tiles = tc_gemm_tiles(a);
    const int num_kb = (a.K + kBK - 1) / kBK;
    if (a.K <= 0 || a.grid <= 0 || a.tail_splits <= 0 || a.full_tiles < 0 || a.full_tiles > tiles)
        return cudaErrorInvalidValue;
    // Every tail slice must own at least one k-block, or its accumulator
    // would never be written.
    const bool clustered = a.cluster_k > 1;
    if (a.full_tiles < tiles && (a.kb_per <= 0 || (a.tail_splits - 1) * a.kb_per >= num_kb ||
                                 a.tail_splits * a.kb_per < num_kb ||
                                 (!clustered && (a.partials == nullptr || (a.swap && a.tile_counters == nullptr)))))
        return cudaErrorInvalidValue;
    // SwiGLU pairs: whole-K tiles only, even N, FP16 output, no bias.
    if (a.swiglu_lut != nullptr && (a.full_tiles != tiles || (a.N & 1) != 0 || a.out_f32 || a.bias != nullptr))
        return cudaErrorInvalidValue;
    // Clusters: swap mode, every tile split, one slice per CTA.
    if (clustered && (!a.swap || a.cluster_k > 8 || a.full_tiles != 0 || a.tail_splits != a.cluster_k ||
                      static_cast<int64_t>(a.grid) != static_cast<int64_t>(tiles) * a.cluster_k))
        return cudaErrorInvalidValue;
    if (a.swap) {
        if (a.M > a.bn) return cudaErrorInvalidValue;  // one token tile
        if (a.bn == 16) return launch_bn<16, true>(a, tmap_w, tmap_x, s);
        if (a.bn == 32) return launch_bn<32, true>(a, tmap_w, tmap_x, s);
        if (a.bn == 64) return launch_bn<64, true>(a, tmap_w, tmap_x, s);
        return cudaErrorInvalidValue;
    }
    if (tc_gemm_segmented(a)) {
        if (a.bn == 256) return launch_bn<256, false, true>(a, tmap_x, tmap_w, s);
        if (a.bn == 128) return launch_bn<128, false, true>(a, tmap_x, tmap_w, s);
        if (a.bn == 64) return launch_bn<64, false, true>(a, tmap_x, tmap_w, s);
        return cudaErrorInvalidValue;
    }
    if (a.bn == 256) return launch_bn<256, false>(a, tmap_x, tmap_w, s);
    if (a.bn == 128) return launch_bn<128, false>(a, tmap_x, tmap_w, s);
    if (a.bn == 64) return launch_bn<64, false>(a, tmap_x, tmap_w, s);
    return cudaErrorInvalidValue;
}

}  // namespace mrt
