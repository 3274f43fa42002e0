// decode_step.cu -- one persistent kernel per greedy decode step.
//
// A decode step of a Qwen2-shaped decoder (qwen_model.cpp:104-376 for one
// token, then inference_engine.cpp:84-95's greedy pick) streams every weight
// once and does very little arithmetic per byte, so it is bound by HBM; what
// separate kernels lose is the time between them, when nothing streams.  Here
// one CTA per SM runs the whole step:
//
//   warp 0      producer: one lane walks this CTA's share of every weight of
//               every layer (fixed row ranges of the tiled weights) and copies
//               it into a ring of 16 KB shared-memory stages with linear bulk
//               copies (L2 evict-first).  It never waits for activations, so
//               the next phase's weights are already arriving while the
//               consumers are at a grid barrier or in attention.
//   warps 1-8   consumers: GEMV over each stage (FP32 FMA; thread
//               (row slot, 8-column chunk), rows summed across the eight
//               chunk lanes in a fixed tree, so results do not depend on
//               timing), then the phase's epilogue.
//
// Phases of a layer, separated by grid barriers (B):
//   qkv GEMV (+ bias, double rounding) B RoPE + KV append + attention B
//   o GEMV B residual add + RMSNorm (every CTA, into its operand buffer)
//   gate|up GEMV + SiLU*up B down GEMV B residual add + RMSNorm (next layer).
// After the last layer: lm_head GEMV, per-CTA greedy candidates B the pick and
// the state update (position, step, token) by CTA 0.
//
// Every wait is bounded: a grid barrier or a ring wait that gives up raises
// the device error flag, and every other wait then returns at once, so a
// failing step ends instead of hanging.  TMA/bulk loads never use cluster
// broadcast and every operand is this GPU's memory.
#include <algorithm>
#include <cstdio>

#include "common.cuh"
#include "decode_step.h"
#include "kernels.h"
#include "mrt_b200.h"

namespace mrt {
namespace {

constexpr int kStepCons = 512;                   // consumer threads (warps 1-16)
constexpr int kStepThreads = 32 + kStepCons;
constexpr int kRingStages = 10;
constexpr int kStage = 16384;                    // bytes per ring stage
constexpr int kRowsPerChunk = 128;               // rows a stage may hold
constexpr int kAttWarps = kStepCons / 32;
constexpr int kAttKeys = 4;                      // keys per warp per round

__device__ __forceinline__ void cons_sync() { asm volatile("bar.sync 1, 512;" ::: "memory"); }

__device__ __forceinline__ unsigned ld_acquire_gpu_u32(const unsigned* p) {
    unsigned v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

__device__ __forceinline__ unsigned long long now_ns() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ uint32_t pk2(uint16_t lo, uint16_t hi) {
    return static_cast<uint32_t>(lo) | (static_cast<uint32_t>(hi) << 16);
}

__device__ __forceinline__ void unpack8h(const uint4& v, float (&x)[8]) {
    const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int e = 0; e < 4; ++e) {
        x[2 * e] = f16_bits_to_f32(static_cast<uint16_t>(w[e] & 0xFFFFu));
        x[2 * e + 1] = f16_bits_to_f32(static_cast<uint16_t>(w[e] >> 16));
    }
}

__device__ __forceinline__ float gain(const void* w, int dt, int64_t i) {
    if (dt == MRT_FP32) return static_cast<const float*>(w)[i];
    const uint16_t v = static_cast<const uint16_t*>(w)[i];
    return dt == MRT_BF16 ? bf16_bits_to_f32(v) : f16_bits_to_f32(v);
}


// Grid barrier of the consumer threads of every CTA (the producer warps keep
// streaming).  a.bar[0] counts arrivals (zero at each launch); barrier n is
// complete when it reaches n * gridDim.x.  Returns false once the kernel is
// aborting.
__device__ bool grid_sync(const StepArgs& a, unsigned& nbar, int ct, volatile int* ok_sh) {
    cons_sync();
    ++nbar;
    if (ct == 0) {
        int ok = 1;
        // Arrive without waiting for an answer (the release covers this
        // CTA's writes, ordered before it by the barrier above), then spin on
        // the counter itself; the error flag and the clock are checked every
        // 256 polls only.
        asm volatile("red.release.gpu.global.add.u32 [%0], 1;" ::"l"(a.bar) : "memory");
        const unsigned target = nbar * gridDim.x;
        const unsigned long long t0 = now_ns();
        for (unsigned it = 1; ld_acquire_gpu_u32(a.bar) < target; ++it) {
            if ((it & 255u) == 0) {
                if (error_raised(a.err)) {
                    ok = 0;
                    break;
                }
                if (now_ns() - t0 > kWaitLimitNs) {
                    raise_error(a.err, kErrEpiWait);
                    ok = 0;
                    break;
                }
            }
        }
        *ok_sh = ok;
    }
    cons_sync();
    return *ok_sh != 0;
}

// One GEMV of the step as this CTA sees it: its rows of a tiled weight, in at
// most two global row ranges (gate and up rows for the fused gate|up weight).
struct Gemv {
    const uint16_t* w;
    int64_t kt;          // k-tiles (64 columns each)
    int64_t a0, a1, b0, b1;
    // Split mode: units u = tile * kt + k-tile (128-row tile, 64-column
    // k-tile) in [u0, u1), i.e. whole 16 KB tiles read front to back; the CTA
    // leaves FP32 partial sums per tile it touches (at most two).
    int split;
    int64_t u0, u1, units;
};



__device__ __forceinline__ int64_t gemv_rows(const Gemv& g) { return (g.a1 - g.a0) + (g.b1 - g.b0); }

__device__ __forceinline__ int64_t gemv_grow(const Gemv& g, int64_t i) {
    const int64_t la = g.a1 - g.a0;
    return i < la ? g.a0 + i : g.b0 + (i - la);
}

// Stages of a GEMV: CTA rows in chunks of <= 128 (chunk-major); within a
// chunk, groups of T k-tiles so that a stage holds <= 16 KB.
struct StageGeo {
    int64_t rows, chunks, T, kgroups;
};

__device__ __forceinline__ StageGeo stage_geo(const Gemv& g) {
    StageGeo s;
    s.rows = gemv_rows(g);
    s.chunks = (s.rows + kRowsPerChunk - 1) / kRowsPerChunk;
    const int64_t crow = s.rows < kRowsPerChunk ? s.rows : kRowsPerChunk;
    s.T = crow > 0 ? kRowsPerChunk / crow : 1;
    if (s.T < 1) s.T = 1;
    s.kgroups = (g.kt + s.T - 1) / s.T;
    return s;
}

// Visit the contiguous pieces of CTA rows [i0, i1) for one k-tile: f(first
// CTA row, end CTA row, first global row).  A piece stays inside one range
// and one 128-row tile, so its rows are consecutive 128-byte rows in memory.
template <typename F>
__device__ __forceinline__ void for_pieces(const Gemv& g, int64_t i0, int64_t i1, F f) {
    const int64_t la = g.a1 - g.a0;
    int64_t i = i0;
    while (i < i1) {
        const int64_t gr = gemv_grow(g, i);
        int64_t e = i1;
        if (i < la && e > la) e = la;
        const int64_t tile_end = (gr / 128 + 1) * 128;
        if (gr + (e - i) > tile_end) e = i + (tile_end - gr);
        f(i, e, gr);
        i = e;
    }
}

// This CTA's rows [n * c / G, n * (c + 1) / G) of an n-row output.
__device__ __forceinline__ void my_rows(int64_t n, int64_t* r0, int64_t* r1) {
    *r0 = n * blockIdx.x / gridDim.x;
    *r1 = n * (blockIdx.x + 1) / gridDim.x;
}

// Units of a split GEMV for this CTA: [U * c / G, U * (c + 1) / G).
__device__ __forceinline__ Gemv split_gemv(const uint16_t* w, int64_t n, int64_t k) {
    Gemv g{};
    g.w = w;
    g.kt = (k + 63) / 64;
    g.split = 1;
    g.units = ((n + 127) / 128) * g.kt;
    g.u0 = g.units * blockIdx.x / gridDim.x;
    g.u1 = g.units * (blockIdx.x + 1) / gridDim.x;
    return g;
}

__device__ __forceinline__ Gemv gemv_of(const StepArgs& a, int l, int which) {
    Gemv g{};
    int64_t r0, r1;
    if (l == a.L) {  // lm_head
        my_rows(a.V, &r0, &r1);
        g = Gemv{a.lm, (a.H + 63) / 64, r0, r1, 0, 0};
        return g;
    }
    const StepLayer& ly = a.layers[l];
    switch (which) {
        case 0:  // q|k|v
            my_rows(a.n_qkv, &r0, &r1);
            g = Gemv{ly.qkv, (a.H + 63) / 64, r0, r1, 0, 0};
            break;
        case 1:  // o
            my_rows(a.H, &r0, &r1);
            g = Gemv{ly.o, (a.nh * a.D + 63) / 64, r0, r1, 0, 0};
            break;
        case 2:  // gate | up, rows interleaved (2j gate j, 2j + 1 up j): one range
            my_rows(a.I, &r0, &r1);
            g = Gemv{ly.gu, (a.H + 63) / 64, 2 * r0, 2 * r1, 0, 0};
            break;
        default:  // down, split along K: whole tiles, contiguous per CTA
            g = split_gemv(ly.down, a.H, a.I);
            break;
    }
    return g;
}

// Element offset of the start of global row gr's 64 columns of k-tile kt in
// the tiled layout (rows of one tile are consecutive 128-byte rows).
__device__ __forceinline__ int64_t tile_row_start(int64_t gr, int64_t kt, int64_t k_tiles) {
    return (((gr >> 7) * k_tiles + kt) << 13) + ((gr & 127) << 6);
}

// The producer lane: every GEMV of the step, layer by layer, in the order the
// consumers use them.  A chunk's rows split into at most four pieces (two row
// ranges, each crossing at most one 128-row tile boundary) whose layout is
// the same in every k-tile, so they are worked out once per chunk and each
// stage is only address arithmetic and bulk copies.  Stops (after its copies
// in flight land) when a wait for a free stage gives up.
__device__ void produce(const StepArgs& a, uint8_t* ring, uint64_t* full, uint64_t* empty) {
    int stage = 0;
    uint32_t phase = 0, issued = 0, issued_par = 0;
    bool ok = true;
    const uint64_t pol = l2_policy_evict_first();
    for (int l = 0; l <= a.L && ok; ++l) {
        const int nw = l == a.L ? 1 : 4;
        for (int which = 0; which < nw && ok; ++which) {
            const Gemv g = gemv_of(a, l, which);
            if (g.split) {
                // Whole tiles, one per stage: unit u is the 16 KB at element u * 8192.
                for (int64_t u = g.u0; u < g.u1; ++u) {
                    if (!mbar_wait(&empty[stage], phase ^ 1u, a.err, kErrTmaWait)) {
                        ok = false;
                        break;
                    }
                    mbar_arrive_expect_tx(&full[stage], kStage);
                    bulk_load_hint(ring + static_cast<int64_t>(stage) * kStage, g.w + (u << 13), kStage, &full[stage], pol);
                    issued |= 1u << stage;
                    issued_par = (issued_par & ~(1u << stage)) | (phase << stage);
                    if (++stage == kRingStages) {
                        stage = 0;
                        phase ^= 1u;
                    }
                }
                continue;
            }
            const StageGeo geo = stage_geo(g);
            for (int64_t ch = 0; ch < geo.chunks && ok; ++ch) {
                const int64_t cr0 = ch * kRowsPerChunk;
                const int64_t cr1 = cr0 + kRowsPerChunk < geo.rows ? cr0 + kRowsPerChunk : geo.rows;
                const uint32_t rows_bytes = static_cast<uint32_t>((cr1 - cr0) * 128);
                int np = 0;
                uint32_t p_off[4], p_bytes[4];
                const uint16_t* p_src[4];
                for_pieces(g, cr0, cr1, [&](int64_t i, int64_t e, int64_t gr) {
                    if (np < 4) {
                        p_off[np] = static_cast<uint32_t>((i - cr0) * 128);
                        p_bytes[np] = static_cast<uint32_t>((e - i) * 128);
                        p_src[np] = g.w + tile_row_start(gr, 0, g.kt);
                    }
                    ++np;
                });
                if (np > 4) {  // cannot happen for rows split as my_rows does; never copy a partial stage
                    raise_error(a.err, kErrTmaWait);
                    ok = false;
                    break;
                }
                for (int64_t kg = 0; kg < geo.kgroups; ++kg) {
                    if (!mbar_wait(&empty[stage], phase ^ 1u, a.err, kErrTmaWait)) {
                        ok = false;
                        break;
                    }
                    const int64_t kt0 = kg * geo.T, kt1 = kt0 + geo.T < g.kt ? kt0 + geo.T : g.kt;
                    const int nkt = static_cast<int>(kt1 - kt0);
                    mbar_arrive_expect_tx(&full[stage], rows_bytes * static_cast<uint32_t>(nkt));
                    uint8_t* dst = ring + static_cast<int64_t>(stage) * kStage;
                    for (int t = 0; t < nkt; ++t) {
                        const int64_t koff = (kt0 + t) << 13;  // one k-tile = 8192 elements
                        for (int p = 0; p < np; ++p)
                            bulk_load_hint(dst + t * rows_bytes + p_off[p], p_src[p] + koff, p_bytes[p], &full[stage], pol);
                    }
                    issued |= 1u << stage;
                    issued_par = (issued_par & ~(1u << stage)) | (phase << stage);
                    if (++stage == kRingStages) {
                        stage = 0;
                        phase ^= 1u;
                    }
                }
            }
        }
    }
    if (!ok) {
        for (int st = 0; st < kRingStages; ++st)
            if (issued & (1u << st)) mbar_wait(&full[st], (issued_par >> st) & 1u, nullptr, kErrDrainWait);
    }
}

// Consumer side of one GEMV: the same stages as the producer.  The product
// runs on the tensor cores as m16n8k16 MMAs (FP16 in, FP32 accumulate) with
// the weights as A (16 rows x 16 columns per ldmatrix) and x as the only
// non-zero column of B, so no FP16->FP32 conversion passes through the
// shader pipes.  Warp w takes row block w % nrb (16 rows) of the current
// chunk and k-tiles w / nrb, w / nrb + G, ... of each stage (G = 16 / nrb
// k-groups); group sums are added in group order through shared memory
// (`red`, 256 floats), so the result never depends on timing.  The pieces of
// a stage are laid out in CTA-row order, one 128-byte row each: CTA row r of
// k-tile t of the stage sits at t * rows * 128 + (r - chunk start) * 128, its
// 16-byte chunks in the swizzled order of its global row.  Rows of a 16-row
// block past the chunk read whatever follows in the ring (never outside it:
// the operand buffer follows the ring) and are discarded.  out(cta_row, sum)
// is called once per row of each finished chunk.
constexpr int kConsWarps = kStepCons / 32;  // 16

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
                 : "r"(addr));
}

__device__ __forceinline__ void mma_16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                                          uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
        "{%0, %1, %2, %3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// Consumer side of a split GEMV: every stage is a whole 128 x 64 tile; warp w
// takes row block w % 8 and k-steps {0, 1} (w < 8) or {2, 3} (w >= 8) of it.
// When the unit range moves to the next tile (and at its end) the two k
// halves are added through `red` and the tile's 128 FP32 row sums go to
// part[blockIdx.x][segment][row] (segment 0 = first tile of the range).
__device__ __forceinline__ bool gemv_split(const Gemv& g, const uint16_t* xs, const uint8_t* ring, uint64_t* full,
                                           uint64_t* empty, int& stage, uint32_t& phase, int ct, int* err, float* red,
                                           float* part) {
    const int w = ct >> 5, lane = ct & 31;
    const int rb = w & 7, kh2 = w >> 3;
    const uint32_t ring_s = smem_u32(ring);
    const uint32_t xs_s = smem_u32(xs);
    const int rr = rb * 16 + (lane & 15);
    const int kh = lane >> 4;
    const int swz = rr & 7;
    float d[4] = {0.0f, 0.0f, 0.0f, 0.0f};
    int seg = 0;
    int64_t tile = g.u0 / g.kt;
    auto flush = [&]() {
        if ((lane & 3) == 0) {
            const int q = lane >> 2;
            red[kh2 * 128 + rb * 16 + q] = d[0];
            red[kh2 * 128 + rb * 16 + q + 8] = d[2];
        }
        cons_sync();
        // A range of at most kt units touches at most two tiles (the host keeps
        // the tiles no more than the CTAs); never write past the two slots.
        if (ct < 128 && seg < 2) part[(static_cast<int64_t>(blockIdx.x) * 2 + seg) * 128 + ct] = red[ct] + red[128 + ct];
        cons_sync();
        d[0] = d[1] = d[2] = d[3] = 0.0f;
    };
    for (int64_t u = g.u0; u < g.u1; ++u) {
        const int64_t t = u / g.kt, kt = u % g.kt;
        if (t != tile) {
            flush();
            ++seg;
            tile = t;
        }
        if (!mbar_wait(&full[stage], phase, err, kErrMmaWait)) return false;
        const uint32_t rowb = ring_s + static_cast<uint32_t>(stage) * kStage + static_cast<uint32_t>(rr) * 128;
#pragma unroll
        for (int j = 0; j < 2; ++j) {
            const int st4 = 2 * kh2 + j;
            uint32_t a0, a1, a2, a3;
            ldsm_x4(rowb + (((2 * st4 + kh) ^ swz) << 4), a0, a1, a2, a3);
            uint32_t b0 = 0, b1 = 0;
            if (lane < 4) {
                const uint32_t xa = xs_s + static_cast<uint32_t>((kt * 64 + st4 * 16 + 2 * lane) * 2);
                asm volatile("ld.shared.b32 %0, [%1];" : "=r"(b0) : "r"(xa));
                asm volatile("ld.shared.b32 %0, [%1];" : "=r"(b1) : "r"(xa + 16));
            }
            mma_16816(d, a0, a1, a2, a3, b0, b1);
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[stage]);
        if (++stage == kRingStages) {
            stage = 0;
            phase ^= 1u;
        }
    }
    if (g.u1 > g.u0) flush();
    return true;
}

// The CTAs that covered one 128-row tile of a split GEMV: c0 .. c1 in order;
// c0's partial of the tile is in its segment seg0 (1 when its range began in
// the tile before), every later CTA's in segment 0.  Units are < 2^31 / G, so
// 32-bit arithmetic is exact.
struct TileSrc {
    int c0, c1, seg0, units;
};

// Whether CTA c of the grid was given any unit of a split GEMV of `units`
// units (with fewer units than CTAs some get none and never write their
// partial slots, which are then not part of any tile's sum).
__device__ __forceinline__ bool cta_has_units(int c, int units) {
    const int G = static_cast<int>(gridDim.x);
    return units * (c + 1) / G > units * c / G;
}

__device__ __forceinline__ int unit_owner(int u, int units) {
    const int G = static_cast<int>(gridDim.x);
    int c = u * G / units;
    while (c + 1 < G && units * (c + 1) / G <= u) ++c;
    while (c > 0 && units * c / G > u) --c;
    return c;
}

__device__ __forceinline__ TileSrc tile_src(int64_t t, int64_t kt, int64_t units) {
    const int u = static_cast<int>(t * kt), U = static_cast<int>(units), G = static_cast<int>(gridDim.x);
    TileSrc s;
    s.c0 = unit_owner(u, U);
    s.c1 = unit_owner(u + static_cast<int>(kt) - 1, U);
    s.seg0 = (U * s.c0 / G) / static_cast<int>(kt) == static_cast<int>(t) ? 0 : 1;
    s.units = U;
    return s;
}

__device__ __forceinline__ const float* tile_part(const float* part, const TileSrc& s, int c) {
    return part + (c == s.c0 ? (static_cast<int64_t>(c) * 2 + s.seg0) * 128 : static_cast<int64_t>(c) * 256);
}

// Row r (0..127) of a tile: the CTAs' partials added in CTA order (loads of
// up to 8 CTAs issued together).
__device__ __forceinline__ float tile_sum(const float* part, const TileSrc& s, int r) {
    float v = 0.0f;
    for (int cb = s.c0; cb <= s.c1; cb += 8) {
        float p[8];
#pragma unroll
        for (int j = 0; j < 8; ++j)
            p[j] = cb + j <= s.c1 && cta_has_units(cb + j, s.units) ? __ldcg(tile_part(part, s, cb + j) + r) : 0.0f;
#pragma unroll
        for (int j = 0; j < 8; ++j)
            if (cb + j <= s.c1 && cta_has_units(cb + j, s.units)) v = cb + j == s.c0 ? p[j] : __fadd_rn(v, p[j]);
    }
    return v;
}

// Rows r0 .. r0 + 7 of a tile (r0 a multiple of 8), as tile_sum.
__device__ __forceinline__ void tile_sum8(const float* part, const TileSrc& s, int r0, float (&v)[8]) {
    for (int cb = s.c0; cb <= s.c1; cb += 8) {
        float4 p0[8], p1[8];
#pragma unroll
        for (int j = 0; j < 8; ++j)
            if (cb + j <= s.c1 && cta_has_units(cb + j, s.units)) {
                const float4* q = reinterpret_cast<const float4*>(tile_part(part, s, cb + j) + r0);
                p0[j] = __ldcg(q);
                p1[j] = __ldcg(q + 1);
            }
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            if (cb + j > s.c1 || !cta_has_units(cb + j, s.units)) continue;
            const float w[8] = {p0[j].x, p0[j].y, p0[j].z, p0[j].w, p1[j].x, p1[j].y, p1[j].z, p1[j].w};
#pragma unroll
            for (int e = 0; e < 8; ++e) v[e] = cb + j == s.c0 ? w[e] : __fadd_rn(v[e], w[e]);
        }
    }
}

__device__ __forceinline__ float split_row(const float* part, int64_t n, int64_t kt, int64_t units) {
    return tile_sum(part, tile_src(n >> 7, kt, units), static_cast<int>(n & 127));
}

template <typename Out>
__device__ __forceinline__ bool gemv_consume(const Gemv& g, const uint16_t* xs, const uint8_t* ring, uint64_t* full,
                                             uint64_t* empty, int& stage, uint32_t& phase, int ct, int* err,
                                             float* red, Out out) {
    const StageGeo geo = stage_geo(g);
    const int w = ct >> 5, lane = ct & 31;
    const uint32_t ring_s = smem_u32(ring);
    const uint32_t xs_s = smem_u32(xs);
    for (int64_t ch = 0; ch < geo.chunks; ++ch) {
        const int64_t cr0 = ch * kRowsPerChunk;
        const int64_t cr1 = cr0 + kRowsPerChunk < geo.rows ? cr0 + kRowsPerChunk : geo.rows;
        const int rc = static_cast<int>(cr1 - cr0);
        const int nrb = (rc + 15) / 16;
        const int G = kConsWarps / nrb;
        const int rb = w % nrb, kgi = w / nrb;
        const bool active = kgi < G;
        // ldmatrix row of this lane: rows rb*16 + lane % 16, columns (lane / 16) * 8 of each 16-wide k-step.
        const int rr = rb * 16 + (lane & 15);
        const int kh = lane >> 4;
        const int swz = rr < rc ? static_cast<int>(gemv_grow(g, cr0 + rr) & 7) : (rr & 7);
        const uint32_t rows_bytes = static_cast<uint32_t>(rc) * 128;
        float d[4] = {0.0f, 0.0f, 0.0f, 0.0f};
        for (int64_t kg = 0; kg < geo.kgroups; ++kg) {
            if (!mbar_wait(&full[stage], phase, err, kErrMmaWait)) return false;
            const int64_t kt0 = kg * geo.T, kt1 = kt0 + geo.T < g.kt ? kt0 + geo.T : g.kt;
            const int nkt = static_cast<int>(kt1 - kt0);
            if (active) {
                const uint32_t sb = ring_s + static_cast<uint32_t>(stage) * kStage + static_cast<uint32_t>(rr) * 128;
                for (int t = kgi; t < nkt; t += G) {
                    const uint32_t rowb = sb + static_cast<uint32_t>(t) * rows_bytes;
                    const int64_t kx = (kt0 + t) * 64;
#pragma unroll
                    for (int st4 = 0; st4 < 4; ++st4) {
                        uint32_t a0, a1, a2, a3;
                        ldsm_x4(rowb + (((2 * st4 + kh) ^ swz) << 4), a0, a1, a2, a3);
                        uint32_t b0 = 0, b1 = 0;
                        if (lane < 4) {
                            const uint32_t xa = xs_s + static_cast<uint32_t>((kx + st4 * 16 + 2 * lane) * 2);
                            asm volatile("ld.shared.b32 %0, [%1];" : "=r"(b0) : "r"(xa));
                            asm volatile("ld.shared.b32 %0, [%1];" : "=r"(b1) : "r"(xa + 16));
                        }
                        mma_16816(d, a0, a1, a2, a3, b0, b1);
                    }
                }
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[stage]);
            if (++stage == kRingStages) {
                stage = 0;
                phase ^= 1u;
            }
        }
        // Column 0 of D: lanes 4q hold rows q (d[0]) and q + 8 (d[2]) of the block.
        if (active && (lane & 3) == 0) {
            const int q = lane >> 2;
            red[kgi * (nrb * 16) + rb * 16 + q] = d[0];
            red[kgi * (nrb * 16) + rb * 16 + q + 8] = d[2];
        }
        cons_sync();
        if (ct < rc) {
            float v = red[ct];
            for (int q = 1; q < G; ++q) v += red[q * (nrb * 16) + ct];
            out(cr0 + ct, v);
        }
        cons_sync();  // red is reused by the next chunk
    }
    return true;
}

// RoPE (cpu_backend.cpp:332-379) of one head vector held PER elements per
// lane (lane l: elements l*PER ..): the pair (i, i + D/2) sits in lanes l and
// l + 16.  Returns the FP16-rounded rotated values as floats.
template <int PER>
__device__ __forceinline__ void rope_lane(const float (&x)[PER], int64_t pos, int lane, const float* cos_t,
                                          const float* sin_t, float (&out)[PER]) {
    const int64_t half = 16 * PER;
#pragma unroll
    for (int e = 0; e < PER; ++e) {
        const float other = __shfl_xor_sync(0xFFFFFFFFu, x[e], 16);
        const int64_t i = (lane & 15) * PER + e;
        const float c = cos_t[pos * half + i], sn = sin_t[pos * half + i];
        float r;
        if (lane < 16)
            r = __fsub_rn(__fmul_rn(x[e], c), __fmul_rn(other, sn));
        else
            r = __fadd_rn(__fmul_rn(other, sn), __fmul_rn(x[e], c));
        out[e] = f16_bits_to_f32(f32_to_f16_bits(r));
    }
}

template <int PER>
__device__ __forceinline__ void load_lane(const uint16_t* p, float (&x)[PER]) {
#pragma unroll
    for (int e = 0; e < PER; ++e) x[e] = f16_bits_to_f32(p[e]);
}

// One attention unit (query head h, key split sp) for the token at `pos`
// (cpu_backend.cpp:171-290 with q_len = 1): RoPE on q and on this step's key,
// the KV-cache append (by one unit per kv head), an online softmax over the
// split's keys (8 keys per warp at a time, loads issued together), the warps
// merged in shared memory; the last split of a head to finish merges every
// split in split order and writes out = fp16(acc * (1 / sum)).
template <int PER>
__device__ __noinline__ void attention_unit(const StepArgs& a, const StepLayer& ly, int64_t pos, int ct, float (*sm_acc)[256],
                               float* sm_m, float* sm_l, volatile int* sm_last) {
    constexpr int D = PER * 32;
    const int h = static_cast<int>(blockIdx.x / a.att_split), sp = static_cast<int>(blockIdx.x % a.att_split);
    const int64_t g_glob = (a.h0 + h) / a.group;
    const int64_t g = g_glob - a.g0;
    const int warp = ct >> 5, lane = ct & 31;
    const int64_t kv_len = pos + 1 < a.max_seq ? pos + 1 : a.max_seq;
    const int64_t chunk = (kv_len + a.att_split - 1) / a.att_split;
    const int64_t k0 = sp * chunk;
    const int64_t k1 = k0 + chunk < kv_len ? k0 + chunk : kv_len;
    float qraw[PER], kraw[PER], qv[PER], kn[PER], vn[PER];
    load_lane<PER>(a.qkv_out + static_cast<int64_t>(h) * D + lane * PER, qraw);
    load_lane<PER>(a.qkv_out + (a.nh + g) * D + lane * PER, kraw);
    load_lane<PER>(a.qkv_out + (a.nh + a.nkv + g) * D + lane * PER, vn);
    rope_lane<PER>(qraw, pos, lane, a.cos_t, a.sin_t, qv);
    rope_lane<PER>(kraw, pos, lane, a.cos_t, a.sin_t, kn);
    const uint16_t* kb = ly.kc + g * a.max_seq * D + lane * PER;
    const uint16_t* vb = ly.vc + g * a.max_seq * D + lane * PER;
    // The first local query head of the kv head appends this step's k and v.
    int64_t h_first = g_glob * a.group - a.h0;
    if (h_first < 0) h_first = 0;
    if (h == h_first && warp == 0 && pos >= k0 && pos < k1 && pos < a.max_seq) {
        uint16_t* kd = ly.kc + (g * a.max_seq + pos) * D + lane * PER;
        uint16_t* vd = ly.vc + (g * a.max_seq + pos) * D + lane * PER;
#pragma unroll
        for (int e = 0; e < PER; ++e) {
            kd[e] = f32_to_f16_bits(kn[e]);
            vd[e] = f32_to_f16_bits(vn[e]);
        }
    }
    float m = -INFINITY, l = 0.0f, acc[PER];
#pragma unroll
    for (int e = 0; e < PER; ++e) acc[e] = 0.0f;
    for (int64_t base = k0 + warp * kAttKeys; base < k1; base += kAttWarps * kAttKeys) {
        const int nk = k1 - base >= kAttKeys ? kAttKeys : static_cast<int>(k1 - base);
        float kx[kAttKeys][PER], vx[kAttKeys][PER];
#pragma unroll
        for (int i = 0; i < kAttKeys; ++i) {
            if (i >= nk) continue;
            const int64_t key = base + i;
            if (key == pos) {
#pragma unroll
                for (int e = 0; e < PER; ++e) {
                    kx[i][e] = kn[e];
                    vx[i][e] = vn[e];
                }
            } else {
                load_lane<PER>(kb + key * D, kx[i]);
                load_lane<PER>(vb + key * D, vx[i]);
            }
        }
        float sc[kAttKeys];
#pragma unroll
        for (int i = 0; i < kAttKeys; ++i) {
            float d = 0.0f;
#pragma unroll
            for (int e = 0; e < PER; ++e) d = __fadd_rn(d, __fmul_rn(qv[e], i < nk ? kx[i][e] : 0.0f));
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) d = __fadd_rn(d, __shfl_xor_sync(0xFFFFFFFFu, d, o));
            sc[i] = i < nk ? __fmul_rn(d, a.scale) : -INFINITY;
        }
        float mr = m;
#pragma unroll
        for (int i = 0; i < kAttKeys; ++i) mr = fmaxf(mr, sc[i]);
        const float corr = m == -INFINITY ? 0.0f : expf(__fsub_rn(m, mr));
        l = __fmul_rn(l, corr);
#pragma unroll
        for (int e = 0; e < PER; ++e) acc[e] = __fmul_rn(acc[e], corr);
#pragma unroll
        for (int i = 0; i < kAttKeys; ++i) {
            if (i >= nk) continue;
            const float p = expf(__fsub_rn(sc[i], mr));
            l = __fadd_rn(l, p);
#pragma unroll
            for (int e = 0; e < PER; ++e) acc[e] = __fadd_rn(acc[e], __fmul_rn(p, vx[i][e]));
        }
        m = mr;
    }
    if (lane == 0) {
        sm_m[warp] = m;
        sm_l[warp] = l;
    }
#pragma unroll
    for (int e = 0; e < PER; ++e) sm_acc[warp][lane * PER + e] = acc[e];
    cons_sync();
    float M = -INFINITY;
    for (int w = 0; w < kAttWarps; ++w) M = fmaxf(M, sm_m[w]);
    float* dst = a.att_part + (static_cast<int64_t>(h) * a.att_split + sp) * (D + 2);
    if (ct == 0) {
        float L = 0.0f;
        for (int w = 0; w < kAttWarps; ++w)
            if (sm_m[w] != -INFINITY) L = __fadd_rn(L, __fmul_rn(sm_l[w], expf(__fsub_rn(sm_m[w], M))));
        dst[0] = M;
        dst[1] = L;
    }
    for (int d = ct; d < D; d += kStepCons) {
        float A = 0.0f;
        for (int w = 0; w < kAttWarps; ++w)
            if (sm_m[w] != -INFINITY) A = __fadd_rn(A, __fmul_rn(sm_acc[w][d], expf(__fsub_rn(sm_m[w], M))));
        dst[2 + d] = A;
    }
    __threadfence();
    cons_sync();
    if (ct == 0) {
        const int prev = atomicAdd(&a.att_cnt[h], 1);
        *sm_last = prev == a.att_split - 1;
        if (*sm_last) a.att_cnt[h] = 0;
    }
    cons_sync();
    if (!*sm_last) return;
    __threadfence();
    const float* ph = a.att_part + static_cast<int64_t>(h) * a.att_split * (D + 2);
    float MM = -INFINITY;
    for (int s2 = 0; s2 < a.att_split; ++s2) MM = fmaxf(MM, ph[s2 * (D + 2)]);
    float LL = 0.0f;
    for (int s2 = 0; s2 < a.att_split; ++s2) {
        const float ms = ph[s2 * (D + 2)];
        if (ms != -INFINITY) LL = __fadd_rn(LL, __fmul_rn(ph[s2 * (D + 2) + 1], expf(__fsub_rn(ms, MM))));
    }
    const float inv = __fdiv_rn(1.0f, LL);
    for (int d = ct; d < D; d += kStepCons) {
        float A = 0.0f;
        for (int s2 = 0; s2 < a.att_split; ++s2) {
            const float ms = ph[s2 * (D + 2)];
            if (ms != -INFINITY) A = __fadd_rn(A, __fmul_rn(ph[s2 * (D + 2) + 2 + d], expf(__fsub_rn(ms, MM))));
        }
        a.attn[static_cast<int64_t>(h) * D + d] = f32_to_f16_bits(__fmul_rn(A, inv));
    }
}

// out = fp16(a + b) (b may be null: out = a), normed = RMSNorm(out) written to
// the operand buffer xs, and out to `res` when given (cpu_backend.cpp:292-330,
// 403-455).  Every CTA computes the same row; one of them stores it.  The row
// passes through xs (FP16 values are exact as floats), so no thread holds it
// in registers.
__device__ __noinline__ void add_norm_cons(const uint16_t* a, const uint16_t* b, int64_t H, const void* w, int wdt,
                                           float eps, uint16_t* xs, uint16_t* res, int ct, float* red,
                                           const float* bpart = nullptr, int64_t bkt = 0, int64_t bunits = 0) {
    const int nv = static_cast<int>(H / 8);
    float ss = 0.0f;
    for (int v = ct; v < nv; v += kStepCons) {
        const uint4 va = *reinterpret_cast<const uint4*>(a + static_cast<int64_t>(v) * 8);
        uint4 vr = va;
        if (bpart != nullptr) {  // b = a split GEMV's rows, summed over its CTAs and rounded to FP16
            float fa[8];
            unpack8h(va, fa);
            const int64_t n0 = static_cast<int64_t>(v) * 8;  // 8 rows of one tile
            float bs[8];
            tile_sum8(bpart, tile_src(n0 >> 7, bkt, bunits), static_cast<int>(n0 & 127), bs);
            uint16_t h[8];
#pragma unroll
            for (int e = 0; e < 8; ++e) h[e] = f32_to_f16_bits(__fadd_rn(fa[e], f16_bits_to_f32(f32_to_f16_bits(bs[e]))));
            vr = make_uint4(pk2(h[0], h[1]), pk2(h[2], h[3]), pk2(h[4], h[5]), pk2(h[6], h[7]));
        } else if (b != nullptr) {
            const uint4 vb = *reinterpret_cast<const uint4*>(b + static_cast<int64_t>(v) * 8);
            float fa[8], fb[8];
            unpack8h(va, fa);
            unpack8h(vb, fb);
            uint16_t h[8];
#pragma unroll
            for (int e = 0; e < 8; ++e) h[e] = f32_to_f16_bits(__fadd_rn(fa[e], fb[e]));
            vr = make_uint4(pk2(h[0], h[1]), pk2(h[2], h[3]), pk2(h[4], h[5]), pk2(h[6], h[7]));
        }
        float x[8];
        unpack8h(vr, x);
        if (res != nullptr) *reinterpret_cast<uint4*>(res + static_cast<int64_t>(v) * 8) = vr;
        *reinterpret_cast<uint4*>(xs + static_cast<int64_t>(v) * 8) = vr;
#pragma unroll
        for (int e = 0; e < 8; ++e) ss = __fadd_rn(ss, __fmul_rn(x[e], x[e]));
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) ss = __fadd_rn(ss, __shfl_xor_sync(0xFFFFFFFFu, ss, o));
    if ((ct & 31) == 0) red[ct >> 5] = ss;
    cons_sync();
    float total = 0.0f;
    for (int wi = 0; wi < kStepCons / 32; ++wi) total = __fadd_rn(total, red[wi]);
    const float rms = __fsqrt_rn(__fadd_rn(__fdiv_rn(total, static_cast<float>(H)), eps));
    const float inv = __fdiv_rn(1.0f, rms);
    for (int v = ct; v < nv; v += kStepCons) {
        float x[8];
        unpack8h(*reinterpret_cast<const uint4*>(xs + static_cast<int64_t>(v) * 8), x);
        uint16_t h[8];
#pragma unroll
        for (int e = 0; e < 8; ++e)
            h[e] = f32_to_f16_bits(__fmul_rn(__fmul_rn(x[e], inv), gain(w, wdt, static_cast<int64_t>(v) * 8 + e)));
        *reinterpret_cast<uint4*>(xs + static_cast<int64_t>(v) * 8) =
            make_uint4(pk2(h[0], h[1]), pk2(h[2], h[3]), pk2(h[4], h[5]), pk2(h[6], h[7]));
    }
    cons_sync();  // xs complete, red free again
}

// Operand buffer <- n FP16 values from global memory, zero-padded to n_pad.
__device__ void load_operand(uint16_t* xs, const uint16_t* src, int64_t n, int64_t n_pad, int ct) {
    for (int64_t v = ct; v < n / 8; v += kStepCons)
        *reinterpret_cast<uint4*>(xs + v * 8) = *reinterpret_cast<const uint4*>(src + v * 8);
    for (int64_t i = n + ct; i < n_pad; i += kStepCons) xs[i] = 0;
    cons_sync();
}

__device__ __forceinline__ void st_release_sys_u64(unsigned long long* p, unsigned long long v) {
    asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}

__device__ __forceinline__ unsigned long long ld_acquire_sys_u64(const unsigned long long* p) {
    unsigned long long v;
    asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}

// Tell every peer this rank's data for `epoch` is complete (CTA 0 only).
__device__ __forceinline__ void tp_signal(const StepArgs& a, unsigned long long epoch) {
    __threadfence_system();
    for (int q = 0; q < a.world; ++q)
        if (q != a.rank) st_release_sys_u64(a.peer_flags[q] + a.rank, epoch);
}

// Wait (bounded) until every peer has published `epoch`; false on timeout.
__device__ __forceinline__ bool tp_wait(const StepArgs& a, unsigned long long epoch) {
    const unsigned long long t0 = now_ns();
    for (int q = 0; q < a.world; ++q) {
        if (q == a.rank) continue;
        while (ld_acquire_sys_u64(a.peer_flags[a.rank] + q) < epoch) {
            __nanosleep(32);
            if (error_raised(a.err)) return false;
            if (now_ns() - t0 > kWaitLimitNs) {
                raise_error(a.err, kErrPeerWait);
                return false;
            }
        }
    }
    return true;
}

// Row-parallel output finished across GPUs (qwen_model.cpp:256 and 288 split
// over ranks): after the grid barrier that follows the local GEMV, CTA 0
// publishes the epoch; every CTA waits for the peers, sums its slice of the
// hidden row over the ranks' FP32 partials in rank order (the same order on
// every rank), rounds once to FP16 into y, and a grid barrier hands y to
// every CTA.
__device__ __noinline__ bool tp_reduce(const StepArgs& a, int site, unsigned long long epoch, uint16_t* y, int ct,
                                       unsigned& nbar, volatile int* ok_sh, int64_t kt = 0, int64_t units = 0) {
    if (ct == 0) {
        if (blockIdx.x == 0) tp_signal(a, epoch);
        *ok_sh = tp_wait(a, epoch) ? 1 : 0;
    }
    cons_sync();
    if (!*ok_sh) return false;
    int64_t s0, s1;
    my_rows(a.H, &s0, &s1);
    // Each rank's row: a plain FP32 row (units == 0) or a split GEMV's
    // partials summed over its CTAs; ranks added in rank order.
    auto rank_row = [&](int q, int64_t n) {
        return units > 0 ? split_row(a.peer_buf[site][q], n, kt, units) : __ldcg(a.peer_buf[site][q] + n);
    };
    for (int64_t n = s0 + ct; n < s1; n += kStepCons) {
        float acc = rank_row(0, n);
        for (int q = 1; q < a.world; ++q) acc = __fadd_rn(acc, rank_row(q, n));
        y[n] = f32_to_f16_bits(acc);
    }
    return grid_sync(a, nbar, ct, ok_sh);
}

template <int PER>
__global__ void __launch_bounds__(kStepThreads, 1) decode_step_kernel(const StepArgs a) {
    extern __shared__ uint8_t step_smem_raw[];
    uint8_t* ring = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(step_smem_raw) + 1023) & ~uintptr_t(1023));
    uint16_t* xs = reinterpret_cast<uint16_t*>(ring + kRingStages * kStage);
    __shared__ __align__(8) uint64_t full[kRingStages];
    __shared__ __align__(8) uint64_t empty[kRingStages];
    __shared__ float red[kStepCons / 32];
    __shared__ float red_rows[256];
    __shared__ int ok_sh;
    __shared__ int last_sh;
    __shared__ uint16_t gu_rows[512];
    __shared__ float att_m[kAttWarps], att_l[kAttWarps];
    __shared__ float att_acc[kAttWarps][256];
    __shared__ float cv_sh[kStepCons / 32];
    __shared__ int64_t ci_sh[kStepCons / 32];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (threadIdx.x == 0) {
        for (int i = 0; i < kRingStages; ++i) {
            mbar_init(&full[i], 1);
            mbar_init(&empty[i], kStepCons / 32);
        }
        fence_barrier_init();
    }
    __syncthreads();
    if (warp == 0) {
        if (lane == 0) produce(a, ring, full, empty);
        return;
    }
    const int ct = threadIdx.x - 32;
    const bool writer = blockIdx.x == 0;
    unsigned nbar = 0;
    int stage = 0;
    uint32_t phase = 0;
    int64_t pos = a.st->pos;
    if (pos < 0 || pos >= a.max_seq) {  // the host keeps positions in range; never index past the tables
        if (ct == 0) raise_error(a.err, kErrBadToken);
        pos = pos < 0 ? 0 : a.max_seq - 1;
    }
    int64_t token = a.st->token;
    if (token < 0 || token >= a.vocab) {
        if (ct == 0) raise_error(a.err, kErrBadToken);
        token = 0;
    }
    const int64_t H = a.H;
    const int64_t ktH = (H + 63) / 64;
    const bool tp = a.world > 1;
    const unsigned long long ep0 = tp ? *a.epoch : 0ull;
    // x = embedding row (qwen_model.cpp:59-64); normed = RMSNorm(x) for layer 0.
    add_norm_cons(a.embed + token * H, nullptr, H, a.layers[0].ln1, a.layers[0].ln1_dt, a.eps, xs, writer ? a.x : nullptr,
                  ct, red);
    for (int64_t i = H + ct; i < ktH * 64; i += kStepCons) xs[i] = 0;
    cons_sync();
    for (int l = 0; l < a.L; ++l) {
        const StepLayer& ly = a.layers[l];
        // q|k|v = fp16(fp16(x W^T) + bias) (qwen_model.cpp:126-155)
        Gemv g = gemv_of(a, l, 0);
        if (!gemv_consume(g, xs, ring, full, empty, stage, phase, ct, a.err, red_rows, [&](int64_t row, float v) {
                const int64_t n = gemv_grow(g, row);
                a.qkv_out[n] = round_out(v, ly.bias, n);
            }))
            return;
        if (!grid_sync(a, nbar, ct, &ok_sh)) return;
        if (blockIdx.x < a.nh * a.att_split) attention_unit<PER>(a, ly, pos, ct, att_acc, att_m, att_l, &last_sh);
        if (!grid_sync(a, nbar, ct, &ok_sh)) return;
        const int64_t ad = a.nh * a.D;
        load_operand(xs, a.attn, ad, ((ad + 63) / 64) * 64, ct);
        g = gemv_of(a, l, 1);
        if (!gemv_consume(g, xs, ring, full, empty, stage, phase, ct, a.err, red_rows, [&](int64_t row, float v) {
                const int64_t n = gemv_grow(g, row);
                if (tp)
                    const_cast<float*>(a.peer_buf[0][a.rank])[n] = v;
                else
                    a.yo[n] = f32_to_f16_bits(v);
            }))
            return;
        if (!grid_sync(a, nbar, ct, &ok_sh)) return;
        if (tp && !tp_reduce(a, 0, ep0 + 2 * l + 1, a.yo, ct, nbar, &ok_sh)) return;
        // r1 = fp16(x + o); normed = RMSNorm(r1) (qwen_model.cpp:321-329)
        add_norm_cons(a.x, a.yo, H, ly.ln2, ly.ln2_dt, a.eps, xs, writer ? a.r1 : nullptr, ct, red);
        for (int64_t i = H + ct; i < ktH * 64; i += kStepCons) xs[i] = 0;
        cons_sync();
        // gate and up rows of this CTA's intermediate range, then SiLU(gate) * up
        // (qwen_model.cpp:278-285: each rounded to FP16 in turn).
        g = gemv_of(a, l, 2);
        const int64_t la = g.a1 - g.a0;
        if (!gemv_consume(g, xs, ring, full, empty, stage, phase, ct, a.err, red_rows,
                          [&](int64_t row, float v) { gu_rows[row] = f32_to_f16_bits(v); }))
            return;
        cons_sync();
        for (int64_t j = ct; 2 * j < la; j += kStepCons) {
            const float sg = f16_bits_to_f32(a.silu_lut[gu_rows[2 * j]]);
            const float up = f16_bits_to_f32(gu_rows[2 * j + 1]);
            a.act[g.a0 / 2 + j] = f32_to_f16_bits(__fmul_rn(sg, up));
        }
        if (!grid_sync(a, nbar, ct, &ok_sh)) return;
        load_operand(xs, a.act, a.I, ((a.I + 63) / 64) * 64, ct);
        g = gemv_of(a, l, 3);
        const int64_t kt_d = g.kt, units_d = g.units;
        if (!gemv_split(g, xs, ring, full, empty, stage, phase, ct, a.err, red_rows, a.part_down)) return;
        if (!grid_sync(a, nbar, ct, &ok_sh)) return;
        // x = fp16(r1 + down); normed = RMSNorm(x) with the next layer's input
        // gains, or the final norm (qwen_model.cpp:331-332, 368-370).
        const bool last_layer = l + 1 == a.L;
        const void* nw = last_layer ? a.norm : a.layers[l + 1].ln1;
        const int ndt = last_layer ? a.norm_dt : a.layers[l + 1].ln1_dt;
        if (tp) {
            if (!tp_reduce(a, 1, ep0 + 2 * l + 2, a.yd, ct, nbar, &ok_sh, kt_d, units_d)) return;
            add_norm_cons(a.r1, a.yd, H, nw, ndt, a.eps, xs, writer ? a.x : nullptr, ct, red);
        } else {
            add_norm_cons(a.r1, nullptr, H, nw, ndt, a.eps, xs, writer ? a.x : nullptr, ct, red, a.part_down, kt_d,
                          units_d);
        }
        for (int64_t i = H + ct; i < ktH * 64; i += kStepCons) xs[i] = 0;
        cons_sync();
    }
    // lm_head rows of this CTA; each thread keeps the first maximum of the
    // FP16 logits it finishes (rows in increasing order), NaN never chosen
    // (inference_engine.cpp:84-95).
    Gemv g = gemv_of(a, a.L, 0);
    float best = -INFINITY;
    int64_t best_i = INT64_MAX;
    if (!gemv_consume(g, xs, ring, full, empty, stage, phase, ct, a.err, red_rows, [&](int64_t row, float v) {
            const float f = f16_bits_to_f32(f32_to_f16_bits(v));
            const int64_t n = a.v0 + gemv_grow(g, row);
            if (f > best || (f == best && n < best_i)) {
                best = f;
                best_i = n;
            }
        }))
        return;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const float ov = __shfl_xor_sync(0xFFFFFFFFu, best, o);
        const int64_t oi = __shfl_xor_sync(0xFFFFFFFFu, best_i, o);
        if (ov > best || (ov == best && oi < best_i)) {
            best = ov;
            best_i = oi;
        }
    }
    if ((ct & 31) == 0) {
        cv_sh[ct >> 5] = best;
        ci_sh[ct >> 5] = best_i;
    }
    cons_sync();
    if (ct == 0) {
        for (int w = 1; w < kStepCons / 32; ++w)
            if (cv_sh[w] > best || (cv_sh[w] == best && ci_sh[w] < best_i)) {
                best = cv_sh[w];
                best_i = ci_sh[w];
            }
        a.cand_val[blockIdx.x] = best;
        a.cand_idx[blockIdx.x] = best_i;
    }
    if (!grid_sync(a, nbar, ct, &ok_sh)) return;
    if (writer && ct == 0) {
        float bv = -INFINITY;
        int64_t bi = INT64_MAX;
        for (unsigned c = 0; c < gridDim.x; ++c) {
            const float v = a.cand_val[c];
            const int64_t i = a.cand_idx[c];
            if (v > bv || (v == bv && i < bi)) {
                bv = v;
                bi = i;
            }
        }
        if (tp) {
            // Vocabulary shards: publish this rank's candidate, then take the
            // first maximum over the ranks in rank (= vocabulary) order.
            const unsigned long long ep = ep0 + 2ull * a.L + 1ull;
            float* mine = a.peer_cand[a.rank];
            mine[0] = bv;
            *reinterpret_cast<int64_t*>(mine + 2) = bi;
            tp_signal(a, ep);
            if (!tp_wait(a, ep)) return;
            bv = -INFINITY;
            bi = INT64_MAX;
            for (int q = 0; q < a.world; ++q) {
                const float v = __ldcg(a.peer_cand[q]);
                const int64_t i = __ldcg(reinterpret_cast<const long long*>(a.peer_cand[q] + 2));
                if (v > bv || (v == bv && i < bi)) {
                    bv = v;
                    bi = i;
                }
            }
            *a.epoch = ep0 + 2ull * a.L + 1ull;
        }
        if (bi == INT64_MAX) bi = 0;  // every logit -inf or NaN: the reference keeps index 0
        const int32_t t = static_cast<int32_t>(bi);
        StepState* st = a.st;
        if (st->step < a.tokens_cap) a.tokens[st->step] = t;
        st->step += 1;
        st->token = t;
        st->pos += 1;
    }
}

}  // namespace

size_t decode_step_smem(int64_t max_operand) {
    const int64_t padded = ((max_operand + 63) / 64) * 64;
    // 1 KB alignment slack, the ring, the operand buffer, and 2 KB after it:
    // a 16-row ldmatrix block of a short chunk reads up to 15 rows (1920 B)
    // past its stage, which must stay inside the allocation.
    return 1024 + static_cast<size_t>(kRingStages) * kStage + static_cast<size_t>(padded) * 2 + 2048;
}

int decode_step_grid() {
    int dev = 0, sms = 0, coop = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return 0;
    if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) return 0;
    if (cudaDeviceGetAttribute(&coop, cudaDevAttrCooperativeLaunch, dev) != cudaSuccess || !coop) return 0;
    return sms;
}

char g_step_diag[256] = "";

template <int PER>
cudaError_t launch_step_t(const StepArgs& a, int grid, size_t smem, cudaStream_t s) {
    cudaError_t e = cudaFuncSetAttribute(decode_step_kernel<PER>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(smem));
    if (e != cudaSuccess) return e;
    e = cudaFuncSetAttribute(decode_step_kernel<PER>, cudaFuncAttributePreferredSharedMemoryCarveout,
                             cudaSharedmemCarveoutMaxShared);
    if (e != cudaSuccess) return e;
    int per_sm = 0;
    e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, decode_step_kernel<PER>, kStepThreads, smem);
    if (e != cudaSuccess) return e;
    if (per_sm < 1) {
        cudaFuncAttributes fa{};
        cudaFuncGetAttributes(&fa, decode_step_kernel<PER>);
        int dev = 0, smem_sm = 0, regs_sm = 0, smem_blk = 0;
        cudaGetDevice(&dev);
        cudaDeviceGetAttribute(&smem_sm, cudaDevAttrMaxSharedMemoryPerMultiprocessor, dev);
        cudaDeviceGetAttribute(&regs_sm, cudaDevAttrMaxRegistersPerMultiprocessor, dev);
        cudaDeviceGetAttribute(&smem_blk, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
        snprintf(g_step_diag, sizeof(g_step_diag),
                 "step kernel does not fit an SM: %d threads x %d regs, static smem %zu + dynamic %zu, local %zu, "
                 "max threads %d; SM: %d regs, %d smem, block opt-in %d",
                 kStepThreads, fa.numRegs, fa.sharedSizeBytes, smem, fa.localSizeBytes, fa.maxThreadsPerBlock,
                 regs_sm, smem_sm, smem_blk);
        return cudaErrorCooperativeLaunchTooLarge;
    }
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(static_cast<unsigned>(grid));
    cfg.blockDim = dim3(kStepThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeCooperative;  // every CTA resident at once: the grid barriers need it
    attr[0].val.cooperative = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    e = cudaLaunchKernelEx(&cfg, decode_step_kernel<PER>, a);
    if (e == cudaSuccess) note_launches(1);
    return e;
}

const char* decode_step_diag() { return g_step_diag; }

cudaError_t launch_decode_step(const StepArgs& a, int grid, cudaStream_t s) {
    const int64_t op = std::max(std::max(a.H, a.nh * a.D), a.I);
    const size_t smem = decode_step_smem(op);
    switch (a.D / 32) {
        case 2: return launch_step_t<2>(a, grid, smem, s);
        case 4: return launch_step_t<4>(a, grid, smem, s);
        case 8: return launch_step_t<8>(a, grid, smem, s);
        default: return cudaErrorInvalidValue;
    }
}

}  // namespace mrt
