// common.cuh -- device helpers shared by the sm_100a kernels.
//
// PTX wrappers for mbarriers, TMA tile loads, tcgen05 (TMEM alloc, MMA,
// commit, loads) and the rounding rule of the reference's FP16 converter.
// Every wait on an mbarrier is bounded: after a time limit it records an
// error code in a device flag that the host reads (mrt_sync) and returns
// false, so a lost arrival ends the kernel instead of hanging the GPU.
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace mrt {

// Device error codes written to the context's flag.
enum : int {
    kErrNone = 0,
    kErrTmaWait = 1,   // producer gave up waiting for a free pipeline stage
    kErrMmaWait = 2,   // MMA issuer gave up waiting for data or a free accumulator
    kErrEpiWait = 3,   // epilogue gave up waiting for a finished accumulator
    kErrDrainWait = 4, // clean-up wait for in-flight copies/MMAs gave up
    kErrSelfTest = 5,  // mrt_selftest_wait_timeout's wait gave up (expected)
    kErrBadToken = 6,  // the decoder's embedding met a token id outside the vocabulary
    kErrPeerWait = 7,  // a cross-GPU all-reduce gave up waiting for a peer's partial
};

// Wall-clock limit of one bounded wait, in nanoseconds of %globaltimer.
constexpr uint64_t kWaitLimitNs = 2000000000ull;

__device__ __forceinline__ uint64_t globaltimer_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// ------------------------------------------------------------------ FP16 rounding

// FP32 -> FP16 bits with the reference's rule (include/mruntime/dtype.h:39-119):
// round-to-nearest-even, overflow to infinity, FP32 denormals to signed zero
// (they lie far below half the smallest FP16 subnormal, so the hardware
// conversion already gives that), and NaN keeping the top ten payload bits,
// forced non-zero -- the one case where the hardware conversion differs.
__device__ __forceinline__ uint16_t f32_to_f16_bits(float v) {
    const uint32_t x = __float_as_uint(v);
    if ((x & 0x7FFFFFFFu) > 0x7F800000u) {
        uint32_t p = (x >> 13) & 0x3FFu;
        if (p == 0) p = 1;
        return static_cast<uint16_t>(((x >> 16) & 0x8000u) | 0x7C00u | p);
    }
    return __half_as_ushort(__float2half_rn(v));
}

__device__ __forceinline__ float f16_bits_to_f32(uint16_t h) {
    return __half2float(__ushort_as_half(h));
}

__device__ __forceinline__ float bf16_bits_to_f32(uint16_t b) {
    return __uint_as_float(static_cast<uint32_t>(b) << 16);
}

// FP32 -> BF16 bits with the reference's rounding trick (dtype.h:153-160).
__device__ __forceinline__ uint16_t f32_to_bf16_bits(float v) {
    uint32_t x = __float_as_uint(v);
    x += 0x7FFFu + ((x >> 16) & 1u);
    return static_cast<uint16_t>(x >> 16);
}

// Output rounding with the optional q/k/v bias of qwen_model.cpp:130-155:
// round the accumulator to FP16, widen, add the FP16 bias, round again.
__device__ __forceinline__ uint16_t round_out(float acc, const uint16_t* bias, int64_t n) {
    uint16_t h = f32_to_f16_bits(acc);
    if (bias != nullptr) h = f32_to_f16_bits(__fadd_rn(f16_bits_to_f32(h), f16_bits_to_f32(bias[n])));
    return h;
}

// Residual add after the output rounding, the reference's add op
// (cpu_backend.cpp:430-455, called at qwen_model.cpp:316 and 324): both FP16
// operands widened, one FP32 add, rounded to FP16.  `res` null: h unchanged.
__device__ __forceinline__ uint16_t add_f16(uint16_t r, uint16_t h) {
    return f32_to_f16_bits(__fadd_rn(f16_bits_to_f32(r), f16_bits_to_f32(h)));
}

__device__ __forceinline__ uint16_t add_residual(uint16_t h, const uint16_t* res, int64_t i) {
    return res == nullptr ? h : add_f16(res[i], h);
}

// ------------------------------------------------------------------ cross-GPU flags

// System-scope release store / acquire load of a 64-bit flag (peer memory
// mapped by CUDA IPC, read and written over NVLink).
__device__ __forceinline__ void st_release_sys(unsigned long long* p, unsigned long long v) {
    asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}

__device__ __forceinline__ unsigned long long ld_acquire_sys(const unsigned long long* p) {
    unsigned long long v;
    asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}

__device__ __forceinline__ unsigned long long global_ns() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
    return t;
}

// ------------------------------------------------------------------ greedy pick

// (value, index) under the reference's greedy rule (inference_engine.cpp:84-95):
// the larger value wins; on equal values the lower index wins (the reference
// scans upwards and only a strictly greater value replaces the best); NaN is
// never chosen, which is the same as reading it as -inf with the lowest-index
// rule, because an all -inf/NaN row then yields index 0, as the reference does.
struct ArgBest {
    float v;
    int64_t i;
};

__device__ __forceinline__ ArgBest arg_better(ArgBest a, ArgBest b) {
    if (b.v > a.v || (b.v == a.v && b.i < a.i)) return b;
    return a;
}

__device__ __forceinline__ float nan_to_ninf(float v) { return v != v ? -INFINITY : v; }

// Best (value, index) over the 32 lanes of a warp, valid in lane 0.
__device__ __forceinline__ ArgBest warp_arg_best(ArgBest b) {
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) {
        ArgBest o;
        o.v = __shfl_down_sync(0xFFFFFFFFu, b.v, off);
        o.i = __shfl_down_sync(0xFFFFFFFFu, b.i, off);
        b = arg_better(b, o);
    }
    return b;
}

// ------------------------------------------------------------------ error flag

__device__ __forceinline__ void raise_error(int* flag, int code) {
    if (flag != nullptr) atomicCAS(flag, 0, code);
}

__device__ __forceinline__ bool error_raised(const int* flag) {
    return flag != nullptr && *reinterpret_cast<const volatile int*>(flag) != 0;
}

// ------------------------------------------------------------------ mbarrier

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}

// Make barrier initialisation visible to the async (TMA / tensor core) proxy.
__device__ __forceinline__ void fence_barrier_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
                 "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.b32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

// Wait for the phase with the given parity to complete.  Gives up (returns
// false, raising `code`) after kWaitLimitNs or as soon as another thread of
// the grid has raised an error.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, int* flag, int code,
                                          uint64_t limit_ns = kWaitLimitNs) {
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = globaltimer_ns();
    for (uint32_t it = 1;; ++it) {
        if (mbar_try_wait(bar, parity)) return true;
        if ((it & 255u) == 0) {
            if (error_raised(flag)) return false;
            if (globaltimer_ns() - t0 > limit_ns) {
                raise_error(flag, code);
                return false;
            }
        }
    }
}

// ------------------------------------------------------------------ TMA

// 2-D tiled bulk tensor load global -> shared, completion counted in bytes on
// `bar`.  c0 is the innermost (contiguous) coordinate in elements.
__device__ __forceinline__ void tma_load_2d(void* smem_dst, const void* tmap, uint64_t* bar,
                                            int32_t c0, int32_t c1) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%2, %3}], [%4];" ::"r"(smem_u32(smem_dst)),
        "l"(reinterpret_cast<uint64_t>(tmap)), "r"(c0), "r"(c1), "r"(smem_u32(bar))
        : "memory");
}

__device__ __forceinline__ void prefetch_tmap(const void* tmap) {
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(tmap)) : "memory");
}

// Linear bulk copy global -> shared (no tensor map), completion counted in
// bytes on `bar`.  Both addresses 16-byte aligned, bytes a multiple of 16.
__device__ __forceinline__ void bulk_load(void* smem_dst, const void* gmem_src, uint32_t bytes, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
            smem_u32(smem_dst)),
        "l"(reinterpret_cast<uint64_t>(gmem_src)), "r"(bytes), "r"(smem_u32(bar))
        : "memory");
}

// An L2 policy that evicts first the lines it fills: for data read once per
// pass (streamed weights), so they do not push out what other kernels reuse.
__device__ __forceinline__ uint64_t l2_policy_evict_first() {
    uint64_t p;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
    return p;
}

// bulk_load with an L2 cache policy (see l2_policy_evict_first).
__device__ __forceinline__ void bulk_load_hint(void* smem_dst, const void* gmem_src, uint32_t bytes, uint64_t* bar,
                                               uint64_t policy) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;" ::"r"(
            smem_u32(smem_dst)),
        "l"(reinterpret_cast<uint64_t>(gmem_src)), "r"(bytes), "r"(smem_u32(bar)), "l"(policy)
        : "memory");
}

// Element offset of (row r, column k) in the tiled weight layout: 128 x 64
// tiles, tile (r / 128, k / 64) at ((r / 128) * k_tiles + k / 64) * 8192, and
// inside a tile row-major 64-element rows whose 16-byte chunks are permuted
// as the 128-byte shared-memory swizzle does (chunk c of row r at c ^ (r % 8)).
__host__ __device__ __forceinline__ int64_t tiled_offset(int64_t r, int64_t k, int64_t k_tiles) {
    const int64_t rr = r & 127, kk = k & 63;
    const int64_t chunk = (kk >> 3) ^ (rr & 7);
    return (((r >> 7) * k_tiles + (k >> 6)) << 13) + (rr << 6) + (chunk << 3) + (kk & 7);
}

// 32-byte store (one whole L2 sector per thread); p must be 32-byte aligned.
__device__ __forceinline__ void st_global_v8(void* p, uint32_t a, uint32_t b, uint32_t c, uint32_t d, uint32_t e,
                                             uint32_t f, uint32_t g, uint32_t h) {
    asm volatile("st.global.v8.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8};" ::"l"(p), "r"(a), "r"(b), "r"(c), "r"(d),
                 "r"(e), "r"(f), "r"(g), "r"(h)
                 : "memory");
}

// ------------------------------------------------------------------ dependent launch

// Let the next kernel in the stream (launched with programmatic stream
// serialisation) start its prologue while this one still runs.
__device__ __forceinline__ void griddep_launch_dependents() {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// Block until the kernels this one depends on have completed and their
// memory is visible (a no-op when launched without a programmatic edge).
__device__ __forceinline__ void griddep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

// ------------------------------------------------------------------ tcgen05

__device__ __forceinline__ void tmem_alloc(uint32_t* dst_smem, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(dst_smem)),
                 "r"(ncols)
                 : "memory");
}

__device__ __forceinline__ void tmem_relinquish() {
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
                 : "memory");
}

__device__ __forceinline__ void tc_fence_before() {
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}

__device__ __forceinline__ void tc_fence_after() {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// D[tmem] (+)= A[smem desc] * B[smem desc]^T, FP16 inputs, FP32 accumulator.
__device__ __forceinline__ void tc_mma_f16(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                           uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
}

// Arrive once on `bar` when every tcgen05 operation this thread issued so far
// has completed.
__device__ __forceinline__ void tc_commit(uint64_t* bar) {
    asm volatile(
        "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
            smem_u32(bar))
        : "memory");
}

// Load 32 consecutive FP32 columns of this warp's 32 TMEM lanes (one lane per thread).
__device__ __forceinline__ void tmem_ld_32cols(uint32_t taddr, uint32_t (&r)[32]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
        "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
        "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
          "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
          "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]),
          "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]),
          "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// Load 16 consecutive FP32 columns of this warp's 32 TMEM lanes.
__device__ __forceinline__ void tmem_ld_16cols(uint32_t taddr, uint32_t (&r)[16]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
        "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
          "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
          "=r"(r[14]), "=r"(r[15])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// Store 16 consecutive FP32 columns of this warp's 32 TMEM lanes and wait for
// the store to complete.
__device__ __forceinline__ void tmem_st_16cols(uint32_t taddr, const uint32_t (&r)[16]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "
        "{%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16};" ::"r"(taddr),
        "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]),
        "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])
        : "memory");
    asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

// Shared-memory matrix descriptor for a K-major tile written by TMA with
// 128-byte swizzling: rows of 64 FP16 (128 B), 8-row groups 1024 B apart.
// Fields: start address >> 4 (bits 0-13), leading byte offset >> 4 = 1
// (bits 16-29, unused for this layout), stride byte offset >> 4 = 64
// (bits 32-45), descriptor version 1 (bits 46-47), base offset 0, swizzle
// mode 2 = 128 B (bits 61-63).
__device__ __forceinline__ uint64_t smem_desc_k128(uint32_t smem_addr) {
    uint64_t d = 0;
    d |= static_cast<uint64_t>((smem_addr & 0x3FFFFu) >> 4);
    d |= static_cast<uint64_t>(1) << 16;
    d |= static_cast<uint64_t>(1024 >> 4) << 32;
    d |= static_cast<uint64_t>(1) << 46;
    d |= static_cast<uint64_t>(2) << 61;
    return d;
}

// Instruction descriptor of tcgen05.mma kind::f16: FP32 accumulator (bits 4-5
// = 1), A and B FP16 (bits 7-9 and 10-12 = 0), both K-major (bits 15, 16 = 0),
// N >> 3 in bits 17-22, M >> 4 in bits 24-28.
__host__ __device__ constexpr uint32_t idesc_f16_f32(uint32_t m, uint32_t n) {
    return (1u << 4) | ((n >> 3) << 17) | ((m >> 4) << 24);
}

// ------------------------------------------------------------------ plain loads

// 16-byte streaming load that skips L1 (weights are read exactly once) and
// asks L2 to fetch the surrounding 256 bytes, which the same warp reads next.
__device__ __forceinline__ uint4 ld_stream_16B(const void* p) {
    uint4 v;
    asm volatile("ld.global.nc.L1::no_allocate.L2::256B.v4.u32 {%0, %1, %2, %3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "l"(p));
    return v;
}

}  // namespace mrt
