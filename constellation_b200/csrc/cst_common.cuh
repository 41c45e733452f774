// Device helpers shared by the sm_100a kernels of the MoE hot path.
//
//  * TMA bulk copies (cp.async.bulk global -> shared, completion on an mbarrier) and
//    the mbarrier primitives that pace the producer/consumer stage rings.  Every wait
//    is bounded (wall clock or poll count): on timeout it records CST_DEV_ERR_TIMEOUT in
//    the context's device error word and returns false, so a broken pipeline ends the
//    kernel with a status the host can read instead of hanging the GPU.
//  * tcgen05 helpers: TMEM alloc/dealloc, kind::f8f6f4 MMA with smem descriptors,
//    commit to mbarriers, TMEM loads and the tcgen05 fences.
//  * E4M3 encode/decode used by the activation packer.
#pragma once

#include <cstdint>
#include <cuda_fp8.h>
#include <cuda_runtime.h>

namespace cst {

constexpr int kBlock = 128;          // FP8 scale block (rows and cols) = weight rows per item
constexpr int kKStep = 32;           // K of one tcgen05.mma kind::f8f6f4
constexpr int kSplits = 3;           // E4M3 terms per activation element
constexpr int kTileCols = 8;         // tokens per n-tile
constexpr int kMaxTilesPerGroup = 2; // routed groups carry at most 16 rows
constexpr int kGroupRows = kMaxTilesPerGroup * kTileCols;
constexpr int kPrefillMaxTiles = 16;  // prefill groups carry at most 128 rows
constexpr int kPrefillGroupRows = kPrefillMaxTiles * kTileCols;
// B bytes of one n-tile for one 128-wide K block: 3 terms x 8 rows x 128 bytes
constexpr int kBTileBytes = kSplits * kTileCols * kBlock;  // 3072
// Activation scales of one n-tile for one K block: a power of two per (term, token)
constexpr int kScalesPerTile = kSplits * kTileCols;  // 24

// Device error word values (written with atomicMax so the first/most severe sticks).
constexpr int CST_DEV_OK = 0;
constexpr int CST_DEV_ERR_TIMEOUT = 1;
constexpr int CST_DEV_ERR_BOUNDS = 2;

constexpr uint32_t kSpinLimit = 1u << 26;

// Programmatic dependent launch.  Kernels of the layer chain are launched with the
// programmatic-stream-serialization attribute (launch_chained in kernels.h), so a kernel
// may become resident while its predecessor on the stream still runs.  Each such kernel
// calls chain_wait() before its first global-memory access -- it returns once every
// prerequisite grid has completed and its writes are visible -- and then chain_release(),
// which lets the next kernel of the chain start its own prologue.  Before chain_wait() a
// kernel touches only shared memory, TMEM and its parameters.  Launched without the
// attribute, both are no-ops.
__device__ __forceinline__ void chain_wait() { asm volatile("griddepcontrol.wait;\n" ::: "memory"); }
__device__ __forceinline__ void chain_release() { asm volatile("griddepcontrol.launch_dependents;\n" ::: "memory"); }

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;\n" ::"r"(smem_u32(bar)), "r"(count));
}

__device__ __forceinline__ void fence_barrier_init() {
    asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
}

__device__ __forceinline__ void fence_proxy_async_smem() {
    asm volatile("fence.proxy.async.shared::cta;\n" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;\n" ::"r"(smem_u32(bar)),
                 "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];\n" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n"
        ".reg .pred p;\n"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n"
        "selp.u32 %0, 1, 0, p;\n"
        "}\n"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

__device__ __forceinline__ uint64_t global_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

// Bounded wait on an mbarrier phase: gives up after kWaitLimitNs of wall time (checked
// every 256 polls) or kSpinLimit polls, whichever comes first.  Returns false and flags
// the error word on timeout.
constexpr uint64_t kWaitLimitNs = 4000000000ull;
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, int* err) {
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = global_ns();
    for (uint32_t i = 1; i < kSpinLimit; ++i) {
        if (mbar_try_wait(bar, parity)) return true;
        if ((i & 255u) == 0u && global_ns() - t0 > kWaitLimitNs) break;
    }
    if (err != nullptr) atomicMax(err, CST_DEV_ERR_TIMEOUT);
    return false;
}

// 1-D bulk copy global -> shared; completes `bytes` of transaction count on `bar`.
// Source and destination must be 16-byte aligned and `bytes` a multiple of 16.
__device__ __forceinline__ void tma_bulk_g2s(void* smem_dst, const void* gmem_src, uint32_t bytes,
                                             uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];\n" ::"r"(
            smem_u32(smem_dst)),
        "l"(gmem_src), "r"(bytes), "r"(smem_u32(bar))
        : "memory");
}

// ---- tcgen05 (5th-generation tensor cores, accumulators in tensor memory) ----------------

// Shared-memory matrix descriptor: K-major operand in 128-byte swizzled 8-row atoms
// (rows of 128 bytes, 16-byte chunk c of row r stored at c ^ (r & 7), atoms 1024 B apart).
// start address >> 4 in bits [0,14), leading byte offset 16 B (unused for swizzled
// K-major), stride byte offset 1024 B in bits [32,46), descriptor version 1 (bits 46-47),
// layout SWIZZLE_128B = 2 in bits [61,64).  The operand buffer must be 1024-byte aligned.
__device__ __forceinline__ uint64_t umma_desc_sw128(uint32_t saddr) {
    uint64_t d = uint64_t((saddr & 0x3FFFFu) >> 4);
    d |= uint64_t(1) << 16;
    d |= uint64_t(1024 >> 4) << 32;
    d |= uint64_t(1) << 46;
    d |= uint64_t(2) << 61;
    return d;
}

// Instruction descriptor, kind::f8f6f4: D fp32 (bits 4-5 = 1), A and B E4M3 (bits 7-9,
// 10-12 = 0), both K-major, N >> 3 in bits [17,23), M >> 4 in bits [24,29).
__host__ __device__ constexpr uint32_t umma_idesc_e4m3(int M, int N) {
    return (1u << 4) | (uint32_t(N >> 3) << 17) | (uint32_t(M >> 4) << 24);
}

// Instruction descriptor, kind::f16 with bf16 A and B (bits 7-9, 10-12 = 1), fp32 D, both
// K-major.  (A and B always carry the same type.)
__host__ __device__ constexpr uint32_t umma_idesc_bf16(int M, int N) {
    return (1u << 4) | (1u << 7) | (1u << 10) | (uint32_t(N >> 3) << 17) | (uint32_t(M >> 4) << 24);
}

__device__ __forceinline__ void tmem_alloc(uint32_t* smem_dst, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;\n" ::"r"(smem_u32(smem_dst)),
                 "r"(ncols)
                 : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;\n" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;\n" ::"r"(taddr), "r"(ncols) : "memory");
}
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;\n" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;\n" ::: "memory"); }

// Arrive (once) on `bar` when every tcgen05 operation this thread issued so far completes.
__device__ __forceinline__ void tc_commit(uint64_t* bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];\n" ::"r"(
                     smem_u32(bar))
                 : "memory");
}

// D[tmem] (+)= A[smem desc] x B[smem desc], E4M3 x E4M3 -> fp32, issued by one thread.
__device__ __forceinline__ void tc_mma_e4m3(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                            uint32_t accumulate) {
    const uint32_t z = 0u;
    asm volatile(
        "{\n"
        ".reg .pred p;\n"
        "setp.ne.b32 p, %4, 0;\n"
        "tcgen05.mma.cta_group::1.kind::f8f6f4 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n"
        "}\n" ::"r"(d_tmem),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate), "r"(z), "r"(z), "r"(z), "r"(z)
        : "memory");
}

// D[tmem] (+)= A[smem desc] x B[smem desc], bf16 x bf16 -> fp32 (K = 16), issued by one thread.
__device__ __forceinline__ void tc_mma_bf16(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                            uint32_t accumulate) {
    const uint32_t z = 0u;
    asm volatile(
        "{\n"
        ".reg .pred p;\n"
        "setp.ne.b32 p, %4, 0;\n"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n"
        "}\n" ::"r"(d_tmem),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate), "r"(z), "r"(z), "r"(z), "r"(z)
        : "memory");
}

// 16 consecutive 32-bit columns of this thread's TMEM lane (warp w reads lanes 32(w%4)..+31).
// The registers are valid only after tmem_wait_ld() and tmem_reg_fence().
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t* r) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];\n"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr));
}
__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;\n" ::: "memory"); }
// Orders every later use of r after the preceding tmem_wait_ld (volatile asms keep their order).
template <int N>
__device__ __forceinline__ void tmem_reg_fence(uint32_t (&r)[N]) {
#pragma unroll
    for (int i = 0; i < N; ++i) asm volatile("" : "+r"(r[i]));
}

// E4M3 round-to-nearest-even with saturation to +-448 (hardware cvt).
__device__ __forceinline__ uint8_t e4m3_rn(float v) {
    return static_cast<uint8_t>(__nv_cvt_float_to_fp8(v, __NV_SATFINITE, __NV_E4M3));
}

__device__ __forceinline__ float e4m3_to_f32(uint8_t b) {
    __half_raw h = __nv_cvt_fp8_to_halfraw(static_cast<__nv_fp8_storage_t>(b), __NV_E4M3);
    return __half2float(__half(h));
}

// Two floats -> two E4M3 bytes in one conversion, `lo` in bits 0..7 (as e4m3_rn each).
__device__ __forceinline__ uint32_t e4m3x2_rn(float lo, float hi) {
    return __nv_cvt_float2_to_fp8x2(make_float2(lo, hi), __NV_SATFINITE, __NV_E4M3);
}

// The two E4M3 bytes in bits 0..15 of b2 as floats, exactly; .x is bits 0..7.
__device__ __forceinline__ float2 e4m3x2_to_f32x2(uint32_t b2) {
    const __half2_raw h = __nv_cvt_fp8x2_to_halfraw2(static_cast<__nv_fp8x2_storage_t>(b2), __NV_E4M3);
    return __half22float2(__half2(h));
}

// Warp maximum of non-negative values in one reduction: the bit patterns of non-negative
// floats order as unsigned integers.  A NaN lane counts as 0, so the result is fmaxf's over
// the other lanes (0 when every lane is NaN, where fmaxf gives NaN; pow2_scale_for maps
// both to 1).
__device__ __forceinline__ float warp_max_nonneg(float a) {
    const uint32_t u = (a == a) ? __float_as_uint(a) : 0u;
    return __uint_as_float(__reduce_max_sync(0xffffffffu, u));
}

// Smallest power of two s with amax / s <= 448 (s = 1 for amax == 0).  Returns s.
__device__ __forceinline__ float pow2_scale_for(float amax) {
    if (!(amax > 0.0f)) return 1.0f;
    const float t = amax * (1.0f / 448.0f);
    uint32_t bits = __float_as_uint(t);
    // round t up to a power of two: clear the mantissa, bump the exponent if it was nonzero
    const uint32_t mant = bits & 0x007FFFFFu;
    uint32_t e = bits & 0x7F800000u;
    if (e == 0) return 1.1754943508222875e-38f * 1.0f;  // tiny amax: smallest normal
    if (mant != 0) e += 0x00800000u;
    if (e >= 0x7F800000u) e = 0x7F000000u;
    return __uint_as_float(e);
}

// 1 / s, exactly, for a power of two s from pow2_scale_for (2^-126 .. 2^127): the exponent
// reflected about 2^0 (2^-127, a subnormal, for s = 2^127).
__device__ __forceinline__ float pow2_recip(float s) {
    const uint32_t b = __float_as_uint(s);
    return b >= 0x7F000000u ? __uint_as_float(0x00400000u) : __uint_as_float(0x7F000000u - b);
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

}  // namespace cst
