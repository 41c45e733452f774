// Fused sigmoid group-limited top-k router for a batch of tokens.
//
// Restates route_token_real (server/moe_layer_runtime.py:232-408) for T tokens at once:
//   logits = gate_weight @ x        fp32, fixed summation order        (:322)
//   scores = sigmoid(logits)                                             (:323)
//   choice = scores + e_score_correction_bias, -inf where not resident   (:325-340)
//   group score = sum of the top-2 choice values of each group          (:343-345)
//   keep the topk_group best groups, choose top_k experts among them    (:347-371)
//   weight = unbiased score / (sum + 1e-20) * routed_scaling_factor     (:373-381)
// Every selection orders candidates by (value desc, index asc), so equal values go to
// the lowest index; the k experts of a token are returned in that order.
//
// Two kernels:
//   router_logits_kernel: [T, H] x [E, H]^T in fp32 on CUDA cores (the router needs exact
//     fp32 products; TF32 tensor cores would change which experts win).  4-token x 8-expert
//     tiles, one per CTA, K split over the CTA's warps and folded in a fixed order, so
//     results are bit-identical from run to run; logits [T, E] are written once.
//   router_select_kernel: one warp per token does the sigmoid / bias / group / top-k
//     logic with warp-shuffle arg-max reductions.
// Large bf16 batches take the logits on the tensor cores instead (router_split_w_kernel +
// router_logits_tc_kernel below: W split exactly into three bf16 terms, fp32 fold per K
// block), and decode-sized batches select with one CTA per token
// (router_select_rank_kernel).
#include <cfloat>
#include <cstdint>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <algorithm>
#include <cudaTypedefs.h>
#include <mutex>

#include "cst_common.cuh"
#include "kernels.h"

namespace cst {

template <typename T>
__device__ __forceinline__ float to_f32(T v);
template <>
__device__ __forceinline__ float to_f32<float>(float v) { return v; }
template <>
__device__ __forceinline__ float to_f32<__nv_bfloat16>(__nv_bfloat16 v) { return __bfloat162float(v); }
template <>
__device__ __forceinline__ float to_f32<__half>(__half v) { return __half2float(v); }

// 4 consecutive activations of one row as fp32 (8- or 16-byte vector load).
template <typename TX>
__device__ __forceinline__ float4 load4x(const TX* x, int64_t off);
template <>
__device__ __forceinline__ float4 load4x<float>(const float* x, int64_t off) {
    return __ldg(reinterpret_cast<const float4*>(x + off));
}
template <>
__device__ __forceinline__ float4 load4x<__nv_bfloat16>(const __nv_bfloat16* x, int64_t off) {
    const uint2 u = __ldg(reinterpret_cast<const uint2*>(x + off));
    return make_float4(__uint_as_float(u.x << 16), __uint_as_float(u.x & 0xffff0000u), __uint_as_float(u.y << 16),
                       __uint_as_float(u.y & 0xffff0000u));
}
template <>
__device__ __forceinline__ float4 load4x<__half>(const __half* x, int64_t off) {
    const uint2 u = __ldg(reinterpret_cast<const uint2*>(x + off));
    const float2 a = __half22float2(*reinterpret_cast<const __half2*>(&u.x));
    const float2 b = __half22float2(*reinterpret_cast<const __half2*>(&u.y));
    return make_float4(a.x, a.y, b.x, b.y);
}

constexpr int kLT = 4;       // tokens per CTA tile
constexpr int kLE = 8;       // experts per CTA tile
constexpr int kLWarps = 4;   // warps per CTA, each over a contiguous quarter of K

// Butterfly half-exchange: after the step with offset o, each lane keeps the half of its
// N values selected by lane bit o and adds the partner's copy of that half.
template <int N>
__device__ __forceinline__ void reduce_half(float* v, int o, int lane) {
    const bool upper = (lane & o) != 0;
#pragma unroll
    for (int i = 0; i < N / 2; ++i) {
        const float keep = upper ? v[i + N / 2] : v[i];
        const float send = upper ? v[i] : v[i + N / 2];
        v[i] = keep + __shfl_xor_sync(0xffffffffu, send, o);
    }
}

// logits[t][e] = sum_k x[t][k] * w[e][k] in fp32 for a 4-token x 8-expert tile per CTA.
// Warp q sums k in [q H/4, (q+1) H/4) with lane l taking columns k = 4 l + 128 j: per step
// one float4 of each expert row and 4 activations of each token row, 128 independent FMA.
// The 32 per-lane sums are folded across the warp by a fixed butterfly (lane l ends with
// output l) and the four warps' sums are added in warp order, so the result is
// bit-identical from run to run.  No global scratch: the tile is written once.  The tile
// keeps a thread under 128 registers, so 4 CTAs fit an SM and a 64-token call's 512 CTAs
// run in one wave with 16 warps per SM hiding each other's load latency.
template <typename TX>
__global__ void __launch_bounds__(kLWarps * 32, 4) router_logits_kernel(const TX* __restrict__ x,
                                                                        const float* __restrict__ w,
                                                                        float* __restrict__ logits, int T, int E,
                                                                        int H) {
    __shared__ float s_part[kLWarps][kLT * kLE];
    chain_wait();
    chain_release();
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int t0 = blockIdx.x * kLT;
    const int e0 = blockIdx.y * kLE;
    const int quarter = H / kLWarps;
    const int k_begin = warp * quarter;
    const int k_end = k_begin + quarter;
    float acc[kLT * kLE];
#pragma unroll
    for (int i = 0; i < kLT * kLE; ++i) acc[i] = 0.0f;
    const TX* xr[kLT];
    const float* wr[kLE];
#pragma unroll
    for (int t = 0; t < kLT; ++t) xr[t] = x + int64_t(min(t0 + t, T - 1)) * H;
#pragma unroll
    for (int e = 0; e < kLE; ++e) wr[e] = w + int64_t(min(e0 + e, E - 1)) * H;
    for (int k = k_begin + 4 * lane; k < k_end; k += 128) {
        float4 wv[kLE], xv[kLT];
#pragma unroll
        for (int e = 0; e < kLE; ++e) wv[e] = __ldg(reinterpret_cast<const float4*>(wr[e] + k));
#pragma unroll
        for (int t = 0; t < kLT; ++t) xv[t] = load4x<TX>(xr[t], k);
#pragma unroll
        for (int t = 0; t < kLT; ++t) {
#pragma unroll
            for (int e = 0; e < kLE; ++e) {
                float a = acc[t * kLE + e];
                a = fmaf(xv[t].x, wv[e].x, a);
                a = fmaf(xv[t].y, wv[e].y, a);
                a = fmaf(xv[t].z, wv[e].z, a);
                a = fmaf(xv[t].w, wv[e].w, a);
                acc[t * kLE + e] = a;
            }
        }
    }
    reduce_half<32>(acc, 16, lane);
    reduce_half<16>(acc, 8, lane);
    reduce_half<8>(acc, 4, lane);
    reduce_half<4>(acc, 2, lane);
    reduce_half<2>(acc, 1, lane);
    s_part[warp][lane] = acc[0];
    __syncthreads();
    if (threadIdx.x < kLT * kLE) {
        const int o = threadIdx.x;
        float sum = s_part[0][o];
#pragma unroll
        for (int q = 1; q < kLWarps; ++q) sum += s_part[q][o];
        const int t = t0 + o / kLE, e = e0 + o % kLE;
        if (t < T && e < E) logits[int64_t(t) * E + e] = sum;
    }
}

// ---- tensor-core logits (bf16 activations) --------------------------------------------
// logits = x W^T with W fp32 split EXACTLY into three bf16 terms, W = W1 + W2 + W3
// (W1 = bf16(W), W2 = bf16(W - W1), W3 = W - W1 - W2: fp32's 24 significant bits are three
// times bf16's 8), so every product x * Wi is exact.  tcgen05.mma kind::f16 (bf16 x bf16 ->
// fp32, K = 16): M = 128 experts per CTA (A = the W terms), N = up to 128 tokens (B = x).
// K is walked in 64-wide blocks (one 128-byte swizzled row).  Each block accumulates into a
// fresh TMEM buffer (4 k-steps x 3 terms) and every thread adds its expert row of that
// buffer into fp32 registers -- the tensor core's internal accumulation never spans more
// than one block, so the result matches an fp32 FMA chain to within summation-order
// rounding.  CTAs along grid.z take disjoint K ranges and write partial logits [z][T][E];
// the selection kernel adds the partials in z order.
//
// Two launches per call:
//   router_split_w_kernel: the three terms of W, once per call, written as the very bytes
//     the MMAs read from shared memory -- per (128-expert tile, K block) 3 x 16 KB, rows of
//     128 bytes with the 128-byte swizzle -- so a CTA copies a block's 48 KB of A operand
//     as one contiguous run instead of converting it again (every token tile used to).
//   router_logits_tc_kernel: kRtStages shared-memory stages filled by cp.async, each
//     thread copying its share of block j + kRtStages - 1 while the MMAs of block j run and
//     it folds block j - 1; x rows are copied into their swizzled places, rows past T
//     zero-filled.  Two TMEM buffers alternate between the MMAs of one block and the fold
//     of the previous one.
constexpr int kRtThreads = 128;
constexpr int kRtKB = 64;                        // bf16 per 128-byte row
constexpr int kRtATerm = 128 * 128;              // bytes of one W term tile (128 rows x 128 B)
constexpr int kRtWBytes = 3 * kRtATerm;          // the three terms of one (expert tile, K block)
constexpr int kRtMaxN = 128;
constexpr int kRtStage = kRtWBytes + kRtMaxN * 128;  // 64 KB
constexpr int kRtStages = 3;
constexpr size_t kRtSmem = size_t(kRtStages) * kRtStage + 1024 + 64;  // + barriers, TMEM slot

__device__ __forceinline__ uint32_t bf16_pair(float a, float b) {
    const __nv_bfloat162 v = __floats2bfloat162_rn(a, b);
    return *reinterpret_cast<const uint32_t*>(&v);
}

// 16-byte asynchronous global -> shared copy; src_bytes 0 fills the 16 bytes with zeros
__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src, uint32_t src_bytes) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(dst), "l"(src), "r"(src_bytes) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
    asm volatile("cp.async.wait_group %0;\n" ::"n"(N) : "memory");
}

// W [E, H] fp32 -> image[((et * (H / 64) + kb) * 3 + term) * 16 KB + r * 128 + ((c ^ (r & 7)) << 4)]
// = the 8 bf16 of term `term` of W[et * 128 + r][kb * 64 + c * 8 .. + 8].  One thread per
// 8 consecutive weights of a row: 32 bytes read, 16 bytes written per term.
__global__ void __launch_bounds__(256) router_split_w_kernel(const float* __restrict__ w, uint8_t* __restrict__ img,
                                                             int E, int H) {
    chain_wait();
    chain_release();
    const int cpr = H / 8;  // 8-column chunks per row
    const int kbn = H / kRtKB;
    const int64_t n = int64_t(E) * cpr;
    for (int64_t q = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; q < n; q += int64_t(gridDim.x) * blockDim.x) {
        const int e = static_cast<int>(q / cpr);
        const int c8 = static_cast<int>(q - int64_t(e) * cpr);
        const float4* src = reinterpret_cast<const float4*>(w + int64_t(e) * H + c8 * 8);
        const float4 p = __ldg(src), s = __ldg(src + 1);
        const float v[8] = {p.x, p.y, p.z, p.w, s.x, s.y, s.z, s.w};
        uint32_t t1[4], t2[4], t3[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const float a = v[2 * i], b = v[2 * i + 1];
            const float a1 = __bfloat162float(__float2bfloat16_rn(a));
            const float b1 = __bfloat162float(__float2bfloat16_rn(b));
            const float ra = a - a1, rb = b - b1;
            const float a2 = __bfloat162float(__float2bfloat16_rn(ra));
            const float b2 = __bfloat162float(__float2bfloat16_rn(rb));
            t1[i] = bf16_pair(a1, b1);
            t2[i] = bf16_pair(a2, b2);
            t3[i] = bf16_pair(ra - a2, rb - b2);
        }
        const int et = e >> 7, r = e & 127, kb = c8 >> 3, c = c8 & 7;
        uint8_t* dst = img + (int64_t(et) * kbn + kb) * kRtWBytes + r * 128 + ((c ^ (r & 7)) << 4);
        *reinterpret_cast<uint4*>(dst) = make_uint4(t1[0], t1[1], t1[2], t1[3]);
        *reinterpret_cast<uint4*>(dst + kRtATerm) = make_uint4(t2[0], t2[1], t2[2], t2[3]);
        *reinterpret_cast<uint4*>(dst + 2 * kRtATerm) = make_uint4(t3[0], t3[1], t3[2], t3[3]);
    }
}

__global__ void __launch_bounds__(kRtThreads, 1) router_logits_tc_kernel(const __nv_bfloat16* __restrict__ x,
                                                                        const uint8_t* __restrict__ wimg,
                                                                        float* __restrict__ part, int T, int E,
                                                                        int H, int N, int nb, int* err) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t* bar = reinterpret_cast<uint64_t*>(smem + kRtStages * kRtStage);  // MMAs of even / odd blocks
    uint64_t* full = bar + 2;                                                   // W bytes of each stage
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(full + kRtStages);
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int t0 = blockIdx.x * N;
    const int e0 = blockIdx.y * 128;
    const int kb0 = blockIdx.z * nb;
    if (tid == 0) {
        mbar_init(&bar[0], 1);
        mbar_init(&bar[1], 1);
        for (int s = 0; s < kRtStages; ++s) mbar_init(&full[s], 1);
        fence_barrier_init();
    }
    if (warp == 0) {
        tmem_alloc(tmem_slot, 2 * kRtMaxN);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    chain_wait();
    chain_release();
    const uint32_t lane_addr = uint32_t(warp * 32) << 16;
    const uint32_t idesc = umma_idesc_bf16(128, N);
    const uint8_t* wblk = wimg + (int64_t(blockIdx.y) * (H / kRtKB) + kb0) * kRtWBytes;  // this CTA's block 0
    // This thread's 16-byte pieces of every x tile, fixed for all K blocks: piece m is row
    // r = q / 8, chunk c = q % 8 of the tile (q = tid + 128 m), placed at its swizzled chunk;
    // rows past T read 0 bytes (zero fill) from a valid address.
    constexpr int kXPer = kRtMaxN * 8 / kRtThreads;
    const int nx = N / 16;  // pieces per thread of an N-row tile (N a multiple of 16)
    const __nv_bfloat16* xsrc[kXPer];
    uint32_t xdst[kXPer];
    uint32_t xin = 0;
#pragma unroll
    for (int m = 0; m < kXPer; ++m) {
        const int q = tid + kRtThreads * m, r = q >> 3, c = q & 7, t = t0 + r;
        const bool in = m < nx && t < T;
        xsrc[m] = x + int64_t(in ? t : 0) * H + c * 8;
        xdst[m] = kRtWBytes + r * 128 + ((c ^ (r & 7)) << 4);
        xin |= (in ? 1u : 0u) << m;
    }
    int issued = -1, waited = -1;  // thread 0: last block whose W copy was issued / seen landed
    // block j into stage j % kRtStages (nothing past the CTA's last block): thread 0 copies its
    // 48 KB of W terms in one bulk copy onto the stage's barrier, every thread its x pieces
    // with cp.async; one cp.async group per call, so group j is block j's
    auto issue = [&](int j) {
        if (j < nb) {
            const int s = j % kRtStages;
            uint8_t* st = smem + s * kRtStage;
            if (tid == 0) {
                mbar_arrive_expect_tx(&full[s], kRtWBytes);
                tma_bulk_g2s(st, wblk + int64_t(j) * kRtWBytes, kRtWBytes, &full[s]);
                issued = j;
            }
            const int k0 = (kb0 + j) * kRtKB;
            const uint32_t sb = smem_u32(st);
#pragma unroll
            for (int m = 0; m < kXPer; ++m)
                if (m < nx) cp_async16(sb + xdst[m], xsrc[m] + k0, ((xin >> m) & 1u) ? 16u : 0u);
        }
        cp_async_commit();
    };
    float acc[kRtMaxN];
#pragma unroll
    for (int i = 0; i < kRtMaxN; ++i) acc[i] = 0.0f;
    bool ok = true;
    // fold the finished block jj (its MMAs committed to bar[jj & 1]) into acc, 32 columns per
    // wait (the upper 16 of a pair past N are read, as garbage, and not used)
    auto fold = [&](int jj) {
        if (!mbar_wait(&bar[jj & 1], (jj >> 1) & 1u, err)) ok = false;
        tc_fence_after();
        const uint32_t base = tmem + lane_addr + (jj & 1) * kRtMaxN;
#pragma unroll
        for (int c0 = 0; c0 < kRtMaxN; c0 += 32) {
            if (c0 < N) {
                uint32_t d[32];
                tmem_ld16(base + c0, d);
                tmem_ld16(base + c0 + 16, d + 16);
                tmem_wait_ld();
                tmem_reg_fence(d);
#pragma unroll
                for (int i = 0; i < 16; ++i) acc[c0 + i] += __uint_as_float(d[i]);
                if (c0 + 16 < N) {
#pragma unroll
                    for (int i = 0; i < 16; ++i) acc[c0 + 16 + i] += __uint_as_float(d[16 + i]);
                }
            }
        }
        tc_fence_before();
    };
#pragma unroll 1
    for (int j = 0; j < kRtStages - 1; ++j) issue(j);
    int committed = -1;  // last block whose MMAs were committed
    for (int j = 0; j < nb; ++j) {
        cp_async_wait<kRtStages - 2>();  // this thread's x pieces of block j (group j) have landed
        fence_proxy_async_smem();        // the tensor cores read what cp.async just wrote
        if (tid == 0) {
            if (mbar_wait(&full[j % kRtStages], (j / kRtStages) & 1u, err)) waited = j;
            else ok = false;
        }
        if (__syncthreads_or(!ok)) break;
        if (tid == 0) {
            tc_fence_after();
            const uint32_t sa = smem_u32(smem + (j % kRtStages) * kRtStage);
#pragma unroll
            for (int ks = 0; ks < 4; ++ks) {
                const uint64_t bdesc = umma_desc_sw128(sa + kRtWBytes + ks * 32);
#pragma unroll
                for (int term = 0; term < 3; ++term) {
                    const uint64_t adesc = umma_desc_sw128(sa + term * kRtATerm + ks * 32);
                    tc_mma_bf16(tmem + (j & 1) * kRtMaxN, adesc, bdesc, idesc, (ks > 0 || term > 0) ? 1u : 0u);
                }
            }
            tc_commit(&bar[j & 1]);
        }
        committed = j;
        // block j - 1's MMAs are complete once its fold has waited for them, so its stage
        // takes block j + kRtStages - 1
        if (j > 0) fold(j - 1);
        issue(j + kRtStages - 1);
    }
    // nothing in flight at exit: x pieces, W bulk copies not yet seen landed, the MMAs
    cp_async_wait<0>();
    if (tid == 0)
        for (int b = waited + 1; b <= issued; ++b) mbar_wait(&full[b % kRtStages], (b / kRtStages) & 1u, err);
    if (ok && committed == nb - 1 && nb > 0) fold(nb - 1);
    else if (committed >= 0) mbar_wait(&bar[committed & 1], (committed >> 1) & 1u, err);
    if (__syncthreads_and(ok && committed == nb - 1)) {
        const int e = e0 + warp * 32 + lane;
        float* out = part + int64_t(blockIdx.z) * T * E;
#pragma unroll
        for (int i = 0; i < kRtMaxN; ++i) {
            const int t = t0 + i;
            if (i < N && t < T) out[int64_t(t) * E + e] = acc[i];
        }
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == 0) tmem_dealloc(tmem, 2 * kRtMaxN);
}

struct RouterArgs {
    const float* logits;    // [ks][T][E] partial logits over disjoint K ranges
    int ks;
    const float* bias;      // [E]
    const uint8_t* resident;  // [E] or null (all resident)
    int T, E, n_group, topk_group, top_k, norm;
    float scale;
    int32_t* topk_idx;      // [T, top_k]
    float* topk_w;          // [T, top_k]
    float* group_scores_out;  // [T, n_group] or null
    float* logits_out;        // [T, E] summed logits or null (the caller's aux copy)
};

// Warp arg-max with (value desc, index asc); inactive candidates carry idx = INT_MAX.
__device__ __forceinline__ void warp_argmax(float& v, int& idx) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, v, o);
        const int oi = __shfl_xor_sync(0xffffffffu, idx, o);
        if (ov > v || (ov == v && oi < idx)) {
            v = ov;
            idx = oi;
        }
    }
}

constexpr int kSelWarps = 4;
constexpr int kMaxE = 1024;

// Warp top-2 of (a >= b) pairs: merge with the partner lane's pair.
__device__ __forceinline__ void warp_top2(float& a, float& b) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const float oa = __shfl_xor_sync(0xffffffffu, a, o);
        const float ob = __shfl_xor_sync(0xffffffffu, b, o);
        const float hi = fmaxf(a, oa);
        const float lo = fmaxf(fminf(a, oa), fmaxf(b, ob));
        a = hi;
        b = lo;
    }
}

// One warp per token.  Lane l holds experts e = l + 32 i (i < EPL) in registers; the
// selection rounds touch only registers and warp shuffles.
template <int EPL>
__global__ void __launch_bounds__(kSelWarps * 32) router_select_kernel(RouterArgs a) {
    __shared__ float s_choice[kSelWarps][EPL * 32];
    __shared__ float s_score[kSelWarps][EPL * 32];
    chain_wait();
    chain_release();
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int t = blockIdx.x * kSelWarps + warp;
    if (t >= a.T) return;
    const int E = a.E;
    const int epg = E / a.n_group;
    const float* __restrict__ lg = a.logits + int64_t(t) * E;
    const int64_t zs = int64_t(a.T) * E;
    float ch[EPL];
    int grp[EPL];
#pragma unroll
    for (int i = 0; i < EPL; ++i) {
        const int e = lane + 32 * i;
        ch[i] = -INFINITY;
        grp[i] = 0x7fffffff;
        if (e < E) {
            float l = lg[e];
            for (int z = 1; z < a.ks; ++z) l += lg[z * zs + e];  // K ranges in order
            if (a.logits_out) a.logits_out[int64_t(t) * E + e] = l;
            const float sg = 1.0f / (1.0f + expf(-l));
            const bool res = (a.resident == nullptr) || (a.resident[e] != 0);
            ch[i] = res ? (sg + a.bias[e]) : -INFINITY;
            s_choice[warp][e] = ch[i];
            s_score[warp][e] = res ? sg : 0.0f;
            grp[i] = e / epg;
        }
    }
    __syncwarp();
    // group scores: sum of the two largest choice values of each group
    float gs = -INFINITY;  // lane g < n_group ends up holding group g's score
    if (epg == 32 && (E & 31) == 0) {
        // group g is exactly register row i = g: a warp top-2 per row
#pragma unroll
        for (int i = 0; i < EPL; ++i) {
            if (i < a.n_group) {
                float m1 = ch[i], m2 = -INFINITY;
                warp_top2(m1, m2);
                if (lane == i) gs = m1 + m2;
            }
        }
    } else if (lane < a.n_group) {
        float m1 = -INFINITY, m2 = -INFINITY;
        for (int j = 0; j < epg; ++j) {
            const float v = s_choice[warp][lane * epg + j];
            if (v > m1) {
                m2 = m1;
                m1 = v;
            } else if (v > m2) {
                m2 = v;
            }
        }
        gs = m1 + m2;
    }
    if (lane < a.n_group && a.group_scores_out) a.group_scores_out[int64_t(t) * a.n_group + lane] = gs;
    // keep the topk_group best groups (value desc, index asc)
    uint32_t gmask = 0u;
    {
        bool used = lane >= a.n_group;
        for (int r = 0; r < a.topk_group; ++r) {
            float bv = used ? -INFINITY : gs;
            int bi = used ? 0x7fffffff : lane;
            warp_argmax(bv, bi);
            gmask |= 1u << bi;
            if (lane == bi) used = true;
        }
    }
    // candidates: choice values of experts in kept groups, -inf elsewhere
    float cand[EPL];
#pragma unroll
    for (int i = 0; i < EPL; ++i) cand[i] = (grp[i] < 32 && ((gmask >> grp[i]) & 1u)) ? ch[i] : -INFINITY;
    // top_k rounds of warp arg-max over (value desc, index asc)
    uint32_t taken = 0u;
    float wsel = 0.0f;
    int isel = -1;
    float denom = 0.0f;
    for (int r = 0; r < a.top_k; ++r) {
        float bv = -INFINITY;
        int bi = 0x7fffffff;
#pragma unroll
        for (int i = 0; i < EPL; ++i) {
            const int e = lane + 32 * i;
            if (e < E && !((taken >> i) & 1u) && (cand[i] > bv || (cand[i] == bv && e < bi))) {
                bv = cand[i];
                bi = e;
            }
        }
        warp_argmax(bv, bi);
        if ((bi & 31) == lane) taken |= 1u << (bi >> 5);
        const float wv = s_score[warp][bi];
        denom += wv;  // sequential sum in selection order
        if (lane == r) {
            isel = bi;
            wsel = wv;
        }
    }
    if (lane < a.top_k) {
        float wv = wsel;
        if (a.norm && a.top_k > 1) wv = wv / (denom + 1e-20f);
        wv = wv * a.scale;
        a.topk_idx[int64_t(t) * a.top_k + lane] = isel;
        a.topk_w[int64_t(t) * a.top_k + lane] = wv;
    }
}

// One CTA per token, one thread per expert (blockDim = E rounded up to a warp).  The same
// arithmetic as router_select_kernel, reorganised so that no step is a long chain of
// dependent shuffles: group top-2 is one warp reduction per group (epg == 32) or a short
// scan, the kept groups and the top-k experts are found by RANK -- an entry's position in
// (value desc, index asc) order is the number of entries ahead of it -- and the k chosen
// experts are written in rank order.  The normaliser adds the chosen unbiased scores in
// that order, as the warp version does, so both give bit-identical results.
__global__ void __launch_bounds__(1024) router_select_rank_kernel(RouterArgs a) {
    __shared__ float s_choice[kMaxE];
    __shared__ float s_score[kMaxE];
    __shared__ float s_gs[32];
    __shared__ int s_keep[32];
    __shared__ int s_sel[16];
    chain_wait();
    chain_release();
    const int t = blockIdx.x;
    const int e = threadIdx.x;
    const int E = a.E;
    const int epg = E / a.n_group;
    const int lane = e & 31, warp = e >> 5;
    float ch = -INFINITY;
    if (e < E) {
        const float* lg = a.logits + int64_t(t) * E + e;
        const int64_t zs = int64_t(a.T) * E;
        float l = lg[0];
        for (int z0 = 1; z0 < a.ks; z0 += 16) {  // K ranges in order, 16 loads in flight
            float v[16];
#pragma unroll
            for (int i = 0; i < 16; ++i) v[i] = z0 + i < a.ks ? lg[(z0 + i) * zs] : 0.0f;
#pragma unroll
            for (int i = 0; i < 16; ++i)
                if (z0 + i < a.ks) l += v[i];
        }
        if (a.logits_out) a.logits_out[int64_t(t) * E + e] = l;
        const float sg = 1.0f / (1.0f + expf(-l));
        const bool res = (a.resident == nullptr) || (a.resident[e] != 0);
        ch = res ? (sg + a.bias[e]) : -INFINITY;
        s_choice[e] = ch;
        s_score[e] = res ? sg : 0.0f;
    }
    // group scores: sum of the two largest choice values of each group
    if (epg == 32 && (E & 31) == 0) {
        float m1 = ch, m2 = -INFINITY;
        warp_top2(m1, m2);
        if (lane == 0 && warp < a.n_group) s_gs[warp] = m1 + m2;
        __syncthreads();
    } else {
        __syncthreads();
        if (e < a.n_group) {
            float m1 = -INFINITY, m2 = -INFINITY;
            for (int j = 0; j < epg; ++j) {
                const float v = s_choice[e * epg + j];
                if (v > m1) {
                    m2 = m1;
                    m1 = v;
                } else if (v > m2) {
                    m2 = v;
                }
            }
            s_gs[e] = m1 + m2;
        }
        __syncthreads();
    }
    // keep the topk_group best groups (value desc, index asc)
    if (e < a.n_group) {
        const float g = s_gs[e];
        int rank = 0;
        for (int j = 0; j < a.n_group; ++j) {
            const float o = s_gs[j];
            rank += (o > g) || (o == g && j < e);
        }
        s_keep[e] = rank < a.topk_group;
        if (a.group_scores_out) a.group_scores_out[int64_t(t) * a.n_group + e] = g;
    }
    __syncthreads();
    // candidates: choice values of experts in kept groups, -inf elsewhere; rank each one
    if (e < E) s_choice[e] = s_keep[e / epg] ? ch : -INFINITY;
    __syncthreads();
    if (e < E) {
        const float c = s_choice[e];
        int rank = 0;
        for (int j = 0; j < E; ++j) {
            const float o = s_choice[j];
            rank += (o > c) || (o == c && j < e);
        }
        if (rank < a.top_k) s_sel[rank] = e;
    }
    __syncthreads();
    if (e < a.top_k) {
        float denom = 0.0f;
        for (int r = 0; r < a.top_k; ++r) denom += s_score[s_sel[r]];  // in selection order
        float wv = s_score[s_sel[e]];
        if (a.norm && a.top_k > 1) wv = wv / (denom + 1e-20f);
        wv = wv * a.scale;
        a.topk_idx[int64_t(t) * a.top_k + e] = s_sel[e];
        a.topk_w[int64_t(t) * a.top_k + e] = wv;
    }
}

// Tensor-core logits apply to bf16 activations with E a multiple of 128 and H of 64, from
// kRtMinTokens tokens on: below that the CUDA-core kernel is faster per call (graph
// replay, E = 256, H = 7168, measured: 64 tokens 25 us vs 33 us, 128 tokens 35 vs 37;
// 256 tokens 55 vs 35, 1024 tokens 156 vs 49, 2048 tokens 303 vs 85 the other way).
// K split: the grid (token tiles x expert tiles x ks) runs one CTA per SM at a time, so the
// critical path is ceil(CTAs / SMs) waves, each of H / 64 / ks K blocks plus the CTA's fixed
// cost (prologue, pipeline fill, partial-sum stores: about kRtCtaCostBlocks blocks,
// measured); ks is the divisor of the K blocks (each CTA keeping >= 2) with the shortest
// path, the smaller ks on a tie, and at most kRtMaxPartials partial floats (the selection
// adds them back).
constexpr int kRtMinTokens = 192;
constexpr int kRtSms = 148;
static bool router_tc_ok(int x_dtype, int T, int E, int H) {
    return x_dtype == 2 && T >= kRtMinTokens && E % 128 == 0 && H % kRtKB == 0;
}
static int router_tc_n(int T) { return T >= kRtMaxN ? kRtMaxN : ((T + 15) / 16) * 16; }  // token tile

int router_tc_split(int T, int E, int H, int64_t cap) {
    constexpr int64_t kRtCtaCostBlocks = 4;
    constexpr int64_t kRtMaxPartials = int64_t(1) << 22;
    const int nbt = H / kRtKB;
    const int N = router_tc_n(T);
    const int64_t base = int64_t((T + N - 1) / N) * (E / 128);
    const int64_t logits = int64_t(T) * E;
    cap = std::min(cap, std::max(logits, kRtMaxPartials));
    int best = 1;
    int64_t best_path = ((base + kRtSms - 1) / kRtSms) * (nbt + kRtCtaCostBlocks);
    for (int ks = 2; ks <= nbt / 2; ++ks) {
        if (nbt % ks != 0 || ks * logits > cap) continue;
        const int64_t path = ((base * ks + kRtSms - 1) / kRtSms) * (nbt / ks + kRtCtaCostBlocks);
        if (path < best_path) {
            best = ks;
            best_path = path;
        }
    }
    return best;
}

// floats of the split-W image (3 bf16 terms of E x H), a multiple of 64 (256 bytes)
static int64_t router_img_floats(int E, int H) { return (int64_t(E) * H * 6 / 4 + 63) / 64 * 64; }

int64_t router_scratch_floats(int x_dtype, int T, int E, int H) {
    if (!router_tc_ok(x_dtype, T, E, H)) return int64_t(T) * E;
    return router_img_floats(E, H) + int64_t(router_tc_split(T, E, H, INT64_MAX)) * T * E;
}

// x_dtype: 1 fp16, 2 bf16, 3 fp32.  `logits` holds `cap` floats of scratch: the partial
// logits, and, on the tensor-core path, in front of them the split-W image (the path is
// taken only when `cap` holds both and x rows start on 16-byte boundaries).
cudaError_t launch_router(const void* x, int x_dtype, const float* w, const float* bias, const uint8_t* resident,
                          int T, int E, int H, int n_group, int topk_group, int top_k, int norm, float scale,
                          float* logits, int64_t cap, int32_t* topk_idx, float* topk_w, float* group_scores_out,
                          int* err, cudaStream_t stream, bool allow_tc, float* logits_out) {
    int ks = 1;
    float* part = logits;
    const int64_t img_floats = router_img_floats(E, H);
    if (allow_tc && err != nullptr && router_tc_ok(x_dtype, T, E, H) && cap >= img_floats + int64_t(T) * E &&
        (reinterpret_cast<uintptr_t>(x) & 15) == 0) {
        static std::mutex mu;
        static bool attr_set[64] = {};
        int dev = 0;
        cudaGetDevice(&dev);
        {
            std::lock_guard<std::mutex> lock(mu);
            if (dev >= 0 && dev < 64 && !attr_set[dev]) {
                const cudaError_t e = cudaFuncSetAttribute(router_logits_tc_kernel,
                                                           cudaFuncAttributeMaxDynamicSharedMemorySize, int(kRtSmem));
                if (e != cudaSuccess) return e;
                attr_set[dev] = true;
            }
        }
        uint8_t* img = reinterpret_cast<uint8_t*>(logits);
        part = logits + img_floats;
        ks = router_tc_split(T, E, H, cap - img_floats);
        const int64_t chunks = int64_t(E) * (H / 8);
        const int split_grid = int(std::min<int64_t>((chunks + 255) / 256, 4096));
        cudaError_t e = launch_chained(router_split_w_kernel, dim3(split_grid), dim3(256), 0, stream, w, img, E, H);
        if (e != cudaSuccess) return e;
        const int N = router_tc_n(T);
        const dim3 grid((T + N - 1) / N, E / 128, ks);
        e = launch_chained(router_logits_tc_kernel, grid, dim3(kRtThreads), kRtSmem, stream,
                           static_cast<const __nv_bfloat16*>(x), static_cast<const uint8_t*>(img), part, T, E, H, N,
                           H / kRtKB / ks, err);
        if (e != cudaSuccess) return e;
    } else {
        const dim3 grid((T + kLT - 1) / kLT, (E + kLE - 1) / kLE);
        cudaError_t e;
        if (x_dtype == 2) {
            e = launch_chained(router_logits_kernel<__nv_bfloat16>, grid, dim3(kLWarps * 32), 0, stream,
                               static_cast<const __nv_bfloat16*>(x), w, logits, T, E, H);
        } else if (x_dtype == 1) {
            e = launch_chained(router_logits_kernel<__half>, grid, dim3(kLWarps * 32), 0, stream,
                               static_cast<const __half*>(x), w, logits, T, E, H);
        } else {
            e = launch_chained(router_logits_kernel<float>, grid, dim3(kLWarps * 32), 0, stream,
                               static_cast<const float*>(x), w, logits, T, E, H);
        }
        if (e != cudaSuccess) return e;
    }
    RouterArgs a{part, ks, bias, resident, T, E, n_group, topk_group, top_k, norm, scale,
                 topk_idx, topk_w, group_scores_out, logits_out};
    if (T <= 2048) {
        // decode-sized batches: one CTA per token, short dependency chains
        return launch_chained(router_select_rank_kernel, dim3(T), dim3((E + 31) / 32 * 32), 0, stream, a);
    } else {
        // large batches: one warp per token keeps the grid small
        const int grid_sel = (T + kSelWarps - 1) / kSelWarps;
        if (E <= 256) return launch_chained(router_select_kernel<8>, dim3(grid_sel), dim3(kSelWarps * 32), 0, stream, a);
        return launch_chained(router_select_kernel<32>, dim3(grid_sel), dim3(kSelWarps * 32), 0, stream, a);
    }
    return cudaGetLastError();
}

// ---------------------------------------------------------------------------------------
// Router without any allocation (cst_route_noalloc).
//
// Some callers of this library cannot call cudaMalloc: a host runtime that has handed all
// device memory to its own pool before loading the library, code that runs while another
// component owns the allocator, or a process that must not grow its footprint after
// start-up.  They still need the router, whose logits kernel writes the [T, E] fp32 logits
// to global scratch that the select kernel reads and that cst_create would otherwise
// allocate.
// This variant keeps that scratch in the file-scope array below instead.  The array is
// part of the library image: every GPU that loads the library holds it (2 MiB) until the
// process exits.  Host code cannot use the array's name as a device address, so the first
// call in each CUDA context looks the address up with cudaGetSymbolAddress (with that
// context current) and caches it under the context's unique id -- a runtime that creates
// its own driver contexts, or calls after cudaDeviceReset, gets the address of its own
// context's copy.  That first call should therefore come before any stream capture.  Every
// call overwrites every scratch element it later reads, so nothing needs clearing between
// calls -- but all calls share the one array: calls that overlap on the GPU (other
// streams, other threads, concurrent graph replays) race on it.  The logits always run on
// the CUDA cores here: that kernel has no device-side waits, so no call can time out with
// nowhere to report it (cst_route reports the tensor-core kernel's bounded waits through
// its context's error word, which this entry point does not have).
constexpr int64_t kNoAllocScratchFloats = int64_t(1) << 19;  // 2 MiB
static __device__ __align__(256) float g_router_noalloc_scratch[kNoAllocScratchFloats];

namespace {
constexpr int kMaxContexts = 64;
struct NoAllocEntry {
    unsigned long long ctx_id;
    float* ptr;
};
NoAllocEntry g_noalloc_cache[kMaxContexts];
int g_noalloc_n = 0;
std::mutex g_noalloc_mu;

// Unique id of the calling thread's current CUDA context (cuCtxGetCurrent + cuCtxGetId,
// reached through the runtime's driver entry points, so the library links no libcuda);
// false when no context is current yet or the driver lacks the calls.
bool current_context_id(unsigned long long* id) {
    static PFN_cuCtxGetCurrent_v4000 get_current = nullptr;
    static PFN_cuCtxGetId_v12000 get_id = nullptr;
    static bool resolved = false;
    if (!resolved) {  // under g_noalloc_mu
        cudaDriverEntryPointQueryResult q1{}, q2{};
        void* f1 = nullptr;
        void* f2 = nullptr;
        if (cudaGetDriverEntryPointByVersion("cuCtxGetCurrent", &f1, 4000, cudaEnableDefault, &q1) == cudaSuccess &&
            q1 == cudaDriverEntryPointSuccess)
            get_current = reinterpret_cast<PFN_cuCtxGetCurrent_v4000>(f1);
        if (cudaGetDriverEntryPointByVersion("cuCtxGetId", &f2, 12000, cudaEnableDefault, &q2) == cudaSuccess &&
            q2 == cudaDriverEntryPointSuccess)
            get_id = reinterpret_cast<PFN_cuCtxGetId_v12000>(f2);
        resolved = true;
    }
    if (!get_current || !get_id) return false;
    CUcontext ctx = nullptr;
    if (get_current(&ctx) != CUDA_SUCCESS || ctx == nullptr) return false;
    return get_id(ctx, id) == CUDA_SUCCESS;
}
}  // namespace

}  // namespace cst

extern "C" int cst_route_noalloc(const void* x, int32_t x_dtype, int32_t T, int32_t hidden, const float* gate_weight,
                                 const float* bias, const uint8_t* resident, int32_t n_experts, int32_t n_group,
                                 int32_t topk_group, int32_t top_k, int32_t norm_topk_prob,
                                 float routed_scaling_factor, int32_t* topk_idx, float* topk_weight, void* stream) {
    using namespace cst;
    clear_last_error();
    if (x_dtype < 1 || x_dtype > 3) return set_last_error(3, "bad x_dtype %d", x_dtype);
    if (hidden <= 0 || hidden % 128) return set_last_error(3, "hidden=%d must be a positive multiple of 128", hidden);
    if (n_experts <= 0 || n_experts > 1024) return set_last_error(3, "n_experts=%d out of [1, 1024]", n_experts);
    if (n_group <= 0 || n_group > 32 || n_experts % n_group)
        return set_last_error(3, "invalid n_group=%d for n_experts=%d", n_group, n_experts);
    if (topk_group <= 0 || topk_group > n_group) return set_last_error(3, "invalid topk_group=%d", topk_group);
    if (top_k <= 0 || top_k > 15 || top_k > n_experts) return set_last_error(3, "invalid top_k=%d", top_k);
    if (T < 0) return set_last_error(3, "T=%d < 0", T);
    const int64_t need = int64_t(T) * n_experts;
    if (need > kNoAllocScratchFloats)
        return set_last_error(3,
                              "cst_route_noalloc: T * n_experts = %lld scratch floats exceed the static "
                              "maximum of %lld (T <= %lld for n_experts = %d); use cst_route",
                              static_cast<long long>(need), static_cast<long long>(kNoAllocScratchFloats),
                              static_cast<long long>(kNoAllocScratchFloats / n_experts), n_experts);
    if (T == 0) return 0;  // empty batch: no work, pointers may be null
    if (!x || !gate_weight || !bias || !topk_idx || !topk_weight) return set_last_error(3, "null pointer");
    if ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(gate_weight)) & 15u)
        return set_last_error(3, "x and gate_weight must be 16-byte aligned");
    float* scratch = nullptr;
    {
        std::lock_guard<std::mutex> lock(g_noalloc_mu);
        unsigned long long cid = 0;
        bool have_id = current_context_id(&cid);
        if (have_id) {
            for (int i = 0; i < g_noalloc_n; ++i)
                if (g_noalloc_cache[i].ctx_id == cid) scratch = g_noalloc_cache[i].ptr;
        }
        if (scratch == nullptr) {
            // first call in this context (the lookup also binds the device's primary context
            // when the thread has none current yet)
            void* p = nullptr;
            const cudaError_t e = cudaGetSymbolAddress(&p, g_router_noalloc_scratch);
            if (e != cudaSuccess || p == nullptr)
                return set_last_error(5, "cudaGetSymbolAddress(router scratch) failed: %s", cudaGetErrorString(e));
            scratch = static_cast<float*>(p);
            if (!have_id) have_id = current_context_id(&cid);
            if (have_id && g_noalloc_n < kMaxContexts) g_noalloc_cache[g_noalloc_n++] = {cid, scratch};
        }
    }
    const cudaError_t e = launch_router(x, x_dtype, gate_weight, bias, resident, T, n_experts, hidden, n_group,
                                        topk_group, top_k, norm_topk_prob, routed_scaling_factor, scratch,
                                        kNoAllocScratchFloats, topk_idx, topk_weight, nullptr, nullptr,
                                        static_cast<cudaStream_t>(stream), /*allow_tc=*/false);
    if (e != cudaSuccess) return set_last_error(5, "router launch failed: %s", cudaGetErrorString(e));
    return 0;
}
