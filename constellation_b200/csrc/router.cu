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
//     fp32 products; TF32 tensor cores would change which experts win).  32x32 output
//     tiles, K split across gridDim.z into fixed slices; partial sums go to
//     partial[z][T][E] and are added in z order by the select kernel, so results are
//     bit-identical from run to run.
//   router_select_kernel: one warp per token does the sigmoid / bias / group / top-k
//     logic with warp-shuffle arg-max reductions.
#include <cfloat>
#include <cstdint>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
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

constexpr int kRT = 32;   // tile edge (experts and tokens)
constexpr int kRK = 128;  // K chunk per shared-memory step
constexpr int kRKP = kRK + 4;

// 16 consecutive activations of row `t` starting at column `k` (vector loads), as fp32.
template <typename TX>
__device__ __forceinline__ void load16(const TX* x, int64_t off, float (&v)[16]);
template <>
__device__ __forceinline__ void load16<float>(const float* x, int64_t off, float (&v)[16]) {
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const float4 f = *reinterpret_cast<const float4*>(x + off + 4 * i);
        v[4 * i] = f.x; v[4 * i + 1] = f.y; v[4 * i + 2] = f.z; v[4 * i + 3] = f.w;
    }
}
template <>
__device__ __forceinline__ void load16<__nv_bfloat16>(const __nv_bfloat16* x, int64_t off, float (&v)[16]) {
#pragma unroll
    for (int i = 0; i < 2; ++i) {
        const uint4 u = *reinterpret_cast<const uint4*>(x + off + 8 * i);
        const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            v[8 * i + 2 * j] = __uint_as_float(w[j] << 16);
            v[8 * i + 2 * j + 1] = __uint_as_float(w[j] & 0xffff0000u);
        }
    }
}
template <>
__device__ __forceinline__ void load16<__half>(const __half* x, int64_t off, float (&v)[16]) {
#pragma unroll
    for (int i = 0; i < 2; ++i) {
        const uint4 u = *reinterpret_cast<const uint4*>(x + off + 8 * i);
        const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&w[j]));
            v[8 * i + 2 * j] = f.x;
            v[8 * i + 2 * j + 1] = f.y;
        }
    }
}

// 32 experts x 32 tokens per CTA over one K slice, 128-wide chunks staged in shared
// memory; the next chunk is fetched into registers while the current one is consumed.
template <typename TX>
__global__ void __launch_bounds__(256) router_logits_kernel(const TX* __restrict__ x, const float* __restrict__ w,
                                                            float* __restrict__ partial, int T, int E, int H,
                                                            int k_slice) {
    __shared__ __align__(16) float xs[kRT][kRKP];
    __shared__ __align__(16) float ws[kRT][kRKP];
    const int e0 = blockIdx.x * kRT;
    const int t0 = blockIdx.y * kRT;
    const int kz = blockIdx.z;
    const int k_begin = kz * k_slice;
    const int tid = threadIdx.x;
    const int tx = tid & 15;  // expert pair
    const int ty = tid >> 4;  // token pair
    const int lr = tid >> 3;         // staged row 0..31
    const int lc = (tid & 7) * 16;   // staged column 0..112
    const bool t_ok = (t0 + lr) < T;
    const bool e_ok = (e0 + lr) < E;
    const int64_t xoff = int64_t(t0 + lr) * H + lc;
    const int64_t woff = int64_t(e0 + lr) * H + lc;
    float rx[16], rw[16];
    auto fetch = [&](int k0) {
        if (t_ok) {
            load16<TX>(x, xoff + k0, rx);
        } else {
#pragma unroll
            for (int i = 0; i < 16; ++i) rx[i] = 0.0f;
        }
        if (e_ok) {
            load16<float>(w, woff + k0, rw);
        } else {
#pragma unroll
            for (int i = 0; i < 16; ++i) rw[i] = 0.0f;
        }
    };
    float acc[2][2] = {{0.f, 0.f}, {0.f, 0.f}};
    fetch(k_begin);
    for (int k0 = k_begin; k0 < k_begin + k_slice; k0 += kRK) {
#pragma unroll
        for (int i = 0; i < 16; i += 4) {
            *reinterpret_cast<float4*>(&xs[lr][lc + i]) = make_float4(rx[i], rx[i + 1], rx[i + 2], rx[i + 3]);
            *reinterpret_cast<float4*>(&ws[lr][lc + i]) = make_float4(rw[i], rw[i + 1], rw[i + 2], rw[i + 3]);
        }
        __syncthreads();
        if (k0 + kRK < k_begin + k_slice) fetch(k0 + kRK);
#pragma unroll 4
        for (int c = 0; c < kRK; c += 4) {
            const float4 x0 = *reinterpret_cast<const float4*>(&xs[2 * ty][c]);
            const float4 x1 = *reinterpret_cast<const float4*>(&xs[2 * ty + 1][c]);
            const float4 w0 = *reinterpret_cast<const float4*>(&ws[2 * tx][c]);
            const float4 w1 = *reinterpret_cast<const float4*>(&ws[2 * tx + 1][c]);
            const float xa[4] = {x0.x, x0.y, x0.z, x0.w}, xb[4] = {x1.x, x1.y, x1.z, x1.w};
            const float wa[4] = {w0.x, w0.y, w0.z, w0.w}, wb[4] = {w1.x, w1.y, w1.z, w1.w};
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                acc[0][0] = fmaf(xa[j], wa[j], acc[0][0]);
                acc[0][1] = fmaf(xa[j], wb[j], acc[0][1]);
                acc[1][0] = fmaf(xb[j], wa[j], acc[1][0]);
                acc[1][1] = fmaf(xb[j], wb[j], acc[1][1]);
            }
        }
        __syncthreads();
    }
#pragma unroll
    for (int i = 0; i < 2; ++i) {
        const int t = t0 + 2 * ty + i;
        if (t >= T) continue;
#pragma unroll
        for (int j = 0; j < 2; ++j) {
            const int e = e0 + 2 * tx + j;
            if (e < E) partial[(int64_t(kz) * T + t) * E + e] = acc[i][j];
        }
    }
}

struct RouterArgs {
    const float* partial;   // [kz][T][E]
    int kz;
    const float* bias;      // [E]
    const uint8_t* resident;  // [E] or null (all resident)
    int T, E, n_group, topk_group, top_k, norm;
    float scale;
    int32_t* topk_idx;      // [T, top_k]
    float* topk_w;          // [T, top_k]
    float* logits_out;      // [T, E] or null
    float* group_scores_out;  // [T, n_group] or null
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
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int t = blockIdx.x * kSelWarps + warp;
    if (t >= a.T) return;
    const int E = a.E;
    const int epg = E / a.n_group;
    const int64_t zstride = int64_t(a.T) * E;
    const float* __restrict__ part = a.partial + int64_t(t) * E;
    float ch[EPL];
    int grp[EPL];
#pragma unroll
    for (int i = 0; i < EPL; ++i) {
        const int e = lane + 32 * i;
        ch[i] = -INFINITY;
        grp[i] = 0x7fffffff;
        if (e < E) {
            // independent read-only loads, then the fixed-order sum over the K slices
            float p[8];
#pragma unroll
            for (int z = 0; z < 8; ++z) p[z] = (z < a.kz) ? __ldg(part + z * zstride + e) : 0.0f;
            float l = 0.0f;
#pragma unroll
            for (int z = 0; z < 8; ++z)
                if (z < a.kz) l += p[z];
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

int router_k_split(int H) {
    const int chunks = H / kRK;
    for (int z : {8, 4, 2}) {
        if (chunks % z == 0) return z;
    }
    return 1;
}

// x_dtype: 1 fp16, 2 bf16, 3 fp32.  partial needs k_split * T * E floats.
cudaError_t launch_router(const void* x, int x_dtype, const float* w, const float* bias, const uint8_t* resident,
                          int T, int E, int H, int n_group, int topk_group, int top_k, int norm, float scale,
                          float* partial, int32_t* topk_idx, float* topk_w, float* logits_out,
                          float* group_scores_out, cudaStream_t stream) {
    const int kz = router_k_split(H);
    dim3 grid((E + kRT - 1) / kRT, (T + kRT - 1) / kRT, kz);
    const int k_slice = H / kz;
    if (x_dtype == 2) {
        router_logits_kernel<__nv_bfloat16><<<grid, 256, 0, stream>>>(
            static_cast<const __nv_bfloat16*>(x), w, partial, T, E, H, k_slice);
    } else if (x_dtype == 1) {
        router_logits_kernel<__half><<<grid, 256, 0, stream>>>(static_cast<const __half*>(x), w, partial, T, E, H,
                                                               k_slice);
    } else {
        router_logits_kernel<float><<<grid, 256, 0, stream>>>(static_cast<const float*>(x), w, partial, T, E, H,
                                                              k_slice);
    }
    RouterArgs a{partial, kz, bias, resident, T, E, n_group, topk_group, top_k, norm, scale,
                 topk_idx, topk_w, logits_out, group_scores_out};
    const int grid_sel = (T + kSelWarps - 1) / kSelWarps;
    if (E <= 256) {
        router_select_kernel<8><<<grid_sel, kSelWarps * 32, 0, stream>>>(a);
    } else {
        router_select_kernel<32><<<grid_sel, kSelWarps * 32, 0, stream>>>(a);
    }
    return cudaGetLastError();
}

// ---------------------------------------------------------------------------------------
// Router without any allocation (cst_route_noalloc).
//
// Some callers of this library cannot call cudaMalloc: a host runtime that has handed all
// device memory to its own pool before loading the library, code that runs while another
// component owns the allocator, or a process that must not grow its footprint after
// start-up.  They still need the router, whose logits kernel writes its K-split partial
// sums ([kz, T, E] fp32) to global scratch that cst_create would otherwise allocate.
// This variant keeps that scratch in the file-scope array below instead.  The array is
// part of the library image: every GPU that loads the library holds it (2 MiB) until the
// process exits.  Host code cannot use the array's name as a device address, so the first
// call on each device looks the address up with cudaGetSymbolAddress (with that device
// current) and caches it; that first call should therefore come before any stream
// capture.  Every call overwrites every scratch element it later reads, so nothing needs
// clearing between calls -- but all calls share the one array: calls that overlap on the
// GPU (other streams, other threads, concurrent graph replays) race on it.
constexpr int64_t kNoAllocScratchFloats = int64_t(1) << 19;  // 2 MiB
static __device__ __align__(256) float g_router_noalloc_scratch[kNoAllocScratchFloats];

namespace {
constexpr int kMaxDevices = 64;
float* g_noalloc_ptr[kMaxDevices] = {};
std::mutex g_noalloc_mu;
}  // namespace

}  // namespace cst

extern "C" int cst_route_noalloc(const void* x, int32_t x_dtype, int32_t T, int32_t hidden, const float* gate_weight,
                                 const float* bias, const uint8_t* resident, int32_t n_experts, int32_t n_group,
                                 int32_t topk_group, int32_t top_k, int32_t norm_topk_prob,
                                 float routed_scaling_factor, int32_t* topk_idx, float* topk_weight, void* stream) {
    using namespace cst;
    clear_last_error();
    if (x_dtype < 1 || x_dtype > 3) return set_last_error(3, "bad x_dtype %d", x_dtype);
    if (!x || !gate_weight || !bias || !topk_idx || !topk_weight) return set_last_error(3, "null pointer");
    if ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(gate_weight)) & 15u)
        return set_last_error(3, "x and gate_weight must be 16-byte aligned");
    if (hidden <= 0 || hidden % 128) return set_last_error(3, "hidden=%d must be a positive multiple of 128", hidden);
    if (n_experts <= 0 || n_experts > 1024) return set_last_error(3, "n_experts=%d out of [1, 1024]", n_experts);
    if (n_group <= 0 || n_group > 32 || n_experts % n_group)
        return set_last_error(3, "invalid n_group=%d for n_experts=%d", n_group, n_experts);
    if (topk_group <= 0 || topk_group > n_group) return set_last_error(3, "invalid topk_group=%d", topk_group);
    if (top_k <= 0 || top_k > 15 || top_k > n_experts) return set_last_error(3, "invalid top_k=%d", top_k);
    if (T < 0) return set_last_error(3, "T=%d < 0", T);
    const int kz = router_k_split(hidden);
    const int64_t need = int64_t(kz) * T * n_experts;
    if (need > kNoAllocScratchFloats)
        return set_last_error(3,
                              "cst_route_noalloc: T * n_experts * %d = %lld scratch floats exceed the static "
                              "maximum of %lld (T <= %lld for n_experts = %d); use cst_route",
                              kz, static_cast<long long>(need), static_cast<long long>(kNoAllocScratchFloats),
                              static_cast<long long>(kNoAllocScratchFloats / (int64_t(kz) * n_experts)), n_experts);
    if (T == 0) return 0;
    int dev = -1;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices)
        return set_last_error(5, "cudaGetDevice failed or device id out of range");
    float* scratch = nullptr;
    {
        std::lock_guard<std::mutex> lock(g_noalloc_mu);
        if (g_noalloc_ptr[dev] == nullptr) {
            void* p = nullptr;
            const cudaError_t e = cudaGetSymbolAddress(&p, g_router_noalloc_scratch);
            if (e != cudaSuccess || p == nullptr)
                return set_last_error(5, "cudaGetSymbolAddress(router scratch) failed: %s", cudaGetErrorString(e));
            g_noalloc_ptr[dev] = static_cast<float*>(p);
        }
        scratch = g_noalloc_ptr[dev];
    }
    const cudaError_t e = launch_router(x, x_dtype, gate_weight, bias, resident, T, n_experts, hidden, n_group,
                                        topk_group, top_k, norm_topk_prob, routed_scaling_factor, scratch, topk_idx,
                                        topk_weight, nullptr, nullptr, static_cast<cudaStream_t>(stream));
    if (e != cudaSuccess) return set_last_error(5, "router launch failed: %s", cudaGetErrorString(e));
    return 0;
}
