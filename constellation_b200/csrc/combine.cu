// Weighted combine: out[t] = sum_k y[row(t, k)] (+ y[row(t, shared)]), cast once.
//
// Replaces combine_outputs_torch (server/moe_layer_runtime.py:148-167, fp32
// `combined.add_(w * y)` per route) and the routed + shared sum of run_sparse_layer
// (server/full_model_runtime.py:348).  The routing weights were already applied in the
// down-projection epilogue; here the rows of a token are added in the fixed order
// k = 0 .. top_k-1 then the shared expert, in fp32, so the result is bit-identical from
// run to run.  Optionally adds a residual (server/full_model_runtime.py:355).
#include <cstdint>
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include "cst_common.cuh"
#include "kernels.h"

namespace cst {


__device__ __forceinline__ float4 load_act4(const void* p, int dtype, int64_t idx) {
    if (dtype == 3) return *reinterpret_cast<const float4*>(static_cast<const float*>(p) + idx);
    const uint2 u = *reinterpret_cast<const uint2*>(static_cast<const uint16_t*>(p) + idx);
    if (dtype == 2) {
        return make_float4(__uint_as_float(u.x << 16), __uint_as_float(u.x & 0xffff0000u),
                           __uint_as_float(u.y << 16), __uint_as_float(u.y & 0xffff0000u));
    }
    const float2 a = __half22float2(*reinterpret_cast<const __half2*>(&u.x));
    const float2 b = __half22float2(*reinterpret_cast<const __half2*>(&u.y));
    return make_float4(a.x, a.y, b.x, b.y);
}

// grid (T, ceil(H / 1024)): one float4 column group per thread, all k rows loaded
// independently, so a token's sum costs one memory latency instead of H / 1024 of them.
__global__ void __launch_bounds__(256) combine_kernel(CombineArgs a) {
    chain_wait();
    chain_release();
    const int t = blockIdx.x;
    if (t >= a.T) return;
    const int32_t* rows = a.tk_row + int64_t(t) * a.K1;
    for (int h = (blockIdx.y * blockDim.x + threadIdx.x) * 4; h < a.H; h += gridDim.y * blockDim.x * 4) {
        // issue every row load before the first add (absent rows read as zero), then sum in k order
        float4 v[16];
#pragma unroll
        for (int k = 0; k < 16; ++k) {
            const int r = (k < a.K1) ? __ldg(rows + k) : -1;
            v[k] = (r >= 0) ? __ldg(reinterpret_cast<const float4*>(a.y + int64_t(r) * a.ldy + h))
                            : make_float4(0.f, 0.f, 0.f, 0.f);
        }
        float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
        for (int k = 0; k < 16; ++k) {
            if (k < a.K1) {
                acc.x += v[k].x;
                acc.y += v[k].y;
                acc.z += v[k].z;
                acc.w += v[k].w;
            }
        }
        if (a.extra) {
            const float4 v = *reinterpret_cast<const float4*>(a.extra + int64_t(t) * a.H + h);
            acc.x += v.x;
            acc.y += v.y;
            acc.z += v.z;
            acc.w += v.w;
        }
        if (a.residual) {
            const float4 v = load_act4(a.residual, a.residual_dtype, int64_t(t) * a.H + h);
            acc.x += v.x;
            acc.y += v.y;
            acc.z += v.z;
            acc.w += v.w;
        }
        const int64_t o = int64_t(t) * a.H + h;
        if (a.out_dtype == 3) {
            *reinterpret_cast<float4*>(static_cast<float*>(a.out) + o) = acc;
        } else if (a.out_dtype == 2) {
            __nv_bfloat162 lo = __floats2bfloat162_rn(acc.x, acc.y);
            __nv_bfloat162 hi = __floats2bfloat162_rn(acc.z, acc.w);
            uint2 u;
            u.x = *reinterpret_cast<uint32_t*>(&lo);
            u.y = *reinterpret_cast<uint32_t*>(&hi);
            *reinterpret_cast<uint2*>(static_cast<uint16_t*>(a.out) + o) = u;
        } else {
            __half2 lo = __floats2half2_rn(acc.x, acc.y);
            __half2 hi = __floats2half2_rn(acc.z, acc.w);
            uint2 u;
            u.x = *reinterpret_cast<uint32_t*>(&lo);
            u.y = *reinterpret_cast<uint32_t*>(&hi);
            *reinterpret_cast<uint2*>(static_cast<uint16_t*>(a.out) + o) = u;
        }
    }
}

cudaError_t launch_combine(const CombineArgs& a, cudaStream_t stream) {
    if (a.T <= 0) return cudaSuccess;
    const dim3 grid(a.T, (a.H + 1023) / 1024);
    return launch_chained(combine_kernel, grid, dim3(256), 0, stream, a);
}

}  // namespace cst
