// RMSNorm between stacked MoE layers: the prenorm the reference applies before the sparse
// FFN, torch.nn.functional.rms_norm(h, (H,), weight, 1e-6)
// (server/full_model_runtime.py:271-276), as one kernel:
//     out[t, c] = h[t, c] * rsqrt(mean_c(h[t, :]^2) + eps) * weight[c]
// with the mean and the products in fp32 and one round-to-nearest-even cast at the end.
// (torch multiplies the weight after casting to the input dtype; the single rounding here
// can differ from it by one unit in the last place.)
//
// One CTA of 256 threads per row: pass 1 sums squares (8 elements per thread step, 16-byte
// loads for 16-bit types), a block reduction, pass 2 re-reads the row (L1/L2) and writes.
#include <cstdint>
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include "cst_common.cuh"
#include "kernels.h"

namespace cst {

namespace {

constexpr int kNormThreads = 256;

__device__ __forceinline__ void load8(const void* base, int dtype, int64_t i, float (&v)[8]) {
    if (dtype == 3) {
        const float4 a = *reinterpret_cast<const float4*>(static_cast<const float*>(base) + i);
        const float4 b = *reinterpret_cast<const float4*>(static_cast<const float*>(base) + i + 4);
        v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w; v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
    } else {
        const uint4 u = *reinterpret_cast<const uint4*>(static_cast<const uint16_t*>(base) + i);
        const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            if (dtype == 2) {
                v[2 * k] = __uint_as_float(w[k] << 16);
                v[2 * k + 1] = __uint_as_float(w[k] & 0xffff0000u);
            } else {
                const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&w[k]));
                v[2 * k] = f.x;
                v[2 * k + 1] = f.y;
            }
        }
    }
}

__device__ __forceinline__ void store8(void* base, int dtype, int64_t i, const float (&v)[8]) {
    if (dtype == 3) {
        *reinterpret_cast<float4*>(static_cast<float*>(base) + i) = make_float4(v[0], v[1], v[2], v[3]);
        *reinterpret_cast<float4*>(static_cast<float*>(base) + i + 4) = make_float4(v[4], v[5], v[6], v[7]);
    } else {
        uint32_t w[4];
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            if (dtype == 2) {
                const __nv_bfloat162 b = __floats2bfloat162_rn(v[2 * k], v[2 * k + 1]);
                w[k] = *reinterpret_cast<const uint32_t*>(&b);
            } else {
                const __half2 h = __floats2half2_rn(v[2 * k], v[2 * k + 1]);
                w[k] = *reinterpret_cast<const uint32_t*>(&h);
            }
        }
        *reinterpret_cast<uint4*>(static_cast<uint16_t*>(base) + i) = make_uint4(w[0], w[1], w[2], w[3]);
    }
}

__global__ void __launch_bounds__(kNormThreads) rmsnorm_kernel(const void* x, int x_dtype, int H, const float* weight,
                                                              float eps, void* out, int out_dtype) {
    __shared__ float s_part[kNormThreads / 32];
    chain_wait();
    chain_release();
    const int64_t row = blockIdx.x;
    const int64_t off = row * H;
    float ss = 0.0f;
    for (int c = threadIdx.x * 8; c < H; c += kNormThreads * 8) {
        float v[8];
        load8(x, x_dtype, off + c, v);
#pragma unroll
        for (int k = 0; k < 8; ++k) ss = fmaf(v[k], v[k], ss);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    if ((threadIdx.x & 31) == 0) s_part[threadIdx.x >> 5] = ss;
    __syncthreads();
    float tot = 0.0f;
#pragma unroll
    for (int w = 0; w < kNormThreads / 32; ++w) tot += s_part[w];  // fixed order: deterministic
    const float r = rsqrtf(tot / float(H) + eps);
    for (int c = threadIdx.x * 8; c < H; c += kNormThreads * 8) {
        float v[8];
        load8(x, x_dtype, off + c, v);
#pragma unroll
        for (int k = 0; k < 8; ++k) v[k] = v[k] * r * (weight ? weight[c + k] : 1.0f);
        store8(out, out_dtype, off + c, v);
    }
}

}  // namespace

cudaError_t launch_rmsnorm(const void* x, int x_dtype, int T, int H, const float* weight, float eps, void* out,
                           int out_dtype, cudaStream_t stream) {
    if (T == 0) return cudaSuccess;
    return launch_chained(rmsnorm_kernel, dim3(T), dim3(kNormThreads), 0, stream, x, x_dtype, H, weight, eps, out,
                          out_dtype);
}

}  // namespace cst
