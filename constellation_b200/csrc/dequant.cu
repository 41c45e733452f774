// Block dequantization of one FP8 E4M3FN matrix: out[r, c] = e4m3(w[r, c]) * scale_inv[r / b, c / b].
//
// The device version of dequant_fp8_weight_blockwise (server/fp8_utils.py:4-39), which the
// reference uses for its fp32 oracle and to expand the shared expert at load time
// (server/backbone_store.py:405-425).  Same semantics: true float8_e4m3fn decode (0x7F /
// 0xFF are NaN, as torch's .float() gives), ragged last blocks via ceil-div grids, one fp32
// multiply per element -- so the result is bit-identical to the reference function.
// HBM-bound: 1 byte read + 4 bytes written per element; 16 elements per thread per step.
#include <cstdint>

#include "cst_common.cuh"
#include "kernels.h"

namespace cst {

__global__ void __launch_bounds__(256) dequant_fp8_kernel(const uint8_t* __restrict__ w, const float* __restrict__ s,
                                                          float* __restrict__ out, int rows, int cols, int block,
                                                          int ncb) {
    const int64_t total = int64_t(rows) * cols;
    const bool vec = (cols % 16) == 0;
    const int64_t step = int64_t(gridDim.x) * blockDim.x;
    if (vec) {
        for (int64_t u = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; u * 16 < total; u += step) {
            const int64_t e0 = u * 16;
            const int r = int(e0 / cols);
            const int c0 = int(e0 - int64_t(r) * cols);
            const uint4 q = *reinterpret_cast<const uint4*>(w + e0);
            const uint32_t words[4] = {q.x, q.y, q.z, q.w};
            float v[16];
#pragma unroll
            for (int i = 0; i < 16; ++i) {
                const int c = c0 + i;
                const float sc = s[int64_t(r / block) * ncb + c / block];
                v[i] = e4m3_to_f32(uint8_t(words[i >> 2] >> (8 * (i & 3)))) * sc;
            }
            float4* o = reinterpret_cast<float4*>(out + e0);
#pragma unroll
            for (int i = 0; i < 4; ++i) o[i] = make_float4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]);
        }
    } else {
        for (int64_t e = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; e < total; e += step) {
            const int r = int(e / cols), c = int(e - int64_t(r) * cols);
            out[e] = e4m3_to_f32(w[e]) * s[int64_t(r / block) * ncb + c / block];
        }
    }
}

cudaError_t launch_dequant_fp8(const uint8_t* w, const float* s, float* out, int rows, int cols, int block,
                               int num_sms, cudaStream_t stream) {
    const int ncb = (cols + block - 1) / block;
    dequant_fp8_kernel<<<num_sms * 8, 256, 0, stream>>>(w, s, out, rows, cols, block, ncb);
    return cudaGetLastError();
}

}  // namespace cst
