// Upload-time relayout of one expert from the reference's row-major format into the
// fragment-major arena chunks described in layout.cuh.
//
// Replaces the six cudaMalloc + cudaMemcpy of UploadExpertCudaV2
// (expert_node_v2/backend/cuda/backend_cuda_v2.cc:94-145): the bytes land in one
// pre-allocated arena slot instead, already in the order the grouped kernels read.
//
// FP8 decode parity: the reference node decodes float8_e4m3fn through a LUT in which
// S.1111.111 (0x7F / 0xFF) means +-448 (fp8_lut_v2.cc:59-61), while E4M3 tensor cores
// read those bytes as NaN.  The relayout rewrites them to 0x7E / 0xFE (exactly +-448),
// so the device path decodes every byte the way the reference node does.
#include <cstdint>

#include "cst_common.cuh"
#include "kernels.h"
#include "layout.cuh"

namespace cst {

__device__ __forceinline__ uint32_t remap_nan_bytes(uint32_t w) {
    const uint32_t m = __vcmpeq4(w & 0x7F7F7F7Fu, 0x7F7F7F7Fu);  // 0xFF in every NaN byte
    return w - (m & 0x01010101u);
}

// One thread per 16-byte fragment unit of the up/gate chunks.
__global__ void relayout_upgate_kernel(const uint8_t* __restrict__ wu, const uint8_t* __restrict__ wg,
                                       uint8_t* __restrict__ dst, int inter, int hidden) {
    const int64_t units = int64_t(2) * inter * hidden / 16;
    const int kbs = hidden / kBlock;
    for (int64_t u = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; u < units;
         u += int64_t(gridDim.x) * blockDim.x) {
        const int64_t chunk = u >> 10;  // 1024 units of 16 B per 16 KB chunk
        const int within = static_cast<int>(u & 1023);
        const int lane = within & 31;
        const int mat = (within >> 5) & 1;
        const int ks = (within >> 6) & 3;
        const int w = within >> 8;
        const int kb = static_cast<int>(chunk % kbs);
        const int mb = static_cast<int>(chunk / kbs);
        const int g = lane >> 2, t = lane & 3;
        const uint8_t* src = mat ? wg : wu;
        uint32_t r[4];
#pragma unroll
        for (int reg = 0; reg < 4; ++reg) {
            const int row = mb * kRowsPerItem + w * kWarpRows + g + 8 * (reg & 1);
            const int col = kb * kBlock + ks * kKStep + 4 * t + 16 * (reg >> 1);
            r[reg] = remap_nan_bytes(
                *reinterpret_cast<const uint32_t*>(src + int64_t(row) * hidden + col));
        }
        reinterpret_cast<uint4*>(dst)[u] = make_uint4(r[0], r[1], r[2], r[3]);
    }
}

// One thread per 16-byte fragment unit of the down chunks (w_down is [hidden, inter]).
__global__ void relayout_down_kernel(const uint8_t* __restrict__ wd, uint8_t* __restrict__ dst,
                                     int inter, int hidden) {
    const int64_t units = int64_t(inter) * hidden / 16;
    const int kbs = inter / kBlock;
    for (int64_t u = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; u < units;
         u += int64_t(gridDim.x) * blockDim.x) {
        const int64_t chunk = u >> 9;  // 512 units per 8 KB chunk
        const int within = static_cast<int>(u & 511);
        const int lane = within & 31;
        const int ks = (within >> 5) & 3;
        const int w = within >> 7;
        const int kb = static_cast<int>(chunk % kbs);
        const int mb = static_cast<int>(chunk / kbs);
        const int g = lane >> 2, t = lane & 3;
        uint32_t r[4];
#pragma unroll
        for (int reg = 0; reg < 4; ++reg) {
            const int row = mb * kRowsPerItem + w * kWarpRows + g + 8 * (reg & 1);
            const int col = kb * kBlock + ks * kKStep + 4 * t + 16 * (reg >> 1);
            r[reg] = remap_nan_bytes(
                *reinterpret_cast<const uint32_t*>(wd + int64_t(row) * inter + col));
        }
        reinterpret_cast<uint4*>(dst)[u] = make_uint4(r[0], r[1], r[2], r[3]);
    }
}

cudaError_t launch_relayout(const uint8_t* wu, const uint8_t* wg, const uint8_t* wd, uint8_t* slot,
                            int inter, int hidden, int num_sms, cudaStream_t stream) {
    const ArenaGeom geo = ArenaGeom::make(hidden, inter);
    const int grid = num_sms * 4;
    relayout_upgate_kernel<<<grid, 256, 0, stream>>>(wu, wg, slot, inter, hidden);
    relayout_down_kernel<<<grid, 256, 0, stream>>>(wd, slot + geo.upgate_bytes, inter, hidden);
    return cudaGetLastError();
}

}  // namespace cst
