// Upload-time relayout of one expert from the reference's row-major format into the
// arena chunks the tcgen05 grouped kernel reads (layout.cuh).
//
// Replaces the six cudaMalloc + cudaMemcpy of UploadExpertCudaV2
// (expert_node_v2/backend/cuda/backend_cuda_v2.cc:94-145): the bytes land in one
// pre-allocated arena slot instead, already in the shared-memory image the tensor cores
// read -- K-major, 128-byte swizzled 8-row atoms -- so the kernel streams every chunk with a
// single TMA bulk copy and no shared-memory shuffling.
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

// One thread per 16-byte swizzle chunk.  A matrix is cut into (128-row block rb,
// 128-column block kb) tiles of 16 KB; `mats` matrices of the same shape are interleaved
// per tile (up and gate: tile (rb, kb) = [up 16 KB | gate 16 KB]).
__global__ void relayout_kernel(const uint8_t* __restrict__ m0, const uint8_t* __restrict__ m1,
                                uint8_t* __restrict__ dst, int rows, int cols, int mats) {
    const int64_t units = int64_t(mats) * rows * cols / 16;
    const int kbs = cols / kBlock;
    for (int64_t u = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; u < units;
         u += int64_t(gridDim.x) * blockDim.x) {
        const int64_t tile = u >> 10;            // 1024 chunks of 16 B per 16 KB tile
        const int within = static_cast<int>(u & 1023);
        const int mat = static_cast<int>(tile % mats);
        const int64_t t2 = tile / mats;
        const int kb = static_cast<int>(t2 % kbs);
        const int rb = static_cast<int>(t2 / kbs);
        const int r = within >> 3;               // row inside the tile (0..127)
        const int pc = within & 7;               // physical chunk position in the 128-byte row
        const int c = pc ^ (r & 7);              // logical 16-byte chunk stored there
        const uint8_t* src = (mat ? m1 : m0) + int64_t(rb * kBlock + r) * cols + kb * kBlock + c * 16;
        uint4 v = *reinterpret_cast<const uint4*>(src);
        v.x = remap_nan_bytes(v.x);
        v.y = remap_nan_bytes(v.y);
        v.z = remap_nan_bytes(v.z);
        v.w = remap_nan_bytes(v.w);
        reinterpret_cast<uint4*>(dst)[u] = v;
    }
}

cudaError_t launch_relayout(const uint8_t* wu, const uint8_t* wg, const uint8_t* wd, uint8_t* slot,
                            int inter, int hidden, int num_sms, cudaStream_t stream) {
    const ArenaGeom geo = ArenaGeom::make(hidden, inter);
    const int grid = num_sms * 4;
    relayout_kernel<<<grid, 256, 0, stream>>>(wu, wg, slot, inter, hidden, 2);
    relayout_kernel<<<grid, 256, 0, stream>>>(wd, nullptr, slot + geo.upgate_bytes, hidden, inter, 1);
    return cudaGetLastError();
}

}  // namespace cst
