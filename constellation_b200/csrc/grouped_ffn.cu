// Grouped FP8 block-scaled expert SwiGLU for decode: the replacement of the reference's
// fused_up_gate_kernel (expert_node_v2/backend/cuda/fused_up_gate_cuda_v2.cu:31-103) and
// down_blockscale_kernel (backend/cuda/down_cuda_v2.cu:18-62), for every resident expert
// and every token routed to it in ONE launch per projection.
//
// Work item = (group, 64-row block of the output dimension).  A group is <= 16 packed
// activation rows of one expert slot (route_pack.cu).  Persistent CTAs walk the item list
// (gridDim = SMs x 2) with 5 warps:
//   warp 4 (one lane): producer.  For each K block of each item it issues three TMA bulk
//     copies into a ring of STAGES shared-memory stages: the weight chunk (16 KB up+gate or
//     8 KB down, contiguous in the arena, already in MMA fragment order), the activation B
//     fragments (3 KB per 8-row n-tile) and their per-row scales.  It runs ahead across
//     item boundaries, so the weight stream never drains between items.
//   warps 0-3: consumers, 16 output rows each.  Per K block: 128-bit shared loads of the A
//     fragments, mma.sync.m16n8k32 E4M3 x E4M3 -> fp32 over the three activation terms, and
//     the block-scale promotion acc += partial * scale_inv[rb, kb] * act_scale[row, kb] in
//     fp32 registers (one 128x128 weight block per K block, as dequant_fp8_weight_blockwise
//     defines the scales).
//   Epilogue (fused): up/gate -> h = silu(gate) * up (silu(g) = g / (1 + exp(-g)), the
//     reference's formula); down -> y * routing weight, written per packed row in fp32 so
//     the combine adds the k contributions in a fixed order.
//
// Every mbarrier wait is bounded (cst_common.cuh); a timeout sets the context's device
// error word, the producer drains its in-flight copies and the CTA exits.
#include <cstdint>

#include "cst_common.cuh"
#include "kernels.h"
#include "layout.cuh"

namespace cst {


template <int MATS>
struct FfnShape {
    static constexpr int kABytes = 4 * 4 * MATS * kAFragBytes;            // 16 KB / 8 KB
    static constexpr int kBBytes = kMaxTilesPerGroup * kBTileBytes;        // 6 KB
    static constexpr int kSBytes = kMaxTilesPerGroup * kTileCols * 4;      // 64 B
    static constexpr int kStage = (kABytes + kBBytes + kSBytes + 127) / 128 * 128;
};

template <int MATS, int STAGES>
__global__ void __launch_bounds__(160, 2) grouped_ffn_kernel(FfnArgs a) {
    using S = FfnShape<MATS>;
    extern __shared__ __align__(1024) uint8_t smem[];
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + STAGES * S::kStage);
    uint64_t* empty = full + STAGES;
    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;

    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 4);
        }
        fence_barrier_init();
    }
    __syncthreads();

    const int n_items = a.meta->n_groups * a.n_mb;

    if (warp == 4) {
        if (lane != 0) return;
        uint32_t it = 0;
        bool ok = true;
        for (int item = blockIdx.x; ok && item < n_items; item += gridDim.x) {
            const int gi = item / a.n_mb;
            const int mb = item - gi * a.n_mb;
            const GroupRec gr = a.groups[gi];
            const int NT = (gr.n_rows + kTileCols - 1) / kTileCols;
            const uint8_t* A = a.arena + int64_t(gr.slot) * a.slot_bytes + a.a_off +
                               int64_t(mb) * a.KB * S::kABytes;
            const uint8_t* B = a.bfrag + int64_t(gr.tile_base) * a.KB * kBTileBytes;
            const float* Sc = a.bscale + int64_t(gr.tile_base) * a.KB * kTileCols;
            const uint32_t bbytes = uint32_t(NT) * kBTileBytes;
            const uint32_t sbytes = uint32_t(NT) * kTileCols * 4;
            for (int kb = 0; kb < a.KB; ++kb) {
                const int s = it % STAGES;
                const uint32_t ph = (it / STAGES) & 1u;
                if (!mbar_wait(&empty[s], ph ^ 1u, a.err)) {
                    ok = false;
                    break;
                }
                uint8_t* st = smem + s * S::kStage;
                mbar_arrive_expect_tx(&full[s], S::kABytes + bbytes + sbytes);
                tma_bulk_g2s(st, A + int64_t(kb) * S::kABytes, S::kABytes, &full[s]);
                tma_bulk_g2s(st + S::kABytes, B + int64_t(kb) * bbytes, bbytes, &full[s]);
                tma_bulk_g2s(st + S::kABytes + S::kBBytes, Sc + int64_t(kb) * NT * kTileCols, sbytes,
                             &full[s]);
                ++it;
            }
        }
        // never leave the CTA with bulk copies still writing its shared memory
        const uint32_t first = it > uint32_t(STAGES) ? it - STAGES : 0u;
        for (uint32_t j = first; j < it; ++j) mbar_wait(&full[j % STAGES], (j / STAGES) & 1u, a.err);
        return;
    }

    // consumers
    const int g = lane >> 2, t = lane & 3;
    uint32_t it = 0;
    for (int item = blockIdx.x; item < n_items; item += gridDim.x) {
        const int gi = item / a.n_mb;
        const int mb = item - gi * a.n_mb;
        const GroupRec gr = a.groups[gi];
        const int NT = (gr.n_rows + kTileCols - 1) / kTileCols;
        const int rb = (mb * kRowsPerItem) / kBlock;
        const uint8_t* slot = a.arena + int64_t(gr.slot) * a.slot_bytes;
        const float* ws0 = reinterpret_cast<const float*>(slot + a.s0_off) + int64_t(rb) * a.scale_ld;
        const float* ws1 = reinterpret_cast<const float*>(slot + a.s1_off) + int64_t(rb) * a.scale_ld;

        float acc[MATS][kMaxTilesPerGroup][4];
#pragma unroll
        for (int m = 0; m < MATS; ++m)
#pragma unroll
            for (int nt = 0; nt < kMaxTilesPerGroup; ++nt)
#pragma unroll
                for (int i = 0; i < 4; ++i) acc[m][nt][i] = 0.0f;

        for (int kb = 0; kb < a.KB; ++kb) {
            const int s = it % STAGES;
            const uint32_t ph = (it / STAGES) & 1u;
            if (!mbar_wait(&full[s], ph, a.err)) return;
            const uint8_t* st = smem + s * S::kStage;
            const uint8_t* sB = st + S::kABytes;
            const float* sS = reinterpret_cast<const float*>(st + S::kABytes + S::kBBytes);
            uint4 af[4][MATS];
#pragma unroll
            for (int ks = 0; ks < 4; ++ks)
#pragma unroll
                for (int m = 0; m < MATS; ++m)
                    af[ks][m] = lds128(st + ((warp * 4 + ks) * MATS + m) * kAFragBytes + lane * 16);
            float wsc[MATS];
            wsc[0] = __ldg(ws0 + kb);
            if constexpr (MATS == 2) wsc[1] = __ldg(ws1 + kb);
#pragma unroll
            for (int nt = 0; nt < kMaxTilesPerGroup; ++nt) {
                if (nt < NT) {
                    float c[MATS][4][4];
#pragma unroll
                    for (int m = 0; m < MATS; ++m)
#pragma unroll
                        for (int ks = 0; ks < 4; ++ks)
#pragma unroll
                            for (int i = 0; i < 4; ++i) c[m][ks][i] = 0.0f;
#pragma unroll
                    for (int ks = 0; ks < 4; ++ks) {
#pragma unroll
                        for (int sp = 0; sp < kSplits; ++sp) {
                            const uint2 b = lds64(sB + ((nt * 4 + ks) * kSplits + sp) * kFragBytes + lane * 8);
#pragma unroll
                            for (int m = 0; m < MATS; ++m) mma_e4m3_16832(c[m][ks], af[ks][m], b.x, b.y);
                        }
                    }
                    const float xs0 = sS[nt * kTileCols + 2 * t];
                    const float xs1 = sS[nt * kTileCols + 2 * t + 1];
#pragma unroll
                    for (int m = 0; m < MATS; ++m) {
                        const float f0 = wsc[m] * xs0, f1 = wsc[m] * xs1;
#pragma unroll
                        for (int i = 0; i < 4; ++i) {
                            const float v = (c[m][0][i] + c[m][1][i]) + (c[m][2][i] + c[m][3][i]);
                            acc[m][nt][i] = fmaf(v, (i & 1) ? f1 : f0, acc[m][nt][i]);
                        }
                    }
                }
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[s]);
            ++it;
        }

        // fused epilogue
#pragma unroll
        for (int nt = 0; nt < kMaxTilesPerGroup; ++nt) {
            if (nt < NT) {
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    const int col = nt * kTileCols + 2 * t + (i & 1);
                    if (col < gr.n_rows) {
                        const int prow = gr.row_start + col;
                        const int orow = mb * kRowsPerItem + warp * kWarpRows + g + 8 * (i >> 1);
                        float v;
                        if constexpr (MATS == 2) {
                            const float up = acc[0][nt][i];
                            const float gate = acc[1][nt][i];
                            v = (gate / (1.0f + expf(-gate))) * up;
                        } else {
                            v = acc[0][nt][i] * a.row_weight[prow];
                        }
                        a.out[int64_t(prow) * a.ld_out + orow] = v;
                    }
                }
            }
        }
    }
}

constexpr int kUpGateStages = 4;
constexpr int kDownStages = 6;

template <int MATS, int STAGES>
size_t ffn_smem_bytes() {
    return size_t(STAGES) * FfnShape<MATS>::kStage + 2 * STAGES * sizeof(uint64_t);
}

cudaError_t grouped_ffn_init_attributes() {
    cudaError_t e = cudaFuncSetAttribute(grouped_ffn_kernel<2, kUpGateStages>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         int(ffn_smem_bytes<2, kUpGateStages>()));
    if (e != cudaSuccess) return e;
    return cudaFuncSetAttribute(grouped_ffn_kernel<1, kDownStages>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                int(ffn_smem_bytes<1, kDownStages>()));
}

cudaError_t launch_grouped_ffn(const FfnArgs& a, bool upgate, int num_sms, cudaStream_t stream) {
    const int grid = num_sms * 2;
    if (upgate) {
        grouped_ffn_kernel<2, kUpGateStages>
            <<<grid, 160, ffn_smem_bytes<2, kUpGateStages>(), stream>>>(a);
    } else {
        grouped_ffn_kernel<1, kDownStages><<<grid, 160, ffn_smem_bytes<1, kDownStages>(), stream>>>(a);
    }
    return cudaGetLastError();
}

}  // namespace cst
