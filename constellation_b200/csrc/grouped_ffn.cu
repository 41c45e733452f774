// Grouped FP8 block-scaled expert SwiGLU on the 5th-generation tensor cores (tcgen05):
// the replacement of the reference's fused_up_gate_kernel
// (expert_node_v2/backend/cuda/fused_up_gate_cuda_v2.cu:31-103) and down_blockscale_kernel
// (backend/cuda/down_cuda_v2.cu:18-62), for every resident expert and every token routed to
// it, in ONE launch per projection.
//
// Work item = (group, 128-row block rb of the output dimension, K split ks); a group is <= 16
// packed activation rows of one expert slot (route_pack.cu).  The K split S (1, 2 or 4) is
// chosen on the device from the group count so that small decode batches still give every
// SM several items; up/gate then writes S raw partial sums that the h packer adds in fixed
// order (pack_act.cu); the down projection never splits; instead a down item takes two
// consecutive 128-row blocks when H / 128 is even, so both projections stream 32 KB of
// weights per K block.  One persistent CTA per SM walks the item list with 6 warps:
//   warp 0, one lane: TMA producer.  Per 128-wide K block kb it bulk-copies the weight tile
//     (16 KB per matrix: up+gate = 32 KB, down = 16 KB; contiguous in the arena and already in
//     the swizzled K-major image the tensor cores read, relayout.cu) and the group's B tile
//     (three E4M3 activation terms x 8 or 16 tokens, 3 or 6 KB) and the block's scales
//     (weight scale_inv entries and the activation terms' powers of two, <= 224 B) into a ring
//     of STAGES shared-memory stages; it runs ahead across item boundaries.
//   warp 1, one lane: MMA issuer.  Per kb: 4 k-steps x MATS of
//     tcgen05.mma.cta_group::1.kind::f8f6f4, M = 128 weight rows, N = 3 terms x 8/16 tokens,
//     K = 32, into one of four TMEM accumulator buffers; tcgen05.commit frees the smem stage
//     and signals the accumulator to the epilogue.
//   warps 2-5: epilogue.  Each thread owns one weight row (its TMEM lane): per kb it loads the
//     accumulator (tcgen05.ld) and the stage's scales into registers, releases both, promotes
//       acc[token] += (D[term0] s0[token] + D[term1] s1[token] + D[term2] s2[token]) * scale_inv[rb, kb]
//     in fp32 -- the block-scaled algebra of dequantize-then-matmul (server/fp8_utils.py:4-39,
//     server/moe_layer_runtime.py:604-609) with the scales applied once per 128x128 block and
//     s0..s2 the powers of two of the activation terms.
//     At the end of an item: up/gate -> the raw up and gate partial sums of split ks (the h
//     packer, pack_act.cu, adds the splits in order and applies SiLU * mul), down -> y *
//     routing weight, written per packed row in fp32 (coalesced along the rows).
// TMEM: MATS x 48 fp32 columns per accumulator buffer, four buffers (512 / 256 columns),
// allocated by warp 2 and freed on every exit path.
//
// Every mbarrier wait is bounded (cst_common.cuh).  On a timeout the role records the
// device error word, stops issuing, waits (bounded) for the work it already launched, and
// the CTA reaches the common exit where TMEM is released.
#include <cstdint>

#include "cst_common.cuh"
#include "kernels.h"
#include "layout.cuh"

namespace cst {

template <int MATS>
struct TcShape {
    static constexpr int kABytes = MATS * 16384;                       // weight tile(s) per kb
    static constexpr int kBBytes = kMaxTilesPerGroup * kBTileBytes;     // 6 KB
    static constexpr int kStage = kABytes + kBBytes;                    // multiple of 1024
    // per-stage scales: 16 B of each weight-scale row (kb rounded down to 4) + the act
    // scales of the group (3 terms x 8 NT tokens, <= 192 B)
    static constexpr int kScBytes = 256;
    static constexpr int kScAct = 32;                                   // act scales at +32
    static constexpr int kColsPerBuf = MATS * 48;
    // four accumulator buffers let the MMA issuer run up to four K blocks ahead of the
    // epilogue (4 x 96 -> 512 columns for two accumulators, 4 x 48 -> 256 for one)
    static constexpr int kTmemBufs = 4;
    static constexpr uint32_t kTmemCols = MATS == 2 ? 512 : 256;
    static_assert(kTmemBufs * kColsPerBuf <= int(kTmemCols), "accumulators exceed the TMEM allocation");
    static_assert(kStage % 1024 == 0, "stages must keep 1024-byte alignment");
};

// K split for this launch: enough (group, row block, split) items to keep every CTA busy
// (at least 16 per CTA, so the last round is a small share) while each item keeps a whole
// number of K blocks and the partial sums fit the output buffer.  Every CTA computes the
// same value from the same inputs.
__device__ __forceinline__ int choose_split(int base_items, int KB, int max_split, int n_rows, int out_rows) {
    int S = 1;
    while (S < max_split && base_items * S < 16 * int(gridDim.x) && KB % (2 * S) == 0 &&
           int64_t(n_rows) * 2 * S <= out_rows)
        S *= 2;
    return S;
}


// MATS accumulators per item: up/gate (DOWN false) -> mat 0 = w_up, mat 1 = w_gate of one
// 128-row block; down (DOWN true) -> MATS consecutive 128-row blocks of w_down (so the down
// projection streams 32 KB per K block too when its row-block count is even).
template <int MATS, int STAGES, bool DOWN>
__global__ void __launch_bounds__(192, 1) grouped_ffn_tc_kernel(FfnArgs a) {
    using S = TcShape<MATS>;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    // each stage's scales sit beside the stages; the epilogue copies a K block's scales to
    // registers and releases the stage and the TMEM buffer before it computes
    uint8_t* bsc_base = smem + STAGES * S::kStage;
    uint64_t* full = reinterpret_cast<uint64_t*>(bsc_base + STAGES * S::kScBytes);
    uint64_t* empty = full + STAGES;
    uint64_t* tfull = empty + STAGES;
    uint64_t* tempty = tfull + S::kTmemBufs;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tempty + S::kTmemBufs);
    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;

    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1 + 4);  // the MMA commit + the four epilogue warps
        }
        for (int b = 0; b < S::kTmemBufs; ++b) {
            mbar_init(&tfull[b], 1);
            mbar_init(&tempty[b], 4);
        }
        fence_barrier_init();
    }
    if (warp == 2) {
        tmem_alloc(tmem_slot, S::kTmemCols);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    chain_wait();
    chain_release();
    const int base_items = a.meta->n_groups * a.n_mb;
    const int n_rows = a.meta->n_rows;
    const int split = choose_split(base_items, a.KB, a.max_split, n_rows, a.out_rows);
    const int KBs = a.KB / split;
    const int n_items = base_items * split;
    if (blockIdx.x == 0 && threadIdx.x == 0) a.meta->split_k = split;

    if (warp == 0) {
        if (lane == 0) {
            // ---------------- TMA producer ----------------
            uint32_t it = 0;
            bool ok = true;
            for (int item = blockIdx.x; ok && item < n_items; item += gridDim.x) {
                const int ks = item % split;
                const int gm = item / split;
                const int gi = gm / a.n_mb;
                const int rb = gm - gi * a.n_mb;
                const GroupRec gr = a.groups[gi];
                const int NT = (gr.n_rows + kTileCols - 1) / kTileCols;
                const uint8_t* slot = a.arena + int64_t(gr.slot) * a.slot_bytes;
                // up/gate: [rb][kb][up | gate] 32 KB per kb; down: [rb][kb] 16 KB per kb
                const uint8_t* A = slot + a.a_off + int64_t(DOWN ? rb * MATS : rb) * a.KB * (DOWN ? 16384 : S::kABytes);
                const uint8_t* B = a.bfrag + int64_t(gr.tile_base) * a.KB * kBTileBytes;
                // scale grids are 256-byte aligned; each stage takes the aligned 16 bytes that
                // hold entry (rb, kb), so a row that starts off a 16-byte boundary still copies
                const float* W0 = reinterpret_cast<const float*>(slot + a.s0_off);
                const float* W1 = reinterpret_cast<const float*>(slot + a.s1_off);
                const int64_t wrow = int64_t(DOWN ? rb * MATS : rb) * a.scale_ld;
                const float* X = a.bscale + int64_t(gr.tile_base) * a.KB * kScalesPerTile;
                const uint32_t bbytes = uint32_t(NT) * kBTileBytes;
                const uint32_t xsb = uint32_t(NT) * kScalesPerTile * 4;
                for (int kb = ks * KBs; kb < (ks + 1) * KBs; ++kb) {
                    const int s = it % STAGES;
                    const uint32_t ph = (it / STAGES) & 1u;
                    if (!mbar_wait(&empty[s], ph ^ 1u, a.err)) {
                        ok = false;
                        break;
                    }
                    uint8_t* st = smem + s * S::kStage;
                    uint8_t* sc = bsc_base + s * S::kScBytes;
                    mbar_arrive_expect_tx(&full[s], S::kABytes + bbytes + 16 * MATS + xsb);
                    if constexpr (DOWN) {
#pragma unroll
                        for (int m = 0; m < MATS; ++m)
                            tma_bulk_g2s(st + m * 16384, A + (int64_t(m) * a.KB + kb) * 16384, 16384, &full[s]);
                    } else {
                        tma_bulk_g2s(st, A + int64_t(kb) * S::kABytes, S::kABytes, &full[s]);
                    }
                    tma_bulk_g2s(st + S::kABytes, B + int64_t(kb) * bbytes, bbytes, &full[s]);
#pragma unroll
                    for (int m = 0; m < MATS; ++m) {
                        // down: scale row of block rb*MATS+m; up/gate: the same row of two grids
                        const int64_t wi = (wrow + (DOWN ? m * a.scale_ld : 0) + kb) & ~int64_t(3);
                        tma_bulk_g2s(sc + 16 * m, (DOWN || m == 0 ? W0 : W1) + wi, 16, &full[s]);
                    }
                    tma_bulk_g2s(sc + S::kScAct, X + int64_t(kb) * NT * kScalesPerTile, xsb, &full[s]);
                    ++it;
                }
            }
            // never leave with bulk copies still writing shared memory
            const uint32_t first = it > uint32_t(STAGES) ? it - STAGES : 0u;
            for (uint32_t j = first; j < it; ++j) mbar_wait(&full[j % STAGES], (j / STAGES) & 1u, a.err);
        }
    } else if (warp == 1) {
        if (lane == 0) {
            // ---------------- MMA issuer ----------------
            uint32_t it = 0;
            bool ok = true;
            const uint32_t smem_base = smem_u32(smem);
            for (int item = blockIdx.x; ok && item < n_items; item += gridDim.x) {
                const int gi = (item / split) / a.n_mb;
                const GroupRec gr = a.groups[gi];
                const int NT = (gr.n_rows + kTileCols - 1) / kTileCols;
                // N = 3 terms x 8 NT tokens = 24 / 48 columns; with M = 128 the MMA takes N in
                // steps of 16, so one n-tile runs at N = 32: B rows 24..31 are whatever the
                // stage holds there and only feed accumulator columns no one reads
                const uint32_t idesc = umma_idesc_e4m3(128, NT == 1 ? 32 : kSplits * kTileCols * NT);
                for (int kk = 0; kk < KBs; ++kk) {
                    const int s = it % STAGES;
                    const uint32_t ph = (it / STAGES) & 1u;
                    const int b = it % S::kTmemBufs;
                    const uint32_t bph = (it / S::kTmemBufs) & 1u;
                    if (!mbar_wait(&full[s], ph, a.err) || !mbar_wait(&tempty[b], bph ^ 1u, a.err)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t st = smem_base + s * S::kStage;
#pragma unroll
                    for (int ks = 0; ks < kBlock / kKStep; ++ks) {
                        const uint64_t bdesc = umma_desc_sw128(st + S::kABytes + ks * kKStep);
#pragma unroll
                        for (int m = 0; m < MATS; ++m) {
                            const uint64_t adesc = umma_desc_sw128(st + m * 16384 + ks * kKStep);
                            tc_mma_e4m3(tmem + b * S::kColsPerBuf + m * 48, adesc, bdesc, idesc, ks > 0 ? 1u : 0u);
                        }
                    }
                    tc_commit(&empty[s]);
                    tc_commit(&tfull[b]);
                    ++it;
                }
            }
            // the MMAs issued last must have finished before TMEM is released
            if (it > 0) mbar_wait(&tfull[(it - 1) % S::kTmemBufs], ((it - 1) / S::kTmemBufs) & 1u, a.err);
        }
    } else {
        // ---------------- epilogue (warps 2..5) ----------------
        const int quarter = warp & 3;                 // TMEM lane quarter this warp may access
        const int row = quarter * 32 + lane;          // weight row inside the 128-row block
        const uint32_t lane_addr = uint32_t(quarter * 32) << 16;
        uint32_t it = 0;
        bool ok = true;
        for (int item = blockIdx.x; item < n_items; item += gridDim.x) {
            const int ks = item % split;
            const int gm = item / split;
            const int gi = gm / a.n_mb;
            const int rb = gm - gi * a.n_mb;
            const GroupRec gr = a.groups[gi];
            const int NT = (gr.n_rows + kTileCols - 1) / kTileCols;
            const int TP = NT * kTileCols;
            float acc[MATS][kGroupRows];
#pragma unroll
            for (int m = 0; m < MATS; ++m)
#pragma unroll
                for (int t = 0; t < kGroupRows; ++t) acc[m][t] = 0.0f;

            for (int kb = ks * KBs; ok && kb < (ks + 1) * KBs; ++kb) {
                const int b = it % S::kTmemBufs;
                const uint32_t bph = (it / S::kTmemBufs) & 1u;
                const int s = it % STAGES;
                const uint32_t ph = (it / STAGES) & 1u;
                if (!mbar_wait(&full[s], ph, a.err) || !mbar_wait(&tfull[b], bph, a.err)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                uint32_t d[MATS][48];
                const uint32_t base = tmem + lane_addr + b * S::kColsPerBuf;
#pragma unroll
                for (int m = 0; m < MATS; ++m) {
                    tmem_ld16(base + m * 48, &d[m][0]);
                    tmem_ld16(base + m * 48 + 16, &d[m][16]);
                    tmem_ld16(base + m * 48 + 32, &d[m][32]);
                }
                const float* sc = reinterpret_cast<const float*>(bsc_base + s * S::kScBytes);
                float wsc[MATS];
#pragma unroll
                for (int m = 0; m < MATS; ++m) {
                    const int64_t wr = int64_t(DOWN ? rb * MATS + m : rb) * a.scale_ld;
                    wsc[m] = sc[4 * m + int((wr + kb) & 3)];
                }
                float xsc[3 * kGroupRows];
#pragma unroll
                for (int i = 0; i < 3 * kGroupRows; ++i) xsc[i] = (i < 3 * TP) ? sc[S::kScAct / 4 + i] : 0.0f;
                tmem_wait_ld();
#pragma unroll
                for (int m = 0; m < MATS; ++m) tmem_reg_fence(d[m]);
                tc_fence_before();
                __syncwarp();
                if (lane == 0) {
                    mbar_arrive(&tempty[b]);
                    mbar_arrive(&empty[s]);
                }
                // acc[t] += (D[term0] s0[t] + D[term1] s1[t] + D[term2] s2[t]) * scale_inv[rb, kb]
                if (NT == 1) {
#pragma unroll
                    for (int t = 0; t < kTileCols; ++t) {
                        const float x0 = xsc[t], x1 = xsc[kTileCols + t], x2 = xsc[2 * kTileCols + t];
#pragma unroll
                        for (int m = 0; m < MATS; ++m) {
                            const float v = fmaf(__uint_as_float(d[m][16 + t]), x2,
                                                 fmaf(__uint_as_float(d[m][8 + t]), x1, __uint_as_float(d[m][t]) * x0));
                            acc[m][t] = fmaf(v, wsc[m], acc[m][t]);
                        }
                    }
                } else {
#pragma unroll
                    for (int t = 0; t < kGroupRows; ++t) {
                        const float x0 = xsc[t], x1 = xsc[kGroupRows + t], x2 = xsc[2 * kGroupRows + t];
#pragma unroll
                        for (int m = 0; m < MATS; ++m) {
                            const float v = fmaf(__uint_as_float(d[m][32 + t]), x2,
                                                 fmaf(__uint_as_float(d[m][16 + t]), x1, __uint_as_float(d[m][t]) * x0));
                            acc[m][t] = fmaf(v, wsc[m], acc[m][t]);
                        }
                    }
                }
                ++it;
            }
            if (!ok) break;
            // one weight row, every token of the group (coalesced along the rows)
#pragma unroll
            for (int t = 0; t < kGroupRows; ++t) {
                if (t < gr.n_rows) {
                    const int prow = gr.row_start + t;
                    if constexpr (!DOWN) {
                        // raw split accumulators; the h packer adds the splits and applies SiLU
                        float* o = a.out + (int64_t(ks) * n_rows + prow) * 2 * a.ld_out + rb * kBlock + row;
                        o[0] = acc[0][t];
                        o[a.ld_out] = acc[1][t];
                    } else {
                        const float rw = a.row_weight[prow];
#pragma unroll
                        for (int m = 0; m < MATS; ++m)
                            a.out[int64_t(prow) * a.ld_out + (rb * MATS + m) * kBlock + row] = acc[m][t] * rw;
                    }
                }
            }
        }
    }

    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == 2) tmem_dealloc(tmem, S::kTmemCols);
}

constexpr int kUpGateStages = 5;
constexpr int kDownStages = 8;

template <int MATS, int STAGES>
size_t tc_smem_bytes() {
    return size_t(STAGES) * TcShape<MATS>::kStage + STAGES * TcShape<MATS>::kScBytes +
           1024 /* alignment slack */ + 512 /* barriers */;
}

cudaError_t grouped_ffn_init_attributes() {
    const cudaFuncAttribute attr = cudaFuncAttributeMaxDynamicSharedMemorySize;
    cudaError_t e = cudaFuncSetAttribute(grouped_ffn_tc_kernel<2, kUpGateStages, false>, attr,
                                         int(tc_smem_bytes<2, kUpGateStages>()));
    if (e == cudaSuccess)
        e = cudaFuncSetAttribute(grouped_ffn_tc_kernel<2, kUpGateStages, true>, attr,
                                 int(tc_smem_bytes<2, kUpGateStages>()));
    if (e == cudaSuccess)
        e = cudaFuncSetAttribute(grouped_ffn_tc_kernel<1, kDownStages, true>, attr,
                                 int(tc_smem_bytes<1, kDownStages>()));
    return e;
}

// up/gate: a.n_mb = I / 128 row blocks.  down: a.n_mb = H / 128 row blocks; pairs of blocks per
// item when that count is even (32 KB of weights per stage, as up/gate) and the launch has
// enough groups to give every SM a pair, else one block per item.
cudaError_t launch_grouped_ffn(const FfnArgs& a, bool upgate, int num_sms, cudaStream_t stream) {
    const bool few_items = a.groups_hint > 0 && int64_t(a.groups_hint) * (a.n_mb / 2) < num_sms;
    if (upgate)
        return launch_chained(grouped_ffn_tc_kernel<2, kUpGateStages, false>, dim3(num_sms), dim3(192),
                              tc_smem_bytes<2, kUpGateStages>(), stream, a);
    if (a.n_mb % 2 == 0 && !few_items) {
        FfnArgs p = a;
        p.n_mb = a.n_mb / 2;
        return launch_chained(grouped_ffn_tc_kernel<2, kUpGateStages, true>, dim3(num_sms), dim3(192),
                              tc_smem_bytes<2, kUpGateStages>(), stream, p);
    }
    return launch_chained(grouped_ffn_tc_kernel<1, kDownStages, true>, dim3(num_sms), dim3(192),
                          tc_smem_bytes<1, kDownStages>(), stream, a);
}

}  // namespace cst
