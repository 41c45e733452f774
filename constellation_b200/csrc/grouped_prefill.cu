// Grouped FP8 block-scaled expert SwiGLU for prefill-sized calls (tcgen05): the same
// products as grouped_ffn.cu (the reference's fused_up_gate_kernel,
// expert_node_v2/backend/cuda/fused_up_gate_cuda_v2.cu:31-103, and down_blockscale_kernel,
// backend/cuda/down_cuda_v2.cu:18-62, for every resident expert and every row routed to
// it), shaped for many rows per expert.
//
// Differences from the decode kernel:
//   * a group holds up to 128 packed rows of one expert (NT <= 16 n-tiles of 8), so every
//     weight tile that reaches shared memory serves up to 128 tokens and each MMA is
//     M = 128 x N = 8 NT (up to 128) x K = 32 -- wide enough that the tensor pipe, not the
//     shared-memory reads of the A tile, sets the pace;
//   * activations carry TWO E4M3 terms (v = s (q1 + q2), row-wise relative error ~1e-3 on
//     a full-size expert, inside the 1e-2 bar), stacked along K: per k-step two MMAs
//     (term 0, term 1) accumulate into the same TMEM columns;
//   * one power-of-two activation scale per packed ROW (pack_act.cu, pack_rows_kernel), so
//     each K block is promoted with the weight scale alone, acc += D * scale_inv[rb, kb],
//     and the row scale multiplies the finished accumulator once.
// Per K block a stage holds the weight tile(s) (32 KB: up + gate, or two down row blocks;
// 16 KB for a single down row block) and the group's B tile (2 terms x 8 NT rows x 128 B,
// at most 32 KB); the weight scales travel in a separate 8-deep ring.  The B tile of
// (group g, kb) starts at byte (tile_base(g) * KB + kb * NT) * 2048, term t at t * NT * 1024.
// Eight epilogue warps: two per TMEM lane quarter, each owning 64 token columns.
//
// Work item = (group, row block pair / row block, K split), one persistent CTA per SM, the
// same producer / MMA / epilogue roles and bounded mbarrier waits as grouped_ffn.cu.
#include <cstdint>

#include "cst_common.cuh"
#include "kernels.h"
#include "layout.cuh"

namespace cst {

constexpr int kPrefillTerms = 2;
constexpr int kPrefillTileBytes = kPrefillTerms * kTileCols * kBlock;  // 2048 per n-tile
constexpr int kPrefillEpiWarps = 8;
constexpr int kPrefillColsPerWarp = kPrefillMaxTiles * kTileCols / (kPrefillEpiWarps / 4);  // 64
constexpr int kPrefillThreads = 64 + 32 * kPrefillEpiWarps;                                   // 320
constexpr int kPrefillScStages = 8;

template <int MATS>
struct PfShape {
    static constexpr int kABytes = MATS * 16384;
    static constexpr int kBBytes = kPrefillMaxTiles * kPrefillTileBytes;  // 32 KB
    static constexpr int kStage = kABytes + kBBytes;
    static constexpr int kStages = MATS == 2 ? 3 : 4;
    static constexpr int kScBytes = 32;  // weight scales: 16 B per accumulator
    static constexpr int kColsPerBuf = MATS * kPrefillMaxTiles * kTileCols;  // 256 / 128
    static constexpr int kTmemBufs = MATS == 2 ? 2 : 4;
    static constexpr uint32_t kTmemCols = 512;
    static_assert(kTmemBufs * kColsPerBuf <= int(kTmemCols), "accumulators exceed the TMEM allocation");
    static_assert(kStage % 1024 == 0, "stages must keep 1024-byte alignment");
};

__device__ __forceinline__ int pf_split(int base_items, int KB, int max_split, int n_rows, int out_rows) {
    int S = 1;
    while (S < max_split && base_items * S < 8 * int(gridDim.x) && KB % (2 * S) == 0 &&
           int64_t(n_rows) * 2 * S <= out_rows)
        S *= 2;
    return S;
}

template <int MATS, bool DOWN>
__global__ void __launch_bounds__(kPrefillThreads, 1) grouped_prefill_kernel(FfnArgs a) {
    using S = PfShape<MATS>;
    constexpr int STAGES = S::kStages;
    constexpr int SC = kPrefillScStages;
    constexpr int CW = kPrefillColsPerWarp;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* sc_base = smem + STAGES * S::kStage;
    uint64_t* full = reinterpret_cast<uint64_t*>(sc_base + SC * S::kScBytes);
    uint64_t* empty = full + STAGES;
    uint64_t* tfull = empty + STAGES;
    uint64_t* tempty = tfull + S::kTmemBufs;
    uint64_t* scfull = tempty + S::kTmemBufs;
    uint64_t* scempty = scfull + SC;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(scempty + SC);
    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;

    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);  // the MMA commit
        }
        for (int j = 0; j < SC; ++j) {
            mbar_init(&scfull[j], 1);
            mbar_init(&scempty[j], kPrefillEpiWarps);
        }
        for (int b = 0; b < S::kTmemBufs; ++b) {
            mbar_init(&tfull[b], 1);
            mbar_init(&tempty[b], kPrefillEpiWarps);
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
    const int split = pf_split(base_items, a.KB, a.max_split, n_rows, a.out_rows);
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
                const uint8_t* A = slot + a.a_off + int64_t(DOWN ? rb * MATS : rb) * a.KB * (DOWN ? 16384 : S::kABytes);
                const uint8_t* B = a.bfrag + int64_t(gr.tile_base) * a.KB * kPrefillTileBytes;
                const float* W0 = reinterpret_cast<const float*>(slot + a.s0_off);
                const float* W1 = reinterpret_cast<const float*>(slot + a.s1_off);
                const int64_t wrow = int64_t(DOWN ? rb * MATS : rb) * a.scale_ld;
                const uint32_t bbytes = uint32_t(NT) * kPrefillTileBytes;
                for (int kb = ks * KBs; kb < (ks + 1) * KBs; ++kb) {
                    const int s = it % STAGES;
                    const uint32_t ph = (it / STAGES) & 1u;
                    const int j = it % SC;
                    const uint32_t jph = (it / SC) & 1u;
                    if (!mbar_wait(&empty[s], ph ^ 1u, a.err) || !mbar_wait(&scempty[j], jph ^ 1u, a.err)) {
                        ok = false;
                        break;
                    }
                    uint8_t* st = smem + s * S::kStage;
                    uint8_t* sc = sc_base + j * S::kScBytes;
                    mbar_arrive_expect_tx(&full[s], S::kABytes + bbytes);
                    mbar_arrive_expect_tx(&scfull[j], 16 * MATS);
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
                        // the aligned 16 bytes of the scale grid that hold entry (rb [+m], kb)
                        const int64_t wi = (wrow + (DOWN ? m * a.scale_ld : 0) + kb) & ~int64_t(3);
                        tma_bulk_g2s(sc + 16 * m, (DOWN || m == 0 ? W0 : W1) + wi, 16, &scfull[j]);
                    }
                    ++it;
                }
            }
            // never leave with bulk copies still writing shared memory
            const uint32_t first = it > uint32_t(STAGES) ? it - STAGES : 0u;
            for (uint32_t q = first; q < it; ++q) mbar_wait(&full[q % STAGES], (q / STAGES) & 1u, a.err);
            const uint32_t first_sc = it > uint32_t(SC) ? it - SC : 0u;
            for (uint32_t q = first_sc; q < it; ++q) mbar_wait(&scfull[q % SC], (q / SC) & 1u, a.err);
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
                // N = 8 NT token columns, in the steps of 16 an M = 128 MMA takes; for odd NT
                // the last 8 B rows read past the term (into the next term or unused stage
                // bytes) and only feed accumulator columns no one stores
                const int N = ((kTileCols * NT + 15) / 16) * 16;
                const uint32_t idesc = umma_idesc_e4m3(128, N);
                const uint32_t term_bytes = uint32_t(NT) * kTileCols * kBlock;
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
#pragma unroll
                        for (int tm = 0; tm < kPrefillTerms; ++tm) {
                            const uint64_t bdesc = umma_desc_sw128(st + S::kABytes + tm * term_bytes + ks * kKStep);
#pragma unroll
                            for (int m = 0; m < MATS; ++m) {
                                const uint64_t adesc = umma_desc_sw128(st + m * 16384 + ks * kKStep);
                                tc_mma_e4m3(tmem + b * S::kColsPerBuf + m * 128, adesc, bdesc, idesc,
                                            (ks > 0 || tm > 0) ? 1u : 0u);
                            }
                        }
                    }
                    tc_commit(&empty[s]);
                    tc_commit(&tfull[b]);
                    ++it;
                }
            }
            if (it > 0) mbar_wait(&tfull[(it - 1) % S::kTmemBufs], ((it - 1) / S::kTmemBufs) & 1u, a.err);
        }
    } else {
        // ---------------- epilogue (warps 2..9) ----------------
        const int quarter = warp & 3;            // TMEM lane quarter this warp may access
        const int half = (warp - 2) >> 2;        // token columns [64 half, 64 half + 64)
        const int row = quarter * 32 + lane;     // weight row inside the 128-row block
        const uint32_t lane_addr = uint32_t(quarter * 32) << 16;
        uint32_t it = 0;
        bool ok = true;
        for (int item = blockIdx.x; ok && item < n_items; item += gridDim.x) {
            const int ks = item % split;
            const int gm = item / split;
            const int gi = gm / a.n_mb;
            const int rb = gm - gi * a.n_mb;
            const GroupRec gr = a.groups[gi];
            const int cols = min(CW, gr.n_rows - half * CW);  // token columns this warp owns (<= 0: none)
            float acc[MATS][CW];
#pragma unroll
            for (int m = 0; m < MATS; ++m)
#pragma unroll
                for (int t = 0; t < CW; ++t) acc[m][t] = 0.0f;

            for (int kb = ks * KBs; kb < (ks + 1) * KBs; ++kb) {
                const int b = it % S::kTmemBufs;
                const uint32_t bph = (it / S::kTmemBufs) & 1u;
                const int j = it % SC;
                const uint32_t jph = (it / SC) & 1u;
                if (!mbar_wait(&scfull[j], jph, a.err) || !mbar_wait(&tfull[b], bph, a.err)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                float wsc[MATS];
                {
                    const float* sc = reinterpret_cast<const float*>(sc_base + j * S::kScBytes);
#pragma unroll
                    for (int m = 0; m < MATS; ++m) {
                        const int64_t wr = int64_t(DOWN ? rb * MATS + m : rb) * a.scale_ld;
                        wsc[m] = sc[4 * m + int((wr + kb) & 3)];
                    }
                }
                __syncwarp();
                if (lane == 0) mbar_arrive(&scempty[j]);
                const uint32_t base = tmem + lane_addr + b * S::kColsPerBuf + half * CW;
#pragma unroll
                for (int c = 0; c < CW / 16; ++c) {
                    if (c * 16 < cols) {
                        uint32_t d[MATS][16];
#pragma unroll
                        for (int m = 0; m < MATS; ++m) tmem_ld16(base + m * 128 + c * 16, &d[m][0]);
                        tmem_wait_ld();
#pragma unroll
                        for (int m = 0; m < MATS; ++m) tmem_reg_fence(d[m]);
#pragma unroll
                        for (int m = 0; m < MATS; ++m)
#pragma unroll
                            for (int t = 0; t < 16; ++t)
                                acc[m][c * 16 + t] = fmaf(__uint_as_float(d[m][t]), wsc[m], acc[m][c * 16 + t]);
                    }
                }
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(&tempty[b]);
                ++it;
            }
            if (!ok) break;
#pragma unroll
            for (int t = 0; t < CW; ++t) {
                if (t < cols) {
                    const int prow = gr.row_start + half * CW + t;
                    const float xs = a.bscale[prow];  // the row's activation scale
                    if constexpr (!DOWN) {
                        float* o = a.out + (int64_t(ks) * n_rows + prow) * 2 * a.ld_out + rb * kBlock + row;
                        o[0] = acc[0][t] * xs;
                        o[a.ld_out] = acc[1][t] * xs;
                    } else {
                        const float f = xs * a.row_weight[prow];
#pragma unroll
                        for (int m = 0; m < MATS; ++m)
                            a.out[int64_t(prow) * a.ld_out + (rb * MATS + m) * kBlock + row] = acc[m][t] * f;
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

template <int MATS>
size_t pf_smem_bytes() {
    return size_t(PfShape<MATS>::kStages) * PfShape<MATS>::kStage + size_t(kPrefillScStages) * PfShape<MATS>::kScBytes +
           1024 /* alignment slack */ + 512 /* barriers */;
}

cudaError_t grouped_prefill_init_attributes() {
    const cudaFuncAttribute attr = cudaFuncAttributeMaxDynamicSharedMemorySize;
    cudaError_t e = cudaFuncSetAttribute(grouped_prefill_kernel<2, false>, attr, int(pf_smem_bytes<2>()));
    if (e == cudaSuccess) e = cudaFuncSetAttribute(grouped_prefill_kernel<2, true>, attr, int(pf_smem_bytes<2>()));
    if (e == cudaSuccess) e = cudaFuncSetAttribute(grouped_prefill_kernel<1, true>, attr, int(pf_smem_bytes<1>()));
    return e;
}

cudaError_t launch_grouped_prefill(const FfnArgs& a, bool upgate, int num_sms, cudaStream_t stream) {
    if (upgate)
        return launch_chained(grouped_prefill_kernel<2, false>, dim3(num_sms), dim3(kPrefillThreads),
                              pf_smem_bytes<2>(), stream, a);
    if (a.n_mb % 2 == 0) {
        FfnArgs p = a;
        p.n_mb = a.n_mb / 2;
        return launch_chained(grouped_prefill_kernel<2, true>, dim3(num_sms), dim3(kPrefillThreads),
                              pf_smem_bytes<2>(), stream, p);
    }
    return launch_chained(grouped_prefill_kernel<1, true>, dim3(num_sms), dim3(kPrefillThreads), pf_smem_bytes<1>(),
                          stream, a);
}

}  // namespace cst
