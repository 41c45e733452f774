// Activation packer: rows of x (bf16 / fp16 / fp32) or of the SwiGLU intermediate h -> E4M3
// tensor-core B fragments, three terms per element.  For h the source is the up/gate
// kernel's raw split accumulators: the packer adds the K splits in fixed order and applies
// h = silu(gate) * up (server/moe_layer_runtime.py:604-609) while loading.
//
// The grouped FFN kernels multiply FP8 E4M3 weights by activations on the FP8 tensor
// pipe.  One E4M3 term carries 4 significant bits, so each activation element v of a
// (row, 128-wide K block) is written as
//     v = s * (q1 + q2 + q3),  q1 = e4m3(v/s), q2 = e4m3(v/s - q1), q3 = e4m3(v/s - q1 - q2)
// (decode kernels; the prefill kernels take the first two terms only)
// with s the smallest power of two that maps the block's max |v| to <= 448.  The decode
// packer gives every term its own power of two, fitted to the block's largest residual
// (v = s1 q1 + s2 q2 + s3 q3), so one large element in a block costs the small ones
// nothing beyond the first term: the three terms reproduce every element to ~2^-12
// relative of the block's residuals, far inside the bf16 resolution of the inputs, and the
// residuals are exact in fp32.  (The prefill packer keeps one scale per row for both of
// its terms; its absolute floor is ~2e-6 of the row max.)  The grouped kernel applies the
// term scales per (row, K block) and the weight scale_inv per 128x128 weight block while
// accumulating in fp32 -- the same algebra as dequantize-then-matmul
// (server/fp8_utils.py:4-39, server/moe_layer_runtime.py:604-609).
//
// One warp per (packed row, 8 consecutive K blocks): the row's metadata is read once and
// the 8 source loads are issued together; per K block 128 elements, 4 per lane, one 32-bit
// store per term.  Rows of a group's last n-tile beyond its row count are not written.
// The tasks run over the packed rows themselves (0 .. meta->n_rows, contiguous in group
// order).  A row's group is found by one load and a warp ballot up to 32 groups, beyond
// that by binary search over the groups' first rows, which every CTA first copies to shared
// memory.  No warp spends a task on an unused tile column (at decode most columns of the
// 8-wide n-tiles are), and the grid is at most the CTAs that fit on the GPU at once (fewer
// when the host's bound on the rows needs fewer), so every task starts in the first wave.
#include <algorithm>
#include <cstdint>
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include "cst_common.cuh"
#include "kernels.h"
#include "layout.cuh"

namespace cst {


__device__ __forceinline__ void load4(const PackActArgs& a, int64_t src_row, int k, int split, float (&v)[4]) {
    if (src_row < 0) {
        v[0] = v[1] = v[2] = v[3] = 0.0f;
        return;
    }
    if (a.src_dtype == kSrcUpGatePartials) {
        // up/gate split accumulators [split][n_rows][2][K]: add the splits in order, then
        // h = silu(gate) * up with silu(g) = g / (1 + exp(-g))
        const float* p = static_cast<const float*>(a.src) + src_row * 2 * a.ld + k;
        const int64_t split_stride = int64_t(a.meta->n_rows) * 2 * a.ld;
        float4 u = *reinterpret_cast<const float4*>(p);
        float4 g = *reinterpret_cast<const float4*>(p + a.ld);
#pragma unroll
        for (int ks = 1; ks < kMaxUpGateSplit; ++ks) {
            if (ks < split) {
                const float4 u2 = *reinterpret_cast<const float4*>(p + ks * split_stride);
                const float4 g2 = *reinterpret_cast<const float4*>(p + ks * split_stride + a.ld);
                u.x += u2.x; u.y += u2.y; u.z += u2.z; u.w += u2.w;
                g.x += g2.x; g.y += g2.y; g.z += g2.z; g.w += g2.w;
            }
        }
        v[0] = (g.x / (1.0f + expf(-g.x))) * u.x;
        v[1] = (g.y / (1.0f + expf(-g.y))) * u.y;
        v[2] = (g.z / (1.0f + expf(-g.z))) * u.z;
        v[3] = (g.w / (1.0f + expf(-g.w))) * u.w;
    } else if (a.src_dtype == 3) {
        const float4 f = *reinterpret_cast<const float4*>(static_cast<const float*>(a.src) + src_row * a.ld + k);
        v[0] = f.x; v[1] = f.y; v[2] = f.z; v[3] = f.w;
    } else if (a.src_dtype == 2) {
        const uint2 u = *reinterpret_cast<const uint2*>(static_cast<const __nv_bfloat16*>(a.src) + src_row * a.ld + k);
        v[0] = __uint_as_float(u.x << 16);
        v[1] = __uint_as_float(u.x & 0xffff0000u);
        v[2] = __uint_as_float(u.y << 16);
        v[3] = __uint_as_float(u.y & 0xffff0000u);
    } else {
        const uint2 u = *reinterpret_cast<const uint2*>(static_cast<const __half*>(a.src) + src_row * a.ld + k);
        const __half2 h0 = *reinterpret_cast<const __half2*>(&u.x);
        const __half2 h1 = *reinterpret_cast<const __half2*>(&u.y);
        const float2 f0 = __half22float2(h0), f1 = __half22float2(h1);
        v[0] = f0.x; v[1] = f0.y; v[2] = f1.x; v[3] = f1.y;
    }
}

constexpr int kPackKbPerTask = 8;  // K blocks one warp packs for one row (at most)
constexpr int kPackSmemGroups = 4096;  // groups whose first rows a CTA keeps in shared memory

// Group of packed row `prow`: the last g with row_start[g] <= prow (groups hold >= 1 row
// each and start in increasing row order).  From shared memory when the CTA staged the
// groups, else from the group records themselves.
__device__ __forceinline__ int group_of_row(const int32_t* s_rs, const GroupRec* groups, int n_groups, int prow) {
    int lo = 0, hi = n_groups - 1;
    while (lo < hi) {
        const int mid = (lo + hi + 1) >> 1;
        const int rs = s_rs ? s_rs[mid] : groups[mid].row_start;
        if (rs <= prow) lo = mid;
        else hi = mid - 1;
    }
    return lo;
}

// KBPT: K blocks one warp packs for one row (x rows: 8; split partials, which read up to 8
// loads per element: 2, so more warps are in flight)
template <int KBPT>
__global__ void __launch_bounds__(256) pack_act_kernel(PackActArgs a) {
    __shared__ int32_t s_rs[kPackSmemGroups];
    chain_wait();
    chain_release();
    const int KB = a.K / kBlock;
    const int n_chunks = (KB + KBPT - 1) / KBPT;
    const int n_rows = a.meta->n_rows;
    const int n_groups = a.meta->n_groups;
    // up to 32 groups (a worker request, a rank's share of a decode batch): each task's
    // warp finds the group with one load and a ballot; more: staged in shared memory
    const bool warp_search = n_groups <= 32;
    const bool staged = !warp_search && n_groups <= kPackSmemGroups;
    if (staged)
        for (int g = threadIdx.x; g < n_groups; g += blockDim.x) s_rs[g] = a.groups[g].row_start;
    if (!warp_search) __syncthreads();  // the same on every thread: meta is read by all
    const int split = a.src_dtype == kSrcUpGatePartials ? a.meta->split_k : 1;
    const int lane = threadIdx.x & 31;
    const int64_t n_tasks = int64_t(n_rows) * n_chunks;
    const int64_t warp_global = (int64_t(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
    const int64_t n_warps = (int64_t(gridDim.x) * blockDim.x) >> 5;
    for (int64_t task = warp_global; task < n_tasks; task += n_warps) {
        // task = (packed row, chunk of KBPT K blocks)
        const int prow = static_cast<int>(task / n_chunks);
        const int chunk = static_cast<int>(task - int64_t(prow) * n_chunks);
        const int64_t src_row = a.row_map ? a.row_map[prow] : prow;
        int gi;
        if (warp_search) {
            // row starts increase with the group index and group 0 starts at row 0, so the
            // highest lane whose group starts at or before prow holds prow
            const int rs = lane < n_groups ? a.groups[lane].row_start : 0x7fffffff;
            gi = 31 - __clz(__ballot_sync(0xffffffffu, rs <= prow));
        } else {
            gi = group_of_row(staged ? s_rs : nullptr, a.groups, n_groups, prow);
        }
        const GroupRec gr = a.groups[gi];
        const int r = prow - gr.row_start;
        const int nt = r / kTileCols;
        const int j = r - nt * kTileCols;
        const int NT = (gr.n_rows + kTileCols - 1) / kTileCols;
        const int kb0 = chunk * KBPT;
        // all source loads of the chunk first
        float v[KBPT][4];
#pragma unroll
        for (int i = 0; i < KBPT; ++i) {
            if (kb0 + i < KB) {
                load4(a, src_row, (kb0 + i) * kBlock + 4 * lane, split, v[i]);
            } else {
                v[i][0] = v[i][1] = v[i][2] = v[i][3] = 0.0f;
            }
        }
        const int tok = nt * kTileCols + j;
        const int TP = NT * kTileCols;
        const int c = lane >> 2;
        // Term sp carries the residual of the terms before it, scaled by its own power of two
        // fitted to the block's largest residual: a large element then limits the resolution
        // of the small ones in its block only through the first term.  The task's K blocks are
        // independent, so each term's block maxima of all of them are reduced side by side,
        // and each term is stored as soon as it is known.
#pragma unroll
        for (int sp = 0; sp < kSplits; ++sp) {
            if (sp >= a.terms) break;
            float m[KBPT];
#pragma unroll
            for (int i = 0; i < KBPT; ++i)
                m[i] = warp_max_nonneg(fmaxf(fmaxf(fabsf(v[i][0]), fabsf(v[i][1])), fmaxf(fabsf(v[i][2]), fabsf(v[i][3]))));
            // K-major, 128-byte swizzled placement: B row n = term * TP + token (TP = 8 NT),
            // 128 bytes of K per row, 16-byte chunk c of row n stored at chunk c ^ (n & 7);
            // the (group, kb) tile is terms x TP rows (3 terms: decode, 2 terms: prefill).
            const int n = sp * TP + tok;
            const int off = n * kBlock + (c ^ (n & 7)) * 16 + 4 * (lane & 3);
#pragma unroll
            for (int i = 0; i < KBPT; ++i) {
                const int kb = kb0 + i;
                if (kb >= KB) break;
                const float s = pow2_scale_for(m[i]);
                const float inv = pow2_recip(s);  // exact: s is a power of two
                // element e in byte e; the scaled residual of each is exact in fp32
                const uint32_t q01 = e4m3x2_rn(v[i][0] * inv, v[i][1] * inv);
                const uint32_t q23 = e4m3x2_rn(v[i][2] * inv, v[i][3] * inv);
                const float2 d01 = e4m3x2_to_f32x2(q01), d23 = e4m3x2_to_f32x2(q23);
                v[i][0] -= d01.x * s;
                v[i][1] -= d01.y * s;
                v[i][2] -= d23.x * s;
                v[i][3] -= d23.y * s;
                const uint32_t w = q01 | (q23 << 16);
                const int64_t gk = int64_t(gr.tile_base) * KB + int64_t(kb) * NT;  // (group, kb) tile
                *reinterpret_cast<uint32_t*>(a.bfrag + gk * (a.terms * kTileCols * kBlock) + off) = w;
                if (lane == 0) a.bscale[gk * kScalesPerTile + sp * TP + tok] = s;
            }
        }
    }
}

// One warp per packed row (task = (n-tile, token column)): pass 1 finds the row's max
// |v| over all K, pass 2 writes the two terms of every K block with that row's scale.  The
// second pass re-reads the row from L2.
__global__ void __launch_bounds__(256) pack_rows_kernel(PackActArgs a) {
    chain_wait();
    chain_release();
    const int KB = a.K / kBlock;
    const int n_tiles = a.meta->n_tiles;
    const int split = a.src_dtype == kSrcUpGatePartials ? a.meta->split_k : 1;
    const int lane = threadIdx.x & 31;
    const int64_t n_tasks = int64_t(n_tiles) * kTileCols;
    const int64_t warp_global = (int64_t(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
    const int64_t n_warps = (int64_t(gridDim.x) * blockDim.x) >> 5;
    for (int64_t task = warp_global; task < n_tasks; task += n_warps) {
        const int tile = static_cast<int>(task / kTileCols);
        const int j = static_cast<int>(task % kTileCols);
        const GroupRec gr = a.groups[a.tile_group[tile]];
        const int nt = tile - gr.tile_base;
        const int NT = (gr.n_rows + kTileCols - 1) / kTileCols;
        const int r = nt * kTileCols + j;
        if (r >= gr.n_rows) continue;  // unread accumulator columns need no data
        const int prow = gr.row_start + r;
        const int64_t src_row = a.row_map ? a.row_map[prow] : prow;
        float s;
        if (a.src_scale) {
            s = a.src_scale[src_row];  // the source row's scale, computed once (row_scale_kernel)
        } else {
            float amax = 0.0f;
            for (int kb0 = 0; kb0 < KB; kb0 += 4) {
                float v[4][4];
#pragma unroll
                for (int i = 0; i < 4; ++i)
                    if (kb0 + i < KB) load4(a, src_row, (kb0 + i) * kBlock + 4 * lane, split, v[i]);
#pragma unroll
                for (int i = 0; i < 4; ++i)
                    if (kb0 + i < KB)
                        amax = fmaxf(amax, fmaxf(fmaxf(fabsf(v[i][0]), fabsf(v[i][1])), fmaxf(fabsf(v[i][2]), fabsf(v[i][3]))));
            }
            amax = warp_max(amax);
            s = pow2_scale_for(amax);
        }
        const float inv = pow2_recip(s);  // exact: s is a power of two
        const int tok = r;
        const int TP = NT * kTileCols;
        const int c = lane >> 2;
        for (int kb0 = 0; kb0 < KB; kb0 += 4) {
            float v[4][4];
#pragma unroll
            for (int i = 0; i < 4; ++i)
                if (kb0 + i < KB) load4(a, src_row, (kb0 + i) * kBlock + 4 * lane, split, v[i]);
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const int kb = kb0 + i;
                if (kb >= KB) break;
                // element e in byte e of each term; the residual after the first is exact
                uint32_t q[2] = {0u, 0u};
                float rsd[4] = {v[i][0] * inv, v[i][1] * inv, v[i][2] * inv, v[i][3] * inv};
#pragma unroll
                for (int sp = 0; sp < 2; ++sp) {
                    const uint32_t q01 = e4m3x2_rn(rsd[0], rsd[1]);
                    const uint32_t q23 = e4m3x2_rn(rsd[2], rsd[3]);
                    q[sp] = q01 | (q23 << 16);
                    if (sp == 0) {
                        const float2 d01 = e4m3x2_to_f32x2(q01), d23 = e4m3x2_to_f32x2(q23);
                        rsd[0] -= d01.x;
                        rsd[1] -= d01.y;
                        rsd[2] -= d23.x;
                        rsd[3] -= d23.y;
                    }
                }
                // (group, kb) tile: 2 terms x TP rows x 128 B, swizzled as in pack_act_kernel
                const int64_t gk = int64_t(gr.tile_base) * KB + int64_t(kb) * NT;
                uint8_t* base = a.bfrag + gk * (2 * kTileCols * kBlock);
#pragma unroll
                for (int sp = 0; sp < 2; ++sp) {
                    const int n = sp * TP + tok;
                    *reinterpret_cast<uint32_t*>(base + n * kBlock + ((c ^ (n & 7)) * 16) + 4 * (lane & 3)) = q[sp];
                }
            }
        }
        if (lane == 0) a.bscale[prow] = s;
    }
}

// Prefill x, token-major.  A prefill call packs each x row for ~9 experts (its routes and
// the shared expert) with ONE power-of-two scale per token (row_scale_kernel), so every
// packed row of a token carries the same bytes.  One warp per (token, 8 K blocks): the
// chunk is loaded and quantized once, then stored into each packed row of the token
// (tk_row: token -> packed row per route, -1 where absent), placed as pack_rows_kernel
// places it.  x is read once instead of once per packed row, and quantized once.
__global__ void __launch_bounds__(256) pack_tokens_kernel(PackActArgs a) {
    __shared__ int32_t s_rs[kPackSmemGroups];
    chain_wait();
    chain_release();
    const int KB = a.K / kBlock;
    const int n_chunks = (KB + kPackKbPerTask - 1) / kPackKbPerTask;
    const int n_groups = a.meta->n_groups;
    const bool staged = n_groups <= kPackSmemGroups;
    if (staged)
        for (int g = threadIdx.x; g < n_groups; g += blockDim.x) s_rs[g] = a.groups[g].row_start;
    __syncthreads();
    const int lane = threadIdx.x & 31;
    const int c = lane >> 2;
    const int64_t n_tasks = int64_t(a.n_src) * n_chunks;
    const int64_t warp_global = (int64_t(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
    const int64_t n_warps = (int64_t(gridDim.x) * blockDim.x) >> 5;
    for (int64_t task = warp_global; task < n_tasks; task += n_warps) {
        const int t = static_cast<int>(task / n_chunks);
        const int chunk = static_cast<int>(task - int64_t(t) * n_chunks);
        int prow[16];
        bool any = false;
#pragma unroll
        for (int k = 0; k < 16; ++k) {
            prow[k] = k < a.K1 ? __ldg(a.tk_row + int64_t(t) * a.K1 + k) : -1;
            any |= prow[k] >= 0;
        }
        if (!any) continue;  // no packed row of this token in this call
        const float s = a.src_scale[t];
        const float inv = pow2_recip(s);  // exact: s is a power of two
        const int kb0 = chunk * kPackKbPerTask;
        float v[kPackKbPerTask][4];
#pragma unroll
        for (int i = 0; i < kPackKbPerTask; ++i) {
            if (kb0 + i < KB) {
                load4(a, t, (kb0 + i) * kBlock + 4 * lane, 1, v[i]);
            } else {
                v[i][0] = v[i][1] = v[i][2] = v[i][3] = 0.0f;
            }
        }
        uint32_t w0[kPackKbPerTask], w1[kPackKbPerTask];
#pragma unroll
        for (int i = 0; i < kPackKbPerTask; ++i) {
            // element e in byte e of each term; the residual after the first is exact
            const float r0 = v[i][0] * inv, r1 = v[i][1] * inv, r2 = v[i][2] * inv, r3 = v[i][3] * inv;
            const uint32_t q01 = e4m3x2_rn(r0, r1);
            const uint32_t q23 = e4m3x2_rn(r2, r3);
            const float2 d01 = e4m3x2_to_f32x2(q01), d23 = e4m3x2_to_f32x2(q23);
            w0[i] = q01 | (q23 << 16);
            w1[i] = e4m3x2_rn(r0 - d01.x, r1 - d01.y) | (e4m3x2_rn(r2 - d23.x, r3 - d23.y) << 16);
        }
#pragma unroll
        for (int k = 0; k < 16; ++k) {
            if (prow[k] < 0) continue;
            const GroupRec gr = a.groups[group_of_row(staged ? s_rs : nullptr, a.groups, n_groups, prow[k])];
            const int tok = prow[k] - gr.row_start;
            const int NT = (gr.n_rows + kTileCols - 1) / kTileCols;
            const int n0 = tok, n1 = NT * kTileCols + tok;
            const int off0 = n0 * kBlock + ((c ^ (n0 & 7)) * 16) + 4 * (lane & 3);
            const int off1 = n1 * kBlock + ((c ^ (n1 & 7)) * 16) + 4 * (lane & 3);
#pragma unroll
            for (int i = 0; i < kPackKbPerTask; ++i) {
                const int kb = kb0 + i;
                if (kb >= KB) break;
                // (group, kb) tile: 2 terms x TP rows x 128 B, swizzled as in pack_act_kernel
                uint8_t* base = a.bfrag + (int64_t(gr.tile_base) * KB + int64_t(kb) * NT) * (2 * kTileCols * kBlock);
                *reinterpret_cast<uint32_t*>(base + off0) = w0[i];
                *reinterpret_cast<uint32_t*>(base + off1) = w1[i];
            }
            if (chunk == 0 && lane == 0) a.bscale[prow[k]] = s;
        }
    }
}

// pack_rows_kernel for rows of at most kRowRegBlocks K blocks with no precomputed scale (h:
// I = 2048 -> 16 blocks): the row is loaded once into registers, 4 elements per lane per
// K block, its max |v| reduced there and both terms written from the registers -- one pass
// over the up/gate partials instead of two (a prefill chunk's partials exceed the L2, so
// the second pass re-read them from HBM).  Same scale, bytes and placement as
// pack_rows_kernel.
constexpr int kRowRegBlocks = 16;
__global__ void __launch_bounds__(256) pack_rows_reg_kernel(PackActArgs a) {
    chain_wait();
    chain_release();
    const int KB = a.K / kBlock;
    const int n_tiles = a.meta->n_tiles;
    const int split = a.src_dtype == kSrcUpGatePartials ? a.meta->split_k : 1;
    const int lane = threadIdx.x & 31;
    const int64_t n_tasks = int64_t(n_tiles) * kTileCols;
    const int64_t warp_global = (int64_t(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
    const int64_t n_warps = (int64_t(gridDim.x) * blockDim.x) >> 5;
    for (int64_t task = warp_global; task < n_tasks; task += n_warps) {
        const int tile = static_cast<int>(task / kTileCols);
        const int j = static_cast<int>(task % kTileCols);
        const GroupRec gr = a.groups[a.tile_group[tile]];
        const int nt = tile - gr.tile_base;
        const int NT = (gr.n_rows + kTileCols - 1) / kTileCols;
        const int r = nt * kTileCols + j;
        if (r >= gr.n_rows) continue;  // unread accumulator columns need no data
        const int prow = gr.row_start + r;
        const int64_t src_row = a.row_map ? a.row_map[prow] : prow;
        float v[kRowRegBlocks][4];
#pragma unroll
        for (int i = 0; i < kRowRegBlocks; ++i) {
            if (i < KB) {
                load4(a, src_row, i * kBlock + 4 * lane, split, v[i]);
            } else {
                v[i][0] = v[i][1] = v[i][2] = v[i][3] = 0.0f;
            }
        }
        float amax = 0.0f;
#pragma unroll
        for (int i = 0; i < kRowRegBlocks; ++i)
            amax = fmaxf(amax, fmaxf(fmaxf(fabsf(v[i][0]), fabsf(v[i][1])), fmaxf(fabsf(v[i][2]), fabsf(v[i][3]))));
        amax = warp_max(amax);
        const float s = pow2_scale_for(amax);
        const float inv = pow2_recip(s);  // exact: s is a power of two
        const int tok = r;
        const int TP = NT * kTileCols;
        const int c = lane >> 2;
#pragma unroll
        for (int i = 0; i < kRowRegBlocks; ++i) {
            if (i >= KB) break;
            // element e in byte e of each term; the residual after the first is exact
            float rsd[4] = {v[i][0] * inv, v[i][1] * inv, v[i][2] * inv, v[i][3] * inv};
            const uint32_t q01 = e4m3x2_rn(rsd[0], rsd[1]);
            const uint32_t q23 = e4m3x2_rn(rsd[2], rsd[3]);
            const float2 d01 = e4m3x2_to_f32x2(q01), d23 = e4m3x2_to_f32x2(q23);
            const uint32_t w0 = q01 | (q23 << 16);
            const uint32_t w1 = e4m3x2_rn(rsd[0] - d01.x, rsd[1] - d01.y) | (e4m3x2_rn(rsd[2] - d23.x, rsd[3] - d23.y) << 16);
            // (group, kb) tile: 2 terms x TP rows x 128 B, swizzled as in pack_act_kernel
            const int64_t gk = int64_t(gr.tile_base) * KB + int64_t(i) * NT;
            uint8_t* base = a.bfrag + gk * (2 * kTileCols * kBlock);
            const int n0 = tok, n1 = TP + tok;
            *reinterpret_cast<uint32_t*>(base + n0 * kBlock + ((c ^ (n0 & 7)) * 16) + 4 * (lane & 3)) = w0;
            *reinterpret_cast<uint32_t*>(base + n1 * kBlock + ((c ^ (n1 & 7)) * 16) + 4 * (lane & 3)) = w1;
        }
        if (lane == 0) a.bscale[prow] = s;
    }
}

// One warp per source row: the power-of-two scale pack_rows_kernel would find for it
// (max |v| over the row -> pow2_scale_for).  Lets the x packer run one pass when a token
// appears in several packed rows.
__global__ void __launch_bounds__(256) row_scale_kernel(PackActArgs a, int n_src_rows, float* out) {
    chain_wait();
    chain_release();
    const int KB = a.K / kBlock;
    const int lane = threadIdx.x & 31;
    const int64_t warp_global = (int64_t(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
    const int64_t n_warps = (int64_t(gridDim.x) * blockDim.x) >> 5;
    for (int64_t row = warp_global; row < n_src_rows; row += n_warps) {
        float amax = 0.0f;
        for (int kb0 = 0; kb0 < KB; kb0 += 8) {  // 8 loads in flight per round
            float v[8][4];
#pragma unroll
            for (int i = 0; i < 8; ++i)
                if (kb0 + i < KB) load4(a, row, (kb0 + i) * kBlock + 4 * lane, 1, v[i]);
#pragma unroll
            for (int i = 0; i < 8; ++i)
                if (kb0 + i < KB)
                    amax = fmaxf(amax, fmaxf(fmaxf(fabsf(v[i][0]), fabsf(v[i][1])), fmaxf(fabsf(v[i][2]), fabsf(v[i][3]))));
        }
        amax = warp_max(amax);
        if (lane == 0) out[row] = pow2_scale_for(amax);
    }
}

cudaError_t launch_row_scale(const PackActArgs& a, int n_src_rows, float* out, int num_sms, cudaStream_t stream) {
    if (a.src_dtype == kSrcUpGatePartials) return cudaErrorInvalidValue;
    if (n_src_rows == 0) return cudaSuccess;
    return launch_chained(row_scale_kernel, dim3(num_sms * 4), dim3(256), 0, stream, a, n_src_rows, out);
}



// CTAs of `kernel` (256 threads) resident on one SM at once; 1 if the query fails
template <typename K>
static int resident_ctas(K kernel) {
    int n = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, kernel, 256, 0) != cudaSuccess || n < 1) {
        cudaGetLastError();
        return 1;
    }
    return n;
}

cudaError_t launch_pack_rows(const PackActArgs& a, int num_sms, cudaStream_t stream) {
    if (a.terms != 2) return cudaErrorInvalidValue;
    if (a.src_scale == nullptr && a.K / kBlock <= kRowRegBlocks) {
        static const int occ = resident_ctas(pack_rows_reg_kernel);
        return launch_chained(pack_rows_reg_kernel, dim3(num_sms * occ), dim3(256), 0, stream, a);
    }
    if (a.src_scale != nullptr && a.tk_row != nullptr && a.src_dtype != kSrcUpGatePartials) {
        static const int occ = resident_ctas(pack_tokens_kernel);
        return launch_chained(pack_tokens_kernel, dim3(num_sms * occ), dim3(256), 0, stream, a);
    }
    return launch_chained(pack_rows_kernel, dim3(num_sms * 8), dim3(256), 0, stream, a);
}

// CTAs for a dense-row launch: one wave (the row count is known on the device only, the
// loop strides over it), or fewer when the host's bound on the rows needs fewer warps
static int pack_grid(const PackActArgs& a, int kbpt, int num_sms, int occ) {
    int64_t grid = int64_t(num_sms) * occ;
    if (a.rows_hint > 0) {
        const int64_t tasks = int64_t(a.rows_hint) * ((a.K / kBlock + kbpt - 1) / kbpt);
        grid = std::min<int64_t>(grid, std::max<int64_t>(1, (tasks + 7) / 8));  // 8 warps per CTA
    }
    return static_cast<int>(grid);
}

cudaError_t launch_pack_act(const PackActArgs& a, int num_sms, cudaStream_t stream) {
    if (a.src_dtype == kSrcUpGatePartials) {
        static const int occ = resident_ctas(pack_act_kernel<2>);
        return launch_chained(pack_act_kernel<2>, dim3(pack_grid(a, 2, num_sms, occ)), dim3(256), 0, stream, a);
    }
    static const int occ = resident_ctas(pack_act_kernel<kPackKbPerTask>);
    return launch_chained(pack_act_kernel<kPackKbPerTask>, dim3(pack_grid(a, kPackKbPerTask, num_sms, occ)),
                          dim3(256), 0, stream, a);
}

}  // namespace cst
