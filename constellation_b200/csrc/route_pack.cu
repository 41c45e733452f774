// Dispatch planning: turn (token, k) -> expert routes into expert-sorted packed rows.
//
// Replaces the reference's per-(token, expert) dispatch loop (dispatch_topk_experts,
// server/moe_layer_runtime.py:111-145, and the placement lookup find_expert_placement,
// server/expert_placement.py:101-106): instead of one socket request per route, every
// route that targets an expert resident on this device becomes one row of a packed
// activation matrix whose rows are sorted by (expert slot, token, k).  The rows of one
// slot are cut into groups of at most 16 rows (two 8-wide MMA n-tiles) that the grouped
// FFN kernels consume.
//
// Decode-sized calls (<= 2048 routes, <= 1024 slots): one CTA of 1024 threads runs a stable
// counting sort by slot.  Warp w owns a contiguous block of routes and counts its routes per
// slot; one pass over the slots turns the per-warp counts into running offsets (warp order)
// and block scans give every slot's first row, group and tile; each warp then places its
// routes in order -- __match_any_sync groups the lanes of a 32-route chunk by slot, and a
// lane's position is its slot's running offset plus the number of lower peer lanes.  Rows
// are therefore sorted by (slot, token, k); no atomic decides an order (they only count).
// Routes whose expert is not resident here get no row (under expert parallelism they
// belong to another rank).  Larger calls take the three-launch counting sort below, which
// yields the same rows in the same order.
#include <cstdint>

#include "cst_common.cuh"
#include "kernels.h"
#include "layout.cuh"

namespace cst {

constexpr int kPackThreads = 1024;
constexpr int kRankSortMaxKeys = 2048;  // up to here one CTA packs; beyond, the three-launch counting sort
constexpr int kPackWarps = kPackThreads / 32;
constexpr int kPackMaxSlotsOneCta = 1024;  // more slots: the multi-CTA counting sort
constexpr int kRoutePackMaxSmem = (kRankSortMaxKeys + (kPackWarps + 2) * kPackMaxSlotsOneCta) * 4;


__device__ __forceinline__ int block_exclusive_scan(int v, int* s_warp, int* total) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    int x = v;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const int y = __shfl_up_sync(0xffffffffu, x, o);
        if (lane >= o) x += y;
    }
    if (lane == 31) s_warp[warp] = x;
    __syncthreads();
    if (warp == 0) {
        int w = s_warp[lane];
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int y = __shfl_up_sync(0xffffffffu, w, o);
            if (lane >= o) w += y;
        }
        s_warp[lane] = w;  // inclusive over warps
    }
    __syncthreads();
    const int warp_prefix = (warp == 0) ? 0 : s_warp[warp - 1];
    const int tot = s_warp[31];
    __syncthreads();
    *total = tot;
    return warp_prefix + x - v;
}

// Route i -> (token t, k, slot); slot -1 when the route has no row on this device.
__device__ __forceinline__ int route_slot(const PackArgs& a, bool mode_rows, int K1, int i, int* t, int* k) {
    int slot;
    if (mode_rows) {
        *t = i;
        *k = 0;
        slot = a.row_slot ? a.row_slot[i] : a.single_slot;
    } else {
        *t = i / K1;
        *k = i % K1;
        if (*k < a.K) {
            const int e = a.topk_idx[*t * a.K + *k];
            slot = (e >= 0 && e < a.E) ? a.slot_of_expert[e] : -1;
            if (slot >= 0 && (slot & kSlotOwnTokensOnly)) {
                // a replicated expert: this rank serves it for its own tokens only
                slot = (*t >= a.shared_t_begin && *t < a.shared_t_end) ? (slot & ~kSlotOwnTokensOnly) : -1;
            }
        } else {
            slot = (*t >= a.shared_t_begin && *t < a.shared_t_end) ? a.shared_slot : -1;
        }
    }
    return (slot >= 0 && slot < a.n_slots) ? slot : -1;
}

__global__ void __launch_bounds__(kPackThreads) route_pack_kernel(PackArgs a) {
    // shared: route slots [kRankSortMaxKeys]; per (warp, slot) counts, then running offsets
    // [32][n_slots]; per slot: count, first row
    extern __shared__ int s_mem[];
    int* s_slot = s_mem;
    int* s_wcnt = s_slot + kRankSortMaxKeys;
    int* s_cnt = s_wcnt + kPackWarps * a.n_slots;
    int* s_first = s_cnt + a.n_slots;
    chain_wait();
    chain_release();
    __shared__ int s_warp[32];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const bool mode_rows = (a.row_slot != nullptr) || (a.single_slot >= 0);
    const int K1 = mode_rows ? 1 : a.K + 1;
    const int n_routes = mode_rows ? a.T : a.T * K1;
    const int G = a.group_rows;
    // warp w owns the contiguous routes [w B, w B + B): keeping them in order inside the
    // warp and the warps in order keeps every slot's rows in route order
    const int B = (n_routes + kPackWarps - 1) / kPackWarps;
    const int r_begin = warp * B, r_end = min(n_routes, r_begin + B);
    for (int i = tid; i < kPackWarps * a.n_slots; i += kPackThreads) s_wcnt[i] = 0;
    for (int i = tid; i < n_routes; i += kPackThreads) {
        int t, k;
        s_slot[i] = route_slot(a, mode_rows, K1, i, &t, &k);
    }
    __syncthreads();
    for (int i = r_begin + lane; i < r_end; i += 32) {
        const int sl = s_slot[i];
        if (sl >= 0) atomicAdd(&s_wcnt[warp * a.n_slots + sl], 1);  // counts: order immaterial
    }
    __syncthreads();
    // per slot: total, and each warp's running offset inside the slot (warp order)
    for (int sl = tid; sl < a.n_slots; sl += kPackThreads) {
        int run = 0;
        for (int w = 0; w < kPackWarps; ++w) {
            const int v = s_wcnt[w * a.n_slots + sl];
            s_wcnt[w * a.n_slots + sl] = run;
            run += v;
        }
        s_cnt[sl] = run;
    }
    __syncthreads();
    // first row / group / tile of every slot: block scans over contiguous slot ranges
    const int per = (a.n_slots + kPackThreads - 1) / kPackThreads;
    const int s0 = min(a.n_slots, tid * per), s1 = min(a.n_slots, s0 + per);
    int rows_l = 0, groups_l = 0, tiles_l = 0;
    for (int sl = s0; sl < s1; ++sl) {
        const int n = s_cnt[sl];
        rows_l += n;
        groups_l += (n + G - 1) / G;
        tiles_l += (n / G) * ((G + kTileCols - 1) / kTileCols) + ((n % G) + kTileCols - 1) / kTileCols;
    }
    int n_rows, n_groups, n_tiles;
    int row = block_exclusive_scan(rows_l, s_warp, &n_rows);
    int g = block_exclusive_scan(groups_l, s_warp, &n_groups);
    int tile = block_exclusive_scan(tiles_l, s_warp, &n_tiles);
    const bool overflow = (n_rows > a.max_rows) || (n_groups > a.max_groups);
    for (int sl = s0; sl < s1; ++sl) {
        const int n = s_cnt[sl];
        s_first[sl] = row;
        if (!overflow) {
            for (int j = 0; j * G < n; ++j) {
                const int rows = min(G, n - j * G);
                const int nt = (rows + kTileCols - 1) / kTileCols;
                a.groups[g] = GroupRec{sl, row + j * G, rows, tile};
                for (int q = 0; q < nt; ++q) a.tile_group[tile + q] = g;
                ++g;
                tile += nt;
            }
        }
        row += n;
    }
    __syncthreads();
    // place every route: slot order, then route (= token, k) order inside a slot
    for (int i = tid; i < n_routes; i += kPackThreads)
        if (s_slot[i] < 0 || overflow) a.tk_row[i] = -1;
    if (!overflow) {
        for (int c = r_begin; c < r_end; c += 32) {
            const int i = c + lane;
            const int sl = i < r_end ? s_slot[i] : -1;
            const uint32_t peers = __match_any_sync(0xffffffffu, sl);
            int base = 0;
            if (sl >= 0) {
                base = s_wcnt[warp * a.n_slots + sl];
                const int p = s_first[sl] + base + __popc(peers & ((1u << lane) - 1u));
                const int t = mode_rows ? i : i / K1;
                const int k = mode_rows ? 0 : i % K1;
                a.row_token[p] = t;
                float wt = 1.0f;
                if (mode_rows) {
                    if (a.row_weight_in) wt = a.row_weight_in[t];
                } else if (k < a.K) {
                    wt = a.topk_w[t * a.K + k];
                }
                a.row_weight[p] = wt;
                a.tk_row[i] = p;  // i = t * K1 + k
            }
            __syncwarp();
            if (sl >= 0 && lane == __ffs(peers) - 1) s_wcnt[warp * a.n_slots + sl] = base + __popc(peers);
            __syncwarp();
        }
    }
    if (tid == 0) {
        a.meta->n_rows = overflow ? 0 : n_rows;
        a.meta->n_groups = overflow ? 0 : n_groups;
        a.meta->n_tiles = overflow ? 0 : n_tiles;
        a.meta->overflow = overflow ? 1 : 0;
    }
}

// ---------------------------------------------------------------------------------------
// Large batches (more than kRankSortMaxKeys routes, e.g. a 4096-token prefill chunk): a
// three-launch counting sort over slots instead of one CTA sorting every key.
//   count:   chunk c of kPackThreads routes -> hist[c][slot] (shared-memory histogram)
//   scan:    one CTA turns hist into each (chunk, slot)'s first packed row, numbers the
//            groups slot by slot and writes the group records, tile map and meta
//   scatter: each route's row = hist[c][slot] + the number of earlier routes of chunk c
//            with the same slot
// Rows of one slot therefore come in (token, k) order, as the sort gives them, and the
// result is identical to the single-CTA path: same rows, same groups, same order.

__global__ void __launch_bounds__(kPackThreads) route_count_kernel(PackArgs a) {
    extern __shared__ int s_hist[];
    chain_wait();
    chain_release();
    const bool mode_rows = (a.row_slot != nullptr) || (a.single_slot >= 0);
    const int K1 = mode_rows ? 1 : a.K + 1;
    const int n_routes = mode_rows ? a.T : a.T * K1;
    for (int s = threadIdx.x; s < a.n_slots; s += kPackThreads) s_hist[s] = 0;
    __syncthreads();
    const int i = blockIdx.x * kPackThreads + threadIdx.x;
    if (i < n_routes) {
        int t, k;
        const int slot = route_slot(a, mode_rows, K1, i, &t, &k);
        if (slot >= 0) atomicAdd(&s_hist[slot], 1);  // a count: the order of adds is immaterial
    }
    __syncthreads();
    for (int s = threadIdx.x; s < a.n_slots; s += kPackThreads)
        a.hist[int64_t(blockIdx.x) * a.n_slots + s] = s_hist[s];
}

__global__ void __launch_bounds__(kPackThreads) route_scan_kernel(PackArgs a, int n_chunks) {
    extern __shared__ int s_tot[];  // per slot: routes, then (reused) first row
    __shared__ int s_warp[32];
    chain_wait();
    chain_release();
    const int tid = threadIdx.x;
    // per slot: running count over chunks (exclusive, in place) and the slot total
    for (int s = tid; s < a.n_slots; s += kPackThreads) {
        int run = 0;
        for (int c = 0; c < n_chunks; ++c) {
            int* h = &a.hist[int64_t(c) * a.n_slots + s];
            const int v = *h;
            *h = run;
            run += v;
        }
        s_tot[s] = run;
    }
    __syncthreads();
    // each thread owns a contiguous range of slots for the block scans
    const int per = (a.n_slots + kPackThreads - 1) / kPackThreads;
    const int s0 = min(a.n_slots, tid * per), s1 = min(a.n_slots, s0 + per);
    const int G = a.group_rows;
    int rows_l = 0, groups_l = 0, tiles_l = 0;
    for (int s = s0; s < s1; ++s) {
        const int n = s_tot[s];
        rows_l += n;
        groups_l += (n + G - 1) / G;
        tiles_l += (n / G) * ((G + kTileCols - 1) / kTileCols) + ((n % G) + kTileCols - 1) / kTileCols;
    }
    int n_rows, n_groups, n_tiles;
    int row = block_exclusive_scan(rows_l, s_warp, &n_rows);
    int g = block_exclusive_scan(groups_l, s_warp, &n_groups);
    int tile = block_exclusive_scan(tiles_l, s_warp, &n_tiles);
    const bool overflow = (n_rows > a.max_rows) || (n_groups > a.max_groups);
    for (int s = s0; s < s1; ++s) {
        const int n = s_tot[s];
        s_tot[s] = row;  // first row of slot s
        if (!overflow) {
            for (int j = 0; j * G < n; ++j) {
                const int rows = min(G, n - j * G);
                const int nt = (rows + kTileCols - 1) / kTileCols;
                a.groups[g] = GroupRec{s, row + j * G, rows, tile};
                for (int q = 0; q < nt; ++q) a.tile_group[tile + q] = g;
                ++g;
                tile += nt;
            }
        }
        row += n;
    }
    __syncthreads();
    for (int s = tid; s < a.n_slots; s += kPackThreads) {
        const int first = s_tot[s];
        for (int c = 0; c < n_chunks; ++c) a.hist[int64_t(c) * a.n_slots + s] += first;
    }
    if (tid == 0) {
        a.meta->n_rows = overflow ? 0 : n_rows;
        a.meta->n_groups = overflow ? 0 : n_groups;
        a.meta->n_tiles = overflow ? 0 : n_tiles;
        a.meta->overflow = overflow ? 1 : 0;
    }
}

__global__ void __launch_bounds__(kPackThreads) route_scatter_kernel(PackArgs a) {
    __shared__ int s_slot[kPackThreads];
    chain_wait();
    chain_release();
    const bool mode_rows = (a.row_slot != nullptr) || (a.single_slot >= 0);
    const int K1 = mode_rows ? 1 : a.K + 1;
    const int n_routes = mode_rows ? a.T : a.T * K1;
    const int i = blockIdx.x * kPackThreads + threadIdx.x;
    int t = 0, k = 0, slot = -1;
    if (i < n_routes) slot = route_slot(a, mode_rows, K1, i, &t, &k);
    s_slot[threadIdx.x] = slot;
    __syncthreads();
    if (i >= n_routes) return;
    if (slot < 0 || a.meta->overflow) {
        a.tk_row[i] = -1;
        return;
    }
    int rank = 0;
    for (int j = 0; j < int(threadIdx.x); ++j) rank += s_slot[j] == slot;
    const int p = a.hist[int64_t(blockIdx.x) * a.n_slots + slot] + rank;
    a.row_token[p] = t;
    float wt = 1.0f;
    if (mode_rows) {
        if (a.row_weight_in) wt = a.row_weight_in[t];
    } else if (k < a.K) {
        wt = a.topk_w[t * a.K + k];
    }
    a.row_weight[p] = wt;
    a.tk_row[i] = p;  // i = t * K1 + k
}

cudaError_t route_pack_init_attributes() {
    return cudaFuncSetAttribute(route_pack_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                kRoutePackMaxSmem);
}

int route_pack_chunks(int n_routes) { return (n_routes + kPackThreads - 1) / kPackThreads; }

cudaError_t launch_route_pack(const PackArgs& a, cudaStream_t stream) {
    const bool mode_rows = (a.row_slot != nullptr) || (a.single_slot >= 0);
    const int n_routes = mode_rows ? a.T : a.T * (a.K + 1);
    if (n_routes > kRankSortMaxKeys || a.n_slots > kPackMaxSlotsOneCta) {
        const int chunks = route_pack_chunks(n_routes);
        if (int64_t(chunks) * a.n_slots > a.hist_cap) return cudaErrorInvalidValue;
        const size_t hs = size_t(a.n_slots) * sizeof(int);
        cudaError_t e = launch_chained(route_count_kernel, dim3(chunks), dim3(kPackThreads), hs, stream, a);
        if (e == cudaSuccess) e = launch_chained(route_scan_kernel, dim3(1), dim3(kPackThreads), hs, stream, a, chunks);
        if (e == cudaSuccess) e = launch_chained(route_scatter_kernel, dim3(chunks), dim3(kPackThreads), 0, stream, a);
        return e;
    }
    const size_t smem = size_t(kRankSortMaxKeys + (kPackWarps + 2) * a.n_slots) * sizeof(int);
    return launch_chained(route_pack_kernel, dim3(1), dim3(kPackThreads), smem, stream, a);
}

}  // namespace cst
