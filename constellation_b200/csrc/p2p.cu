// Peer-memory exchange for expert parallelism: the all-gather of the tokens' rows and the
// combine of the routed (and shared) expert outputs fused with the cross-rank reduction,
// both over NVLink stores.
//
//   gather_push_kernel + gather_wait_kernel: every rank stores its own rows into every
//     rank's gathered-row slots and counts them there; the owner waits (bounded) for all
//     ranks' rows before the router reads them.  A rank's slots are rewritten by the next
//     exchange only after every rank has pushed the combine of this one, which each rank
//     does after its last read of the gathered rows (the activation packer), so one slot
//     set per rank suffices here too.
//
// The reference reduces nothing across GPUs -- its coordinator gathers one expert result
// per (token, expert) socket request and sums them on the host (server/moe_layer_runtime.py
// :111-229).  Here every rank holds a quarter / an eighth of the experts and, after the
// grouped kernels, a weighted output row per (gathered token, local route).  Instead of
// adding them into an fp32 [T, H] partial and handing that to an NCCL reduce-scatter:
//
//   combine_push_kernel  (one CTA per (owner rank, 4-token block, 1024-column chunk)): each
//     of those tokens' rows in the fixed k order, the sum stored straight into the OWNING rank's
//     receive buffer (slot [this rank][token - owner * tl]) through the peer mapping, then
//     one release-ordered add on the owner's arrival counter for this rank.
//   reduce_cast_kernel   (one CTA per (own token, chunk)): waits -- bounded -- until every
//     rank's counter shows all its pushing CTAs of this exchange, then adds the
//     world partial sums in rank order, the residual, and casts once.
//
// Ordering: the add is a release at system scope, cumulative over the CTA's stores through
// the barrier before it, and the reader polls with acquire loads, so a reader that sees the
// count sees every partial it covers.  The epoch word is a device counter that every rank
// advances by the same amount per exchange, so CUDA graphs replay it unchanged.  Counters
// and epoch are 32-bit words that wrap (a long-lived server passes 2^31 pushing CTAs within
// days), so "arrived" is the sign of the wrapped difference, never a plain comparison; a
// counter trails its target by at most the CTAs of one exchange, far below 2^31.  A receive
// slot is rewritten only by the next exchange's push, which a rank issues after that
// exchange's gather -- and every rank starts its gather only after finishing its own reduce
// of this exchange -- so one buffer per rank suffices.
#include <cstdint>
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include "cst_common.cuh"
#include "kernels.h"

namespace cst {

namespace {

__device__ __forceinline__ uint32_t ld_acquire_sys(const int32_t* p) {
    uint32_t v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];\n" : "=r"(v) : "l"(p) : "memory");
    return v;
}

__device__ __forceinline__ void red_release_sys_add(int32_t* p, uint32_t v) {
    asm volatile("red.release.sys.global.add.u32 [%0], %1;\n" ::"l"(p), "r"(v) : "memory");
}

// counter `have` has not reached `want` yet, modulo 2^32
__device__ __forceinline__ bool before(uint32_t have, uint32_t want) { return int32_t(have - want) < 0; }

// grid (world x token blocks, column chunks): CTA (q, b, c) sums the rows of owner q's
// tokens [b kPushTok, b kPushTok + kPushTok) over its 1024-column chunk and stores them into
// q's slot [this rank]; then one release-ordered add on q's arrival counter for this rank
// (cumulative over the CTA's stores through the barrier).  CTA (0, 0) also advances this
// rank's epoch word by the number of pushing CTAs per owner, which the reduce launch reads.
__global__ void __launch_bounds__(256) combine_push_kernel(PushArgs a) {
    const int nblk = (a.tl + kPushTok - 1) / kPushTok;
    const int q = blockIdx.x / nblk;
    const int i0 = (blockIdx.x - q * nblk) * kPushTok;
    const int h = (blockIdx.y * blockDim.x + threadIdx.x) * 4;
    float* dst = a.peers.recv[q] + int64_t(a.peers.rank) * a.peers.tl_cap * a.H;
    // presence words of this rank in q's buffer: a token with no row here is not pushed
    int32_t* pres = a.peers.pres_off
                        ? reinterpret_cast<int32_t*>(reinterpret_cast<uint8_t*>(a.peers.recv[q]) + a.peers.pres_off) +
                              int64_t(a.peers.rank) * a.peers.tl_cap
                        : nullptr;
    const int i_end = min(a.tl, i0 + kPushTok);
    // a token's row indices are loaded together, the next token's while this one is summed
    int nxt[16];
    auto load_rows = [&](int i, int (&r)[16]) {
        const int32_t* rows = a.tk_row + int64_t(q * a.tl + i) * a.K1;
#pragma unroll
        for (int k = 0; k < 16; ++k) r[k] = (k < a.K1) ? __ldg(rows + k) : -1;
    };
    if (i0 < i_end) load_rows(i0, nxt);
    for (int i = i0; i < i_end; ++i) {
        int rw[16];
#pragma unroll
        for (int k = 0; k < 16; ++k) rw[k] = nxt[k];
        if (i + 1 < i_end) load_rows(i + 1, nxt);
        bool present = pres == nullptr;
#pragma unroll
        for (int k = 0; k < 16; ++k) present |= rw[k] >= 0;
        if (pres != nullptr && blockIdx.y == 0 && threadIdx.x == 0) pres[i] = present ? 1 : 0;
        if (!present || h >= a.H) continue;
        {
            float4 v[16];
#pragma unroll
            for (int k = 0; k < 16; ++k) {
                const int r = rw[k];
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
            *reinterpret_cast<float4*>(dst + int64_t(i) * a.H + h) = acc;  // local or peer store (NVLink)
        }
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        red_release_sys_add(a.peers.flags[q] + a.peers.rank, 1u);
        // the epoch word counts the pushing CTAs every rank sends each rank, summed over
        // all exchanges so far (every rank runs the same exchanges with the same tl)
        if (blockIdx.x == 0 && blockIdx.y == 0) {
            uint32_t* epoch = reinterpret_cast<uint32_t*>(a.peers.epoch);
            *epoch += gridDim.y * uint32_t((a.tl + kPushTok - 1) / kPushTok);
        }
    }
}

// The all-gather half.  grid (world x row blocks): CTA (q, b) copies this rank's rows
// [b kGatherRows, b kGatherRows + kGatherRows) into rank q's gathered-row slots (row
// rank * tl + i) with 16-byte stores, then one release-ordered add on q's gather counter
// for this rank.  CTA (0, 0) advances this rank's gather epoch by the blocks per owner.
__global__ void __launch_bounds__(256) gather_push_kernel(GatherArgs a) {
    const int nblk = (a.tl + kGatherRows - 1) / kGatherRows;
    const int q = blockIdx.x / nblk;
    const int r0 = (blockIdx.x - q * nblk) * kGatherRows;
    const int rows = min(a.tl, r0 + kGatherRows) - r0;
    const int64_t row16 = int64_t(a.H) * 2 / 16;  // 16-byte units per row
    const uint4* src = reinterpret_cast<const uint4*>(a.x) + int64_t(r0) * row16;
    uint4* dst = reinterpret_cast<uint4*>(reinterpret_cast<uint8_t*>(a.peers.recv[q]) + a.peers.x_off) +
                 (int64_t(a.peers.rank) * a.tl + r0) * row16;
    for (int64_t i = threadIdx.x; i < rows * row16; i += blockDim.x) dst[i] = __ldg(src + i);  // local or peer store
    __syncthreads();
    if (threadIdx.x == 0) {
        red_release_sys_add(a.peers.flags[q] + kGatherFlags + a.peers.rank, 1u);
        if (blockIdx.x == 0) {
            uint32_t* epoch = reinterpret_cast<uint32_t*>(a.peers.gather_epoch);
            *epoch += uint32_t(nblk);
        }
    }
}

// One warp: lane r waits (bounded, like reduce_cast_kernel) until rank r's gather counter
// here covers every block of this exchange; a wait that gives up sets the error word.  The
// kernels after it on the stream read the gathered rows.
__global__ void __launch_bounds__(32) gather_wait_kernel(GatherArgs a) {
    const int r = threadIdx.x;
    if (r >= a.peers.world) return;
    const uint32_t target = *reinterpret_cast<const uint32_t*>(a.peers.gather_epoch);
    const int32_t* flag = a.peers.flags[a.peers.rank] + kGatherFlags + r;
    uint32_t n = 0;
    while (before(ld_acquire_sys(flag), target)) {
        if (++n >= (1u << 22)) {
            if (a.err) atomicMax(a.err, CST_DEV_ERR_TIMEOUT);
            return;
        }
        __nanosleep(100);
    }
}

template <int OUT>
__device__ __forceinline__ void store_out(void* out, int64_t o, float4 v) {
    if constexpr (OUT == 3) {
        *reinterpret_cast<float4*>(static_cast<float*>(out) + o) = v;
    } else if constexpr (OUT == 2) {
        const __nv_bfloat162 lo = __floats2bfloat162_rn(v.x, v.y), hi = __floats2bfloat162_rn(v.z, v.w);
        uint2 u;
        u.x = *reinterpret_cast<const uint32_t*>(&lo);
        u.y = *reinterpret_cast<const uint32_t*>(&hi);
        *reinterpret_cast<uint2*>(static_cast<uint16_t*>(out) + o) = u;
    } else {
        const __half2 lo = __floats2half2_rn(v.x, v.y), hi = __floats2half2_rn(v.z, v.w);
        uint2 u;
        u.x = *reinterpret_cast<const uint32_t*>(&lo);
        u.y = *reinterpret_cast<const uint32_t*>(&hi);
        *reinterpret_cast<uint2*>(static_cast<uint16_t*>(out) + o) = u;
    }
}

__device__ __forceinline__ float4 load4_any(const void* p, int dtype, int64_t idx) {
    if (dtype == 3) return *reinterpret_cast<const float4*>(static_cast<const float*>(p) + idx);
    const uint2 u = *reinterpret_cast<const uint2*>(static_cast<const uint16_t*>(p) + idx);
    if (dtype == 2)
        return make_float4(__uint_as_float(u.x << 16), __uint_as_float(u.x & 0xffff0000u), __uint_as_float(u.y << 16),
                           __uint_as_float(u.y & 0xffff0000u));
    const float2 lo = __half22float2(*reinterpret_cast<const __half2*>(&u.x));
    const float2 hi = __half22float2(*reinterpret_cast<const __half2*>(&u.y));
    return make_float4(lo.x, lo.y, hi.x, hi.y);
}

template <int OUT>
__global__ void __launch_bounds__(256) reduce_cast_kernel(ReduceArgs a) {
    __shared__ int s_ok;
    const int t = blockIdx.x;  // own token
    if (threadIdx.x == 0) {
        // every rank's pushing CTAs for this rank, over all exchanges up to this one
        const uint32_t target = *reinterpret_cast<const uint32_t*>(a.peers.epoch);
        const int32_t* flags = a.peers.flags[a.peers.rank];
        bool ok = true;
        for (int r = 0; r < a.peers.world && ok; ++r) {
            // bounded: 2^22 polls with a short sleep (about 1 s on B200), then the device error word
            uint32_t n = 0;
            while (before(ld_acquire_sys(flags + r), target)) {
                if (++n >= (1u << 22)) {
                    ok = false;
                    break;
                }
                __nanosleep(100);
            }
        }
        if (!ok && a.err) atomicMax(a.err, CST_DEV_ERR_TIMEOUT);
        s_ok = ok;
    }
    __syncthreads();
    __threadfence();
    const float* recv = a.peers.recv[a.peers.rank];
    const int32_t* pres =
        a.peers.pres_off ? reinterpret_cast<const int32_t*>(reinterpret_cast<const uint8_t*>(recv) + a.peers.pres_off)
                         : nullptr;
    for (int h = (blockIdx.y * blockDim.x + threadIdx.x) * 4; h < a.H; h += gridDim.y * blockDim.x * 4) {
        float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
        if (s_ok) {
            for (int r = 0; r < a.peers.world; ++r) {  // rank order
                if (pres != nullptr && pres[int64_t(r) * a.peers.tl_cap + t] == 0) continue;  // nothing pushed
                const float4 v =
                    *reinterpret_cast<const float4*>(recv + (int64_t(r) * a.peers.tl_cap + t) * a.H + h);
                acc.x += v.x;
                acc.y += v.y;
                acc.z += v.z;
                acc.w += v.w;
            }
        }
        if (a.residual) {
            const float4 v = load4_any(a.residual, a.residual_dtype, int64_t(t) * a.H + h);
            acc.x += v.x;
            acc.y += v.y;
            acc.z += v.z;
            acc.w += v.w;
        }
        store_out<OUT>(a.out, int64_t(t) * a.H + h, acc);
    }
}

}  // namespace

int push_chunks(int H) { return (H + 1023) / 1024; }

cudaError_t launch_combine_push(const PushArgs& a, cudaStream_t stream) {
    if (a.T == 0) return cudaSuccess;
    const dim3 grid(a.peers.world * ((a.tl + kPushTok - 1) / kPushTok), push_chunks(a.H));
    combine_push_kernel<<<grid, 256, 0, stream>>>(a);
    return cudaGetLastError();
}

cudaError_t launch_gather_rows(const GatherArgs& a, cudaStream_t stream) {
    if (a.tl == 0) return cudaSuccess;
    const int nblk = (a.tl + kGatherRows - 1) / kGatherRows;
    gather_push_kernel<<<a.peers.world * nblk, 256, 0, stream>>>(a);
    gather_wait_kernel<<<1, 32, 0, stream>>>(a);
    return cudaGetLastError();
}

cudaError_t launch_reduce_cast(const ReduceArgs& a, cudaStream_t stream) {
    if (a.tl == 0) return cudaSuccess;
    const dim3 grid(a.tl, push_chunks(a.H));
    if (a.out_dtype == 3) {
        reduce_cast_kernel<3><<<grid, 256, 0, stream>>>(a);
    } else if (a.out_dtype == 2) {
        reduce_cast_kernel<2><<<grid, 256, 0, stream>>>(a);
    } else {
        reduce_cast_kernel<1><<<grid, 256, 0, stream>>>(a);
    }
    return cudaGetLastError();
}

}  // namespace cst
