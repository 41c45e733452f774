// Launch interfaces of the hot-path kernels (host side of the .cu files in this folder).
#pragma once

#include <cstddef>
#include <cstdint>
#include <cuda_runtime.h>

#include "layout.cuh"

namespace cst {

// Launch of a kernel of the layer chain with programmatic stream serialization: the kernel
// may start its prologue while the previous kernel on `stream` finishes; it waits for it
// (chain_wait in cst_common.cuh) before touching global memory.
template <typename... KArgs, typename... Args>
cudaError_t launch_chained(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
                           Args... args) {
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kernel, static_cast<KArgs>(args)...);
}

// capi.cu: the thread's cst_last_error() message, for entry points in other files
void clear_last_error();
int set_last_error(int code, const char* fmt, ...);

// infer_codec.cu: the fixed 20 bytes of an InferResponse body (status, batch, hidden,
// output dtype, output byte count), little-endian
constexpr int kInferRequestFixedBytes = 24;
constexpr int kInferResponseFixedBytes = 20;
void put_infer_response_fixed(uint8_t* body, int32_t status, int32_t batch, int32_t hidden, uint32_t out_dtype,
                              uint32_t nbytes);

// relayout.cu
cudaError_t launch_relayout(const uint8_t* wu, const uint8_t* wg, const uint8_t* wd, uint8_t* slot,
                            int inter, int hidden, int num_sms, cudaStream_t stream);

// dequant.cu
cudaError_t launch_dequant_fp8(const uint8_t* w, const float* s, float* out, int rows, int cols, int block,
                               int num_sms, cudaStream_t stream);

// router.cu
// `logits` holds `cap` floats: scratch for the partial logits of a K split, or the caller's
// [T, E] logits when cap == T * E (no split).  err: device error word (the tensor-core
// logits kernel's bounded waits report there); with allow_tc false the logits always run
// on the CUDA cores, whose kernel has no waits, and err may be null.  logits_out: [T, E]
// copy of the summed logits the selection used (or null), so a caller that asks for them
// gets exactly the routing of a call that does not.
int router_tc_split(int T, int E, int H, int64_t cap);
int64_t router_scratch_floats(int x_dtype, int T, int E, int H);  // scratch a call of T tokens may use
cudaError_t launch_router(const void* x, int x_dtype, const float* w, const float* bias, const uint8_t* resident,
                          int T, int E, int H, int n_group, int topk_group, int top_k, int norm, float scale,
                          float* logits, int64_t cap, int32_t* topk_idx, float* topk_w, float* group_scores_out,
                          int* err, cudaStream_t stream, bool allow_tc = true, float* logits_out = nullptr);

// route_pack.cu
// A slot-table entry with this bit set is an expert served only for the tokens of the call's
// own-token range (shared_t_begin..shared_t_end): a replica of a hot expert that every rank
// holds and applies to its own tokens alone.
constexpr int32_t kSlotOwnTokensOnly = int32_t(1) << 30;
struct PackArgs {
    // mode A (routes): topk_idx/topk_w [T, K]; slot_of_expert [E]
    const int32_t* topk_idx;
    const float* topk_w;
    const int32_t* slot_of_expert;
    int E;
    int K;
    int shared_slot;  // -1: none
    int shared_t_begin, shared_t_end;  // tokens [begin, end) get a shared-expert row
    // mode B (rows): row_slot [T] (one route per row, weight row_weight or 1), or every
    // row to `single_slot` when row_slot is null and single_slot >= 0
    const int32_t* row_slot;
    int single_slot;
    const float* row_weight_in;
    int T;
    int n_slots;
    int max_rows;
    int max_groups;
    // outputs
    GroupRec* groups;
    int32_t* tile_group;  // [max_rows] group of each n-tile
    int32_t* row_token;   // [max_rows]
    float* row_weight;    // [max_rows]
    int32_t* tk_row;      // [T, K + 1] (mode A) or [T] (mode B); -1 = not here
    PackMeta* meta;
    int group_rows;   // rows per group: 16 (decode kernels) or 64 (prefill kernels)
    int* hist;        // counting-sort scratch for calls of more than 2048 routes
    int64_t hist_cap; // ints available at hist (>= ceil(routes / 1024) * n_slots)
};
constexpr int kRoutePackMaxRows = 1 << 18;  // packed rows per call
cudaError_t route_pack_init_attributes();
cudaError_t launch_route_pack(const PackArgs& a, cudaStream_t stream);

// pack_act.cu
struct PackActArgs {
    const void* src;         // [rows_src, K] activations
    int src_dtype;           // 1 fp16, 2 bf16, 3 fp32
    int64_t ld;              // row stride of src in elements
    const int32_t* row_map;  // packed row -> source row (x pack); null: identity (h pack)
    const GroupRec* groups;
    const int32_t* tile_group;
    const PackMeta* meta;
    int K;                   // H (x) or I (h)
    uint8_t* bfrag;          // B fragments
    float* bscale;           // per (row, K block) scales
    int terms;               // E4M3 terms per element: 3 (decode kernels) or 2 (prefill kernels)
    const float* src_scale = nullptr;  // prefill: per source row scale (row_scale_kernel), or null
    // prefill x, token-major (with src_scale): tk_row [n_src, K1] -> packed row of each of a
    // source row's routes, -1 where absent; the packer then reads each source row once
    const int32_t* tk_row = nullptr;
    int K1 = 0;
    int n_src = 0;
    // an upper bound on the packed rows known on the host (0: none); a small call then
    // launches only the CTAs its tasks can use
    int rows_hint = 0;
};
// src_dtype 4: `src` holds the up/gate kernel's split accumulators (meta->split_k splits of
// meta->n_rows rows each); the packer adds the splits in order and applies
// h = silu(gate) * up before quantizing.
constexpr int kSrcUpGatePartials = 4;
constexpr int kMaxUpGateSplit = 4;  // largest K split of the up/gate launch
cudaError_t launch_pack_act(const PackActArgs& a, int num_sms, cudaStream_t stream);
// Prefill packing: two E4M3 terms and ONE power-of-two scale per packed row (written to
// bscale[row]), so the prefill kernel promotes each K block with the weight scale alone and
// applies the row scale once per output.  terms must be 2.
cudaError_t launch_pack_rows(const PackActArgs& a, int num_sms, cudaStream_t stream);
// out[r] = the scale pack_rows_kernel would compute for source row r (r < n_src_rows)
cudaError_t launch_row_scale(const PackActArgs& a, int n_src_rows, float* out, int num_sms, cudaStream_t stream);

// grouped_ffn.cu
struct FfnArgs {
    const uint8_t* arena;
    int64_t slot_bytes;
    int64_t a_off;   // byte offset of this projection's tiles inside a slot
    int64_t s0_off;  // scale grid (up or down)
    int64_t s1_off;  // scale grid (gate), up/gate only
    int KB;          // K / 128
    int n_mb;        // output rows / 128
    int scale_ld;    // columns of the scale grid (= KB)
    const GroupRec* groups;
    PackMeta* meta;           // read: n_groups; written (block 0): the K split chosen
    const uint8_t* bfrag;
    const float* bscale;
    // up/gate: raw fp32 accumulators out[((split * n_rows + row) * 2 + mat) * ld_out + col],
    //          n_rows = meta->n_rows
    // down:    out[row * ld_out + col] = accumulator * row_weight[row]
    float* out;
    int64_t ld_out;
    int out_rows;             // up/gate: rows `out` holds (split * n_rows * 2 <= out_rows * 2)
    int max_split;            // largest K split this launch may choose (1 = never split)
    const float* row_weight;  // down only
    int* err;
    // down: an upper bound on the groups of this launch known on the host (one expert's
    // request: ceil(rows / group rows)), or 0 when the routing decides it on the device.
    // Below one row-block pair per SM the launch takes single row blocks per item, which
    // doubles the items a lone expert spreads over.
    int groups_hint;
};
cudaError_t grouped_ffn_init_attributes();
cudaError_t launch_grouped_ffn(const FfnArgs& a, bool upgate, int num_sms, cudaStream_t stream);

// grouped_prefill.cu: the same contract for groups of up to 128 rows and 2-term activations
cudaError_t grouped_prefill_init_attributes();
cudaError_t launch_grouped_prefill(const FfnArgs& a, bool upgate, int num_sms, cudaStream_t stream);

// norm.cu: out = x * rsqrt(mean(x^2) + eps) * weight (weight may be null), per row of H
// (H a multiple of 8, 16-byte aligned rows)
cudaError_t launch_rmsnorm(const void* x, int x_dtype, int T, int H, const float* weight, float eps, void* out,
                           int out_dtype, cudaStream_t stream);

// p2p.cu: the combine fused with the cross-rank reduction over peer memory
constexpr int kMaxPeers = 8;
struct PeerSet {
    int world, rank;
    int tl;       // tokens each rank owns
    int tl_cap;   // token capacity of one receive slot
    float* recv[kMaxPeers];      // rank q's receive buffer [world][tl_cap][H] (mapped here)
    int32_t* flags[kMaxPeers];   // rank q's arrival counters [world]
    int32_t* epoch;              // this rank's exchange counter
    int32_t* done;               // reserved
    int64_t x_off;               // byte offset of the gathered-row slots from recv[q] (0: none)
    int32_t* gather_epoch;       // this rank's gather counter
    int64_t pres_off;            // byte offset of the presence words [world][tl_cap] from recv[q]
                                 // (0: none -- every partial is pushed and added)
};
// Gathered-row exchange: arrival counters at flags[q] + kGatherFlags
constexpr int kGatherFlags = 8;
constexpr int kGatherRows = 4;  // rows per pushing CTA
struct GatherArgs {
    PeerSet peers;
    const void* x;   // this rank's [tl, H] rows, 2-byte elements
    int tl;
    int H;
    int* err;
};
cudaError_t launch_gather_rows(const GatherArgs& a, cudaStream_t stream);
struct PushArgs {
    const float* y;         // weighted expert output rows
    int64_t ldy;
    const int32_t* tk_row;  // [T, K1]; -1 = absent
    int K1;
    int T;                  // gathered tokens = world * tl
    int H;
    int tl;
    PeerSet peers;
};
struct ReduceArgs {
    PeerSet peers;
    int tl;
    int H;
    int chunks;             // column chunks per pushed token block (push_chunks(H))
    const void* residual;   // [tl, H] or null
    int residual_dtype;
    void* out;              // [tl, H]
    int out_dtype;
    int* err;
};
int push_chunks(int H);
constexpr int kPushTok = 4;  // owner tokens per pushing CTA
cudaError_t launch_combine_push(const PushArgs& a, cudaStream_t stream);
cudaError_t launch_reduce_cast(const ReduceArgs& a, cudaStream_t stream);

// combine.cu
struct CombineArgs {
    const float* y;         // [rows, H] fp32 weighted expert outputs
    int64_t ldy;
    const int32_t* tk_row;  // [T, K1]; -1 = contribution absent on this device
    int K1;
    int T;
    int H;
    const void* residual;   // [T, H] in residual_dtype, or null
    int residual_dtype;
    void* out;              // [T, H]
    int out_dtype;          // 1 fp16, 2 bf16, 3 fp32
    const float* extra;     // [T, H] fp32 added before the cast (remote contributions), or null
};
cudaError_t launch_combine(const CombineArgs& a, cudaStream_t stream);

}  // namespace cst
