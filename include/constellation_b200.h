/*
 * constellation_b200 -- C ABI of the B200 (sm_100a) MoE-layer hot path.
 *
 * Plain pointers, sizes and status codes; no C++ or torch types cross this boundary.
 * Every device pointer argument is caller-owned, except the expert arena the context
 * allocates and fills through cst_upload_expert.  All work is enqueued on the `stream`
 * argument (a cudaStream_t passed as void*; NULL = legacy default stream); nothing
 * synchronises the device except cst_device_error, cst_serve_infer_request (it returns the
 * output bytes) and cst_destroy.
 *
 * Empty batches: a token or row count of 0 is a no-op that returns CST_OK once the scalar
 * arguments are valid, whatever the data pointers (a zero-size device buffer may be NULL).
 * The exceptions keep the reference's rules: cst_expert_forward answers batch 0 with
 * CST_ERR_BACKEND like the worker, and a peer exchange needs tl >= 1.
 *
 * Threading: one context per device; calls on one context must be serialised by the
 * caller, like the reference node's one worker thread per GPU
 * (expert_node_v2/main.cc:132-149) and its registry lock (worker.cc:120, control.cc:172).
 *
 * Status codes (int): 0 ok; 1 unknown expert; 2 expert not resident on this device;
 * 4 backend failure -- these three mirror the worker reply statuses
 * (expert_node_v2/worker.cc:112-131) -- plus 3 invalid argument, 5 CUDA error,
 * 6 NCCL / peer error, 7 a device-side wait hit its iteration limit.
 * cst_last_error() returns the message of the last failure on the calling thread.
 */
#ifndef CONSTELLATION_B200_H_
#define CONSTELLATION_B200_H_

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define CST_OK 0
#define CST_ERR_UNKNOWN_EXPERT 1
#define CST_ERR_NOT_RESIDENT 2
#define CST_ERR_INVALID_ARG 3
#define CST_ERR_BACKEND 4
#define CST_ERR_CUDA 5
#define CST_ERR_PEER 6
#define CST_ERR_DEVICE_TIMEOUT 7

/* Activation dtypes; 1 and 2 are the values of common::ActivationDType
 * (common/protocol.h:48-52). */
#define CST_DTYPE_FP16 1
#define CST_DTYPE_BF16 2
#define CST_DTYPE_FP32 3

/* cst_moe_layer / cst_moe_routed flags */
#define CST_FLAG_ADD_SHARED 1u

typedef struct cst_ctx cst_ctx;

/* Layer geometry and router hyper-parameters.  Mirrors the router config that
 * run_moe_layer reads (server/moe_layer_runtime.py:428-522: n_group, topk_group, top_k,
 * norm_topk_prob, routed_scaling_factor, n_routed_experts, hidden_size) plus the expert
 * shape of ExpertWorkspaceConfigV2 (expert_node_v2/expert_format_v2.h:31-34).
 * hidden_dim and inter_dim must be multiples of 128; block_size must be 128. */
typedef struct cst_config {
    int32_t hidden_dim;
    int32_t inter_dim;
    int32_t n_routed_experts; /* router width E (<= 1024) */
    int32_t n_group;          /* <= 32, divides E */
    int32_t topk_group;
    int32_t top_k;            /* <= 15 */
    int32_t norm_topk_prob;
    float routed_scaling_factor;
    int32_t block_size;
    int32_t n_slots;          /* expert slots in this device's arena (routed + shared) */
    int32_t max_tokens;       /* largest T of one layer call */
    int32_t max_rows;         /* largest number of (token, expert) rows per call; 0 = max_tokens*(top_k+1) */
} cst_config;

/* One expert in the reference upload format (ExpertTensorBundleV2,
 * expert_node_v2/expert_format_v2.h:59-86): float8_e4m3fn weights, row-major, and fp32
 * scale_inv grids [ceil(rows/row_block), ceil(cols/col_block)], row-major.  Pointers may
 * be host or device memory. */
typedef struct cst_expert_weights {
    const uint8_t* w_up;         /* [rows=inter, cols=hidden] */
    const float* w_up_scale;
    const uint8_t* w_gate;       /* [inter, hidden] */
    const float* w_gate_scale;
    const uint8_t* w_down;       /* [hidden, inter] */
    const float* w_down_scale;
    int32_t rows;                /* inter */
    int32_t cols;                /* hidden */
    int32_t row_block;
    int32_t col_block;
} cst_expert_weights;

/* Creates a context on `device`: validates the config, allocates the expert arena
 * (n_slots experts in the kernels' fragment-major layout) and the per-call workspace
 * sized for max_rows.  Replaces CreateBackendWorkspaceV2 / InitExpertWorkspaceCudaV2
 * (backend/backend_workspace_v2.cc:30-89, backend/cuda/backend_cuda_v2.cc:166-197). */
int cst_create(int32_t device, const cst_config* cfg, cst_ctx** out);
void cst_destroy(cst_ctx* ctx);

/* Uploads one expert into arena slot `slot` and makes router expert `expert_id`
 * (0 <= expert_id < n_routed_experts) resident there; expert_id = -1 uploads the shared
 * expert (see cst_set_shared_slot).  Validates dtype-free shape / block / size rules of
 * BuildExpertWeightsViewV2 (expert_format_v2.cc:68-175).  Replaces the backend registry's
 * upload_expert hook UploadExpertCudaV2 (backend/cuda/backend_cuda_v2.cc:94-145,
 * backend/backend_registry_v2.h:20-23).  Stream-ordered; the source may be reused once
 * the stream has passed this call. */
int cst_upload_expert(cst_ctx* ctx, int32_t slot, int32_t expert_id, const cst_expert_weights* w,
                      void* stream);

/* Makes `slot` non-resident (the free_expert_weights hook, FreeExpertWeightsCudaV2,
 * backend/cuda/backend_cuda_v2.cc:147-164).  The arena memory is kept for reuse. */
int cst_free_expert(cst_ctx* ctx, int32_t slot);

/* Slot holding router expert `expert_id`, or -1 (ExpertRegistryV2::FindDeviceStorage,
 * expert_node_v2/expert_registry_v2.cc:437). */
int32_t cst_find_slot(const cst_ctx* ctx, int32_t expert_id);

/* Marks resident router expert `expert_id` as served for this rank's own tokens only (1) or
 * for every token routed to it (0, the default).  Expert parallelism gives each expert one
 * owner rank, which serves it for all gathered tokens; a hot expert replicated on every rank
 * and marked here is instead applied by each rank to the tokens it owns (the shared expert's
 * token range of cst_moe_routed_range / cst_moe_routed_push; every token in cst_moe_layer),
 * which spreads its rows over the ranks.  No counterpart in the reference (its coordinator
 * places one replica per expert, server/expert_placement.py).  Load-time call: it
 * synchronises the device. */
int cst_set_expert_own_tokens_only(cst_ctx* ctx, int32_t expert_id, int32_t own_tokens_only);

/* Marks `slot` as the shared expert (-1: none). */
int cst_set_shared_slot(cst_ctx* ctx, int32_t slot);

/* Kernel shape of the grouped expert products (the reference runs one batch-1 matvec per
 * (token, expert), backend/cuda/backend_cuda_v2.cc:205-255; it has no such choice).
 * CST_GEMM_AUTO (default) takes the prefill kernels once a call averages >= 32 rows per
 * expert: groups of up to 128 rows, activations in two E4M3 terms (row-wise relative error
 * ~1e-3) instead of three (~2e-5).  The other two values force one shape. */
#define CST_GEMM_AUTO 0
#define CST_GEMM_DECODE 1
#define CST_GEMM_PREFILL 2
int cst_set_gemm_mode(cst_ctx* ctx, int32_t mode);

/* Routing for T tokens (route_token_real, server/moe_layer_runtime.py:232-408, batched):
 *   x            [T, hidden] in x_dtype (device)
 *   gate_weight  [n_routed_experts, hidden] fp32 (device)
 *   bias         [n_routed_experts] fp32 e_score_correction_bias (device)
 *   resident     [n_routed_experts] uint8 mask or NULL (all resident)
 *   top_k        experts per token (<= cfg.top_k; callers pass min(top_k, #resident))
 *   topk_idx     [T, top_k] int32 out, sorted by (biased score desc, index asc)
 *   topk_weight  [T, top_k] fp32 out
 *   logits, group_scores: optional fp32 outputs [T, E] and [T, n_group] (aux), or NULL. */
int cst_route(cst_ctx* ctx, const void* x, int32_t x_dtype, int32_t T, const float* gate_weight,
              const float* bias, const uint8_t* resident, int32_t top_k, int32_t* topk_idx,
              float* topk_weight, float* logits, float* group_scores, void* stream);

/* cst_route without a context and without any allocation.  It has no counterpart in the
 * reference; it exists for callers that cannot call cudaMalloc -- a host runtime that has
 * already handed the device memory to its own pool, code running while another component
 * owns the allocator, or a process that must not grow after start-up -- and therefore
 * cannot create a context.  The caller passes every input and output (device pointers,
 * same meaning as cst_route plus the router hyper-parameters); the router's scratch (the
 * [T, n_experts] fp32 logits) lives in a 2 MiB static device array inside this library,
 * which every GPU that loads the library holds until the process exits.  Limit:
 * T * n_experts <= 524288 floats -- T <= 2048 at 256 experts; larger calls return
 * CST_ERR_INVALID_ARG with a message naming the limit.
 * The first call in each CUDA context (the device's primary context, or a driver context
 * the caller made current) looks the array's device address up (cudaGetSymbolAddress with
 * that context current) and caches it under the context's unique id, so make that first
 * call before any stream capture.  All calls share the one array: calls that overlap on
 * the GPU (other streams, threads or graph replays) race on it.  The logits always run on
 * the CUDA cores (a kernel with no device-side waits, so no call can time out unreported);
 * results equal cst_route's wherever cst_route does the same (below 192 bf16 tokens, or
 * fp16 / fp32 input); from 192 bf16 tokens on cst_route sums the logits on the tensor
 * cores in another order, so a logit may differ in its last bits and an expert choice
 * only on a near-tie. */
int cst_route_noalloc(const void* x, int32_t x_dtype, int32_t T, int32_t hidden, const float* gate_weight,
                      const float* bias, const uint8_t* resident, int32_t n_experts, int32_t n_group,
                      int32_t topk_group, int32_t top_k, int32_t norm_topk_prob, float routed_scaling_factor,
                      int32_t* topk_idx, float* topk_weight, void* stream);

/* Routed experts for given routes + fp32 combine (+ shared expert when flags has
 * CST_FLAG_ADD_SHARED): run_topk_moe_layer / dispatch_topk_experts / combine_outputs_torch
 * (server/moe_layer_runtime.py:111-229) for a batch.  Routes to experts that are not
 * resident here contribute nothing.  out: [T, hidden] in out_dtype. */
int cst_moe_routed(cst_ctx* ctx, const void* x, int32_t x_dtype, int32_t T, const int32_t* topk_idx,
                   const float* topk_weight, int32_t top_k, uint32_t flags, void* out, int32_t out_dtype,
                   void* stream);

/* cst_moe_routed with the shared expert applied only to tokens [shared_begin, shared_end):
 * the expert-parallel form, where every rank runs its own experts on all gathered tokens
 * but the shared expert only on the tokens it owns, inside the same grouped launches
 * (run_shared_expert_block, server/deepseek_full_model_executor.py:264-316, per rank). */
int cst_moe_routed_range(cst_ctx* ctx, const void* x, int32_t x_dtype, int32_t T, const int32_t* topk_idx,
                         const float* topk_weight, int32_t top_k, int32_t shared_begin, int32_t shared_end,
                         void* out, int32_t out_dtype, void* stream);

/* Whole layer: route -> dispatch -> grouped FP8 SwiGLU -> combine (+ shared).
 * run_moe_layer (server/moe_layer_runtime.py:411-578) batched over T tokens, plus the
 * shared-expert sum of run_sparse_layer (server/full_model_runtime.py:283-348).
 * topk_idx / topk_weight receive the routes when non-NULL.  residual (same dtype as
 * x, or NULL) is added before the final cast (full_model_runtime.py:355). */
int cst_moe_layer(cst_ctx* ctx, const void* x, int32_t x_dtype, int32_t T, const float* gate_weight,
                  const float* bias, const uint8_t* resident, int32_t top_k, uint32_t flags,
                  const void* residual, void* out, int32_t out_dtype, int32_t* topk_idx,
                  float* topk_weight, void* stream);

/* Grouped expert FFN over rows that are already assigned to slots (the expert node's
 * batched request path): y[r] = row_weight[r] * Expert_{row_slot[r]}(x[r]).
 *   x          [R, hidden] in x_dtype; row_slot [R] int32 slot ids; row_weight [R] or NULL (1.0)
 *   y          [R, hidden] in y_dtype (fp32 keeps the unrounded expert output) */
int cst_grouped_ffn(cst_ctx* ctx, const void* x, int32_t x_dtype, int32_t R, const int32_t* row_slot,
                    const float* row_weight, void* y, int32_t y_dtype, void* stream);

/* One expert, `batch` rows: the BackendWorkspaceV2::RunExpertRequest replacement
 * (backend/backend_workspace_v2.h:18-21; backend/cuda/backend_workspace_cuda_v2.cc:139-181)
 * without its batch_size == 1 restriction.  in_dtype / out_dtype: CST_DTYPE_FP16 or BF16
 * (any pair, as the reference dispatches).  Returns 1 for an expert id outside the router
 * range and 2 when the expert is not resident on this device, like the worker. */
int cst_expert_forward(cst_ctx* ctx, int32_t expert_id, const void* x, int32_t in_dtype, int32_t batch,
                       void* y, int32_t out_dtype, void* stream);

/* out[t] = SharedExpert(x[t]) + extra[t] (+ residual[t]), one final cast, for T rows.
 * The last step of an expert-parallel layer: `extra` ([T, hidden] fp32, or NULL) is the
 * routed sum that came back from the other ranks; the shared expert is applied to the
 * rank's own tokens (run_shared_expert_block, server/deepseek_full_model_executor.py:264-316,
 * and the sums of server/full_model_runtime.py:348-355).  Without a resident shared
 * expert only extra + residual is written. */
int cst_shared_combine(cst_ctx* ctx, const void* x, int32_t x_dtype, int32_t T, const float* extra,
                       const void* residual, void* out, int32_t out_dtype, void* stream);

/* out[t] = sum_{k < k1, tk_row[t,k] >= 0} rows[tk_row[t,k]] (+ extra[t]) (+ residual[t]), fp32
 * sums in k order, one final cast: the source-side combine of an all-to-all return
 * (combine_outputs_torch, server/moe_layer_runtime.py:148-167, over rows that already
 * carry their routing weight).  rows: [*, hidden] fp32 with row stride ld_rows. */
int cst_combine_rows(cst_ctx* ctx, const float* rows, int64_t ld_rows, const int32_t* tk_row, int32_t k1,
                     int32_t T, const float* extra, const void* residual, int32_t residual_dtype, void* out,
                     int32_t out_dtype, void* stream);

/* out[r, c] = float8_e4m3fn(w[r, c]) * scale_inv[r / block, c / block] on the current device:
 * dequant_fp8_weight_blockwise (server/fp8_utils.py:4-39), bit-identical (true e4m3fn
 * decode, 0x7F/0xFF -> NaN; ceil-div block grid for ragged shapes; one fp32 multiply).
 * w [rows, cols] uint8, scale_inv [ceil(rows/block), ceil(cols/block)] fp32, out fp32. */
int cst_dequant_fp8(const uint8_t* w, const float* scale_inv, int32_t rows, int32_t cols, int32_t block,
                    float* out, void* stream);

/* out[t, :] = x[t, :] * rsqrt(mean(x[t, :]^2) + eps) * weight on the current device: the
 * prenorm before the sparse FFN, torch.nn.functional.rms_norm(h, (H,), weight, 1e-6)
 * (server/full_model_runtime.py:271-276), fp32 math and one final RNE cast.  x, out
 * [T, H] in x_dtype / out_dtype (16-byte aligned, H a multiple of 8); weight [H] fp32 or
 * NULL (all ones).  x == out is allowed. */
int cst_rmsnorm(const void* x, int32_t x_dtype, int32_t T, int32_t H, const float* weight, float eps, void* out,
                int32_t out_dtype, void* stream);

/* ---- Peer-memory exchange (expert parallelism, one process per GPU, NVLink) -----------
 * No counterpart in the reference: its coordinator collects one expert result per
 * (token, expert) socket request and sums them on the host (server/moe_layer_runtime.py
 * :111-229).  Here the per-rank combine stores every token's partial sum straight into the
 * owning rank's memory, which then adds the ranks' partials in order -- the NCCL
 * reduce-scatter of the all-gather exchange, fused into the combine. */
typedef struct {
    uint8_t bytes[64];  /* a cudaIpcMemHandle_t */
} cst_ipc_handle;

/* Zeroed device memory on the current device that other processes can map; *ptr and
 * *handle receive the local address and its IPC handle.  Free with cst_ipc_free. */
int cst_ipc_alloc(int64_t bytes, void** ptr, cst_ipc_handle* handle);
/* Maps another process's cst_ipc_alloc allocation (same node, peer access) at *ptr. */
int cst_ipc_open(const cst_ipc_handle* handle, void** ptr);
int cst_ipc_close(void* ptr);
int cst_ipc_free(void* ptr);

#define CST_MAX_PEERS 8
/* One rank's view of the exchange buffers.  Each rank allocates one buffer of
 * world * tl_cap * hidden floats (its receive slots, slot r for rank r) followed by 64
 * int32 (arrival counters at [0, world), epoch at [32], [33] reserved), zeroed; recv[q] and
 * flags[q] are rank q's buffer and counters as mapped in this process (q == rank: local).
 * Counters and epoch wrap modulo 2^32; only their differences are compared. */
typedef struct {
    int32_t world, rank;
    int32_t tl;      /* tokens each rank owns: the gathered batch is world * tl tokens */
    int32_t tl_cap;  /* token capacity of one receive slot */
    float* recv[CST_MAX_PEERS];
    int32_t* flags[CST_MAX_PEERS];
    int32_t* epoch;  /* this rank's exchange counter */
    int32_t* done;   /* reserved (a zeroed int32 of this rank) */
    int64_t x_offset;       /* byte offset from recv[q] of rank q's gathered-row slots
                             * [world * tl_cap, hidden] 2-byte rows; 0: none (cst_gather_rows) */
    int32_t* gather_epoch;  /* this rank's gather counter (zeroed int32); gather arrival counters
                             * are flags[q][8 + r] */
    int64_t presence_offset; /* byte offset from recv[q] of rank q's presence words
                              * [world][tl_cap] int32 (16-byte aligned), or 0: with it, a rank
                              * that has no row for a token pushes no partial for it, only a 0
                              * presence word, and the owner skips that rank's slot */
} cst_peer_set;

/* The all-gather of the expert-parallel exchange over peer memory: this rank's tl rows of x
 * ([tl, hidden], fp16 or bf16) are stored into every rank's gathered-row slots (rows
 * rank * tl ..), each block of rows followed by a release-ordered add on that rank's gather
 * counter for this rank; then the stream waits (bounded, about 1 s; the device error word on
 * timeout) until every rank's rows of this exchange have arrived here.  Afterwards this
 * rank's slots hold all world * tl rows, rank-major: the x of cst_moe_routed_push. */
int cst_gather_rows(cst_ctx* ctx, const cst_peer_set* peers, const void* x, int32_t x_dtype, void* stream);

/* The routed experts resident here on all world * tl gathered tokens, the shared expert on
 * this rank's own tokens, and the combine pushed to the owners: token t's partial sum
 * (this device's routes in k order, then the shared row) is stored into rank
 * (t / tl)'s receive slot [this rank], each column chunk followed by a release-ordered
 * add on that rank's arrival counter for this rank.  Follow with cst_reduce_pushed. */
int cst_moe_routed_push(cst_ctx* ctx, const void* x, int32_t x_dtype, const int32_t* topk_idx,
                        const float* topk_weight, int32_t top_k, const cst_peer_set* peers, void* stream);
/* out[t] = sum over ranks r = 0 .. world-1 of rank r's pushed partial for this rank's token
 * t (+ residual[t]), one cast.  Waits (bounded, about 1 s) until every rank's
 * counter shows all chunks of this exchange; a wait that gives up sets the device error
 * word (cst_device_error) and leaves only the residual in out. */
int cst_reduce_pushed(cst_ctx* ctx, const cst_peer_set* peers, const void* residual, int32_t residual_dtype,
                      void* out, int32_t out_dtype, void* stream);

/* ---- Expert-node requests ------------------------------------------------------------
 * The worker's InferRequest / InferResponse bodies (common/infer_codec.cc:7-76 over the
 * little-endian helpers of common/protocol.cc:13-80; common/protocol.py:503-577 on the
 * coordinator side), and the handling of one request (expert_node_v2/worker.cc:83-140 with
 * backend/cuda/backend_workspace_cuda_v2.cc:19-181), minus the socket and the 16-byte
 * message header.  The four codec calls are host-only and touch no device. */
#define CST_INFER_REQUEST_FIXED_BYTES 24  /* i32 expert_id, batch_size, hidden_dim; u32 input_dtype, output_dtype, n */
#define CST_INFER_RESPONSE_FIXED_BYTES 20 /* i32 status_code, batch_size, hidden_dim; u32 output_dtype, n */
typedef struct {
    int32_t expert_id;  /* global id: layer * experts_per_layer + local id (expert_placement.py:4-24) */
    int32_t batch_size;
    int32_t hidden_dim;
    uint32_t input_dtype; /* CST_DTYPE_FP16 / CST_DTYPE_BF16 (0 = unknown) */
    uint32_t output_dtype;
    uint32_t activation_bytes;
    const uint8_t* activation; /* decode: points into the decoded body */
} cst_infer_request;
typedef struct {
    int32_t status_code; /* 0 ok, 1 unknown expert, 2 not on this device, 4 backend failure */
    int32_t batch_size;
    int32_t hidden_dim;
    uint32_t output_dtype;
    uint32_t output_bytes;
    const uint8_t* output; /* decode: points into the decoded body */
} cst_infer_response;
/* EncodeInferRequestBody / EncodeInferResponseBody: *len = bytes the body takes (set even
 * when it fails); CST_ERR_INVALID_ARG if body is NULL or cap is short. */
int cst_encode_infer_request(const cst_infer_request* msg, uint8_t* body, int64_t cap, int64_t* len);
int cst_encode_infer_response(const cst_infer_response* msg, uint8_t* body, int64_t cap, int64_t* len);
/* DecodeInferRequestBody / DecodeInferResponseBody: CST_OK, or CST_ERR_INVALID_ARG for a
 * body that ends inside a field or the payload, or has trailing bytes. */
int cst_decode_infer_request(const uint8_t* body, int64_t len, cst_infer_request* out);
int cst_decode_infer_response(const uint8_t* body, int64_t len, cst_infer_response* out);
/* One request body in, one response body out, with the worker's rules: the response
 * echoes batch_size, hidden_dim and output_dtype; status 1 if no context holds the
 * expert's layer (layers[expert_id / experts_per_layer], NULL entries allowed), 2 if the
 * layer's context does not hold the expert, 4 if the request is unusable (batch outside
 * [1, the context's max rows] -- the reference takes batch 1 only --, hidden_dim not the
 * context's, a dtype outside fp16/bf16, activation bytes != batch * hidden * 2) or the
 * device run failed (cst_last_error() has the cause); 0 with batch * hidden * 2 output
 * bytes otherwise.  Returns CST_OK when *resp_len bytes of response were written;
 * CST_ERR_INVALID_ARG when the request does not decode (the worker sends no reply) or
 * resp_cap is short (*resp_len = the size needed, nothing run).  The activation is copied
 * to the device on `stream`, the expert runs there, the output is copied back into
 * resp_body and the stream is synchronised before the call returns. */
int cst_serve_infer_request(cst_ctx* const* layers, int32_t n_layers, int32_t experts_per_layer,
                            const uint8_t* req_body, int64_t req_len, uint8_t* resp_body, int64_t resp_cap,
                            int64_t* resp_len, void* stream);

/* Synchronises the context's device, then returns CST_OK or CST_ERR_DEVICE_TIMEOUT if a
 * kernel's bounded wait gave up since the last call (and clears the flag). */
int cst_device_error(cst_ctx* ctx);

/* Per-stage device timing (the reference has only ad hoc host timers, server/client.py:130-176,
 * and cudaEvent means in its benchmark harness, test_benchmark_run_expert_cuda_v2.cc:310-368).
 * When enabled, every layer-level call records CUDA events at its stage boundaries:
 *   0 router, 1 route_pack, 2 pack x, 3 grouped up/gate, 4 pack h, 5 grouped down, 6 combine.
 * cst_profile_read waits for the recorded calls, writes max_calls x CST_N_STAGES
 * milliseconds (row-major) and returns the number of calls written (negative status on error). */
#define CST_N_STAGES 7
int cst_profile_enable(cst_ctx* ctx, int32_t enable);
int cst_profile_read(cst_ctx* ctx, float* stage_ms, int32_t max_calls);

/* Context facts: out[0] arena bytes, [1] bytes per slot, [2] workspace bytes,
 * [3] number of SMs, [4] resident routed experts, [5] shared slot, [6] device address of
 * the arena (slot s starts at [6] + s * [1]). Returns #values written. */
int cst_ctx_info(const cst_ctx* ctx, int64_t* out, int32_t n);

/* Message of the last failing call on this thread ("" if none). */
const char* cst_last_error(void);

/* ABI version (major * 100 + minor). */
int32_t cst_abi_version(void);

#ifdef __cplusplus
}
#endif

#endif /* CONSTELLATION_B200_H_ */
