// C ABI of the hot path (include/constellation_b200.h): context, expert arena, workspace
// and the layer-level entry points that chain the kernels of this folder.
//
// Per call, everything is enqueued on the caller's stream with no host synchronisation:
//   cst_moe_layer   = router (2 kernels) -> route_pack -> pack x -> grouped up/gate ->
//                     pack h -> grouped down -> combine          (8 launches)
//   cst_moe_routed  = the same without the router
//   cst_grouped_ffn / cst_expert_forward = route_pack (rows mode) -> ... -> combine
// Capacity checks happen on the host from the call's shapes, so no device overflow can
// occur and nothing has to be read back.
#include <algorithm>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <string>
#include <vector>

#include <cuda_runtime.h>

#include "../../include/constellation_b200.h"
#include "cst_common.cuh"
#include "kernels.h"
#include "layout.cuh"

using namespace cst;

namespace {

thread_local std::string g_last_error;

int fail(int code, const char* fmt, ...) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    std::vsnprintf(buf, sizeof(buf), fmt, ap);
    va_end(ap);
    g_last_error = buf;
    return code;
}

}  // namespace

namespace cst {
void clear_last_error() { g_last_error.clear(); }
int set_last_error(int code, const char* fmt, ...) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    std::vsnprintf(buf, sizeof(buf), fmt, ap);
    va_end(ap);
    g_last_error = buf;
    return code;
}
}  // namespace cst

namespace {

#define CST_CUDA(call)                                                                      \
    do {                                                                                       \
        cudaError_t e_ = (call);                                                               \
        if (e_ != cudaSuccess)                                                                 \
            return fail(CST_ERR_CUDA, "%s failed: %s (%s:%d)", #call, cudaGetErrorString(e_), \
                        __FILE__, __LINE__);                                                   \
    } while (0)

struct Workspace {
    float* router_logits = nullptr;   // router partial logits (router_cap floats)
    int64_t router_cap = 0;
    int32_t* topk_idx = nullptr;      // [max_tokens, 16]
    float* topk_w = nullptr;
    GroupRec* groups = nullptr;       // [max_rows]
    int32_t* tile_group = nullptr;    // [max_rows]
    int32_t* row_token = nullptr;     // [max_rows]
    float* row_weight = nullptr;
    int32_t* tk_row = nullptr;        // [max(max_tokens * 16, max_rows)]
    PackMeta* meta = nullptr;
    uint8_t* xfrag = nullptr;         // [max_rows, H/128, 3072]
    float* xscale = nullptr;          // [max_rows, H/128, 24] (3 terms x 8 tokens per n-tile)
    float* h = nullptr;               // up/gate partial sums [part_rows, 2, I]
    uint8_t* hfrag = nullptr;
    float* hscale = nullptr;
    float* y = nullptr;               // [max_rows, H]
    int* err = nullptr;
    float* tok_scale = nullptr;       // prefill: per x row scale [max(max_tokens, max_rows)]
    int* hist = nullptr;              // packer counting-sort scratch
    int64_t hist_cap = 0;
};

}  // namespace

struct cst_ctx {
    int device = -1;
    cst_config cfg{};
    int num_sms = 0;
    ArenaGeom geo{};
    uint8_t* arena = nullptr;
    uint8_t* staging = nullptr;        // 3 * I * H bytes for uploads
    int32_t* d_slot_of_expert = nullptr;
    std::vector<int32_t> slot_of_expert;  // router expert -> slot
    std::vector<uint8_t> own_tokens_only;  // router expert -> served for this rank's own tokens only
    std::vector<int32_t> slot_table;       // the device copy's staging: slot | kSlotOwnTokensOnly
    std::vector<int32_t> expert_of_slot;  // slot -> router expert, -1 shared, -2 empty
    int32_t shared_slot = -1;
    int max_rows = 0;
    int part_rows = 0;  // rows of up/gate partial sums the workspace holds (K splits x rows)
    int gemm_mode = CST_GEMM_AUTO;  // cst_set_gemm_mode
    uint8_t* ws_base = nullptr;
    size_t ws_bytes = 0;
    Workspace ws;
    // cst_serve_infer_request: device copies of one request's activation and output,
    // allocated at the first request (max rows x hidden x 2 bytes each)
    uint8_t* serve_io = nullptr;
    size_t serve_half = 0;
    // stage profiling (cst_profile_enable): one event per stage boundary per call
    bool prof = false;
    std::vector<cudaEvent_t> ev_pool;
    std::vector<std::vector<cudaEvent_t>> prof_calls;
};

namespace {

// Stage boundaries of one call: 0 start | router | route_pack | pack x | up/gate | pack h |
// down | combine -> 8 events, 7 stages (CST_N_STAGES).
constexpr int kProfEvents = CST_N_STAGES + 1;

void prof_begin(cst_ctx* c, cudaStream_t s) {
    if (!c->prof) return;
    std::vector<cudaEvent_t> ev(kProfEvents);
    for (auto& e : ev) {
        if (!c->ev_pool.empty()) {
            e = c->ev_pool.back();
            c->ev_pool.pop_back();
        } else {
            cudaEventCreate(&e);
        }
    }
    c->prof_calls.push_back(std::move(ev));
    cudaEventRecord(c->prof_calls.back()[0], s);
}

// Records the end of `stage` (and of every earlier stage not recorded in this call).
void prof_mark(cst_ctx* c, int stage, cudaStream_t s) {
    if (!c->prof || c->prof_calls.empty()) return;
    cudaEventRecord(c->prof_calls.back()[stage + 1], s);
}

void prof_fill_skipped(cst_ctx* c, int upto_stage, cudaStream_t s) {
    if (!c->prof || c->prof_calls.empty()) return;
    for (int st = 0; st <= upto_stage; ++st) cudaEventRecord(c->prof_calls.back()[st + 1], s);
}

}  // namespace

namespace {

int ensure_device(const cst_ctx* c) {
    int cur = -1;
    CST_CUDA(cudaGetDevice(&cur));
    if (cur != c->device) CST_CUDA(cudaSetDevice(c->device));
    return CST_OK;
}

// The device slot table: slot of each router expert (-1: not here), with kSlotOwnTokensOnly
// set for experts served only for the tokens of this rank's shared-expert range.
cudaError_t upload_slot_table(cst_ctx* c, cudaStream_t s) {
    c->slot_table.resize(c->slot_of_expert.size());
    for (size_t e = 0; e < c->slot_of_expert.size(); ++e) {
        const int32_t v = c->slot_of_expert[e];
        c->slot_table[e] = (v >= 0 && c->own_tokens_only[e]) ? (v | kSlotOwnTokensOnly) : v;
    }
    return cudaMemcpyAsync(c->d_slot_of_expert, c->slot_table.data(), c->slot_table.size() * 4,
                           cudaMemcpyHostToDevice, s);
}

bool valid_dtype(int d) { return d == CST_DTYPE_FP16 || d == CST_DTYPE_BF16 || d == CST_DTYPE_FP32; }

// Activation rows are read and written with 8/16-byte vector accesses.
bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// rows-mode packing encodes the row index in 14 bits of the sort key (route_pack.cu)
constexpr int kMaxRowsModeRows = 16383;

size_t carve(uint8_t** cursor, size_t bytes) {
    const size_t a = (bytes + 255) / 256 * 256;
    *cursor += a;
    return a;
}

int alloc_workspace(cst_ctx* c) {
    const cst_config& f = c->cfg;
    const int H = f.hidden_dim, I = f.inter_dim, E = f.n_routed_experts;
    const int64_t R = c->max_rows;
    struct Piece {
        void** p;
        size_t bytes;
    };
    Workspace& w = c->ws;
    const size_t tk = size_t(std::max<int64_t>(int64_t(f.max_tokens) * 16, R));
    const int64_t max_routes = std::max<int64_t>(int64_t(f.max_tokens) * (f.top_k + 1), R);
    // the router's largest K split of any batch up to max_tokens (bf16 activations)
    w.router_cap = int64_t(f.max_tokens) * E;
    for (int t = 1; t <= f.max_tokens; ++t) w.router_cap = std::max(w.router_cap, router_scratch_floats(2, t, E, H));
    w.hist_cap = ((max_routes + 1023) / 1024) * std::max(f.n_slots, 1);
    std::vector<Piece> pieces = {
        {reinterpret_cast<void**>(&w.router_logits), size_t(w.router_cap) * 4},
        {reinterpret_cast<void**>(&w.topk_idx), size_t(f.max_tokens) * 16 * 4},
        {reinterpret_cast<void**>(&w.topk_w), size_t(f.max_tokens) * 16 * 4},
        {reinterpret_cast<void**>(&w.groups), size_t(R) * sizeof(GroupRec)},
        {reinterpret_cast<void**>(&w.tile_group), size_t(R) * 4},
        {reinterpret_cast<void**>(&w.row_token), size_t(R) * 4},
        {reinterpret_cast<void**>(&w.row_weight), size_t(R) * 4},
        {reinterpret_cast<void**>(&w.tk_row), tk * 4},
        {reinterpret_cast<void**>(&w.meta), sizeof(PackMeta)},
        {reinterpret_cast<void**>(&w.xfrag), size_t(R) * (H / kBlock) * kBTileBytes},
        {reinterpret_cast<void**>(&w.xscale), size_t(R) * (H / kBlock) * kScalesPerTile * 4},
        {reinterpret_cast<void**>(&w.h), size_t(c->part_rows) * 2 * I * 4},
        {reinterpret_cast<void**>(&w.hfrag), size_t(R) * (I / kBlock) * kBTileBytes},
        {reinterpret_cast<void**>(&w.hscale), size_t(R) * (I / kBlock) * kScalesPerTile * 4},
        {reinterpret_cast<void**>(&w.y), size_t(R) * H * 4},
        {reinterpret_cast<void**>(&w.err), 256},
        {reinterpret_cast<void**>(&w.hist), size_t(w.hist_cap) * 4},
        {reinterpret_cast<void**>(&w.tok_scale), size_t(std::max<int64_t>(f.max_tokens, R)) * 4},
    };
    size_t total = 0;
    for (auto& p : pieces) total += (p.bytes + 255) / 256 * 256;
    CST_CUDA(cudaMalloc(&c->ws_base, total));
    CST_CUDA(cudaMemset(c->ws_base, 0, total));
    c->ws_bytes = total;
    uint8_t* cur = c->ws_base;
    for (auto& p : pieces) {
        *p.p = cur;
        carve(&cur, p.bytes);
    }
    return CST_OK;
}

// Prefill-shaped kernels once a call averages >= 32 rows per expert: groups of 128 rows
// spread each weight tile over more tokens and two activation terms cut the tensor work.
constexpr int kPrefillMinRowsPerExpert = 32;

bool use_prefill(const cst_ctx* c, const PackArgs& pa) {
    if (c->gemm_mode == CST_GEMM_DECODE) return false;
    if (c->gemm_mode == CST_GEMM_PREFILL) return true;
    int64_t rows, experts;
    if (pa.row_slot == nullptr && pa.single_slot >= 0) {
        rows = pa.T;
        experts = 1;
    } else if (pa.row_slot != nullptr) {
        rows = pa.T;
        experts = std::max(1, c->cfg.n_slots);
    } else {
        rows = int64_t(pa.T) * pa.K;
        experts = std::max(1, c->cfg.n_routed_experts);
    }
    return rows >= kPrefillMinRowsPerExpert * experts;
}

// route_pack -> pack x -> up/gate -> pack h -> down.  Leaves y rows and tk_row filled.
int run_experts(cst_ctx* c, PackArgs pa, const void* x, int x_dtype, cudaStream_t s) {
    const int H = c->cfg.hidden_dim, I = c->cfg.inter_dim;
    Workspace& w = c->ws;
    const bool pf = use_prefill(c, pa);
    const int terms = pf ? 2 : kSplits;
    auto grouped = pf ? launch_grouped_prefill : launch_grouped_ffn;
    pa.n_slots = c->cfg.n_slots;
    pa.max_rows = c->max_rows;
    pa.max_groups = c->max_rows;
    pa.groups = w.groups;
    pa.tile_group = w.tile_group;
    pa.row_token = w.row_token;
    pa.row_weight = w.row_weight;
    pa.tk_row = w.tk_row;
    pa.meta = w.meta;
    pa.group_rows = pf ? kPrefillGroupRows : kGroupRows;
    pa.hist = w.hist;
    pa.hist_cap = w.hist_cap;
    CST_CUDA(launch_route_pack(pa, s));
    prof_mark(c, 1, s);

    PackActArgs px{x, x_dtype, H, w.row_token, w.groups, w.tile_group, w.meta, H, w.xfrag, w.xscale, terms};
    const bool rows_mode = (pa.row_slot != nullptr) || (pa.single_slot >= 0);
    const int64_t rows_bound = rows_mode ? int64_t(pa.T) : int64_t(pa.T) * (pa.K + 1);
    px.rows_hint = int(std::min<int64_t>(rows_bound, c->max_rows));
    if (pf) {
        // every token's scale once, then one pass per packed row
        CST_CUDA(launch_row_scale(px, pa.T, w.tok_scale, c->num_sms, s));
        px.src_scale = w.tok_scale;
        px.tk_row = w.tk_row;
        px.K1 = rows_mode ? 1 : pa.K + 1;
        px.n_src = pa.T;
        CST_CUDA(launch_pack_rows(px, c->num_sms, s));
    } else {
        CST_CUDA(launch_pack_act(px, c->num_sms, s));
    }
    prof_mark(c, 2, s);

    FfnArgs up{};
    up.arena = c->arena;
    up.slot_bytes = c->geo.slot_bytes;
    up.a_off = 0;
    up.s0_off = c->geo.su_off;
    up.s1_off = c->geo.sg_off;
    up.KB = H / kBlock;
    up.n_mb = I / kBlock;  // one 128-row weight block per work item
    up.scale_ld = H / kBlock;
    up.groups = w.groups;
    up.meta = w.meta;
    up.bfrag = w.xfrag;
    up.bscale = w.xscale;
    up.out = w.h;
    up.ld_out = I;
    up.out_rows = c->part_rows;
    up.max_split = kMaxUpGateSplit;
    up.row_weight = nullptr;
    up.err = w.err;
    CST_CUDA(grouped(up, true, c->num_sms, s));
    prof_mark(c, 3, s);

    PackActArgs ph{w.h, kSrcUpGatePartials, I, nullptr, w.groups, w.tile_group, w.meta, I, w.hfrag, w.hscale, terms};
    ph.rows_hint = px.rows_hint;
    CST_CUDA(pf ? launch_pack_rows(ph, c->num_sms, s) : launch_pack_act(ph, c->num_sms, s));
    prof_mark(c, 4, s);

    FfnArgs dn = up;
    dn.a_off = c->geo.upgate_bytes;
    dn.s0_off = c->geo.sd_off;
    dn.s1_off = c->geo.sd_off;
    dn.KB = I / kBlock;
    dn.n_mb = H / kBlock;
    dn.scale_ld = I / kBlock;
    dn.bfrag = w.hfrag;
    dn.bscale = w.hscale;
    dn.out = w.y;
    dn.ld_out = H;
    dn.row_weight = w.row_weight;
    dn.out_rows = c->max_rows;
    dn.max_split = 1;
    // one expert's rows (cst_expert_forward, the shared expert alone): the group count is
    // known here; routed calls leave it to the device
    dn.groups_hint = pa.single_slot >= 0 ? (pa.T + pa.group_rows - 1) / pa.group_rows : 0;
    CST_CUDA(grouped(dn, false, c->num_sms, s));
    prof_mark(c, 5, s);
    return CST_OK;
}

int check_ctx(const cst_ctx* c) {
    if (c == nullptr) return fail(CST_ERR_INVALID_ARG, "null context");
    return CST_OK;
}

}  // namespace

extern "C" {

int32_t cst_abi_version(void) { return 100; }

const char* cst_last_error(void) { return g_last_error.c_str(); }

int cst_create(int32_t device, const cst_config* cfg, cst_ctx** out) {
    g_last_error.clear();
    if (cfg == nullptr || out == nullptr) return fail(CST_ERR_INVALID_ARG, "null cfg/out");
    *out = nullptr;
    const cst_config& f = *cfg;
    if (f.block_size != kBlock) return fail(CST_ERR_INVALID_ARG, "block_size must be 128, got %d", f.block_size);
    if (f.hidden_dim <= 0 || f.hidden_dim % kBlock || f.inter_dim <= 0 || f.inter_dim % kBlock)
        return fail(CST_ERR_INVALID_ARG, "hidden_dim (%d) and inter_dim (%d) must be positive multiples of 128",
                    f.hidden_dim, f.inter_dim);
    if (f.n_routed_experts <= 0 || f.n_routed_experts > 1024)
        return fail(CST_ERR_INVALID_ARG, "n_routed_experts must be in [1, 1024]");
    if (f.n_group <= 0 || f.n_group > 32 || f.n_routed_experts % f.n_group)
        return fail(CST_ERR_INVALID_ARG, "invalid n_group=%d for n_routed_experts=%d", f.n_group,
                    f.n_routed_experts);
    if (f.topk_group <= 0 || f.topk_group > f.n_group)
        return fail(CST_ERR_INVALID_ARG, "invalid topk_group=%d for n_group=%d", f.topk_group, f.n_group);
    if (f.top_k <= 0 || f.top_k > 15 || f.top_k > f.n_routed_experts)
        return fail(CST_ERR_INVALID_ARG, "invalid top_k=%d", f.top_k);
    if (f.n_slots < 0 || f.n_slots > 8191) return fail(CST_ERR_INVALID_ARG, "n_slots must be in [0, 8191]");
    if (f.max_tokens <= 0 || f.max_tokens > 16383) return fail(CST_ERR_INVALID_ARG, "max_tokens must be in [1, 16383]");
    auto* c = new cst_ctx();
    c->device = device;
    c->cfg = f;
    c->max_rows = f.max_rows > 0 ? f.max_rows : f.max_tokens * (f.top_k + 1);
    // room for a 4-way K split of up/gate while the rows are few (the split is only chosen
    // when items are scarce, i.e. for a few hundred rows)
    c->part_rows = std::max(c->max_rows, std::min(4 * c->max_rows, 8192));
    if (c->max_rows > kRoutePackMaxRows) {
        delete c;
        return fail(CST_ERR_INVALID_ARG, "max_rows=%d exceeds %d", c->max_rows, kRoutePackMaxRows);
    }
    c->geo = ArenaGeom::make(f.hidden_dim, f.inter_dim);
    c->slot_of_expert.assign(f.n_routed_experts, -1);
    c->own_tokens_only.assign(f.n_routed_experts, 0);
    c->expert_of_slot.assign(f.n_slots, -2);
    int rc = CST_OK;
    auto bail = [&](int code) {
        cst_destroy(c);
        return code;
    };
    if (cudaSetDevice(device) != cudaSuccess) return bail(fail(CST_ERR_CUDA, "cudaSetDevice(%d) failed", device));
    int sms = 0;
    if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device) != cudaSuccess)
        return bail(fail(CST_ERR_CUDA, "cannot query SM count"));
    c->num_sms = sms;
    int major = 0, minor = 0;
    cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, device);
    cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, device);
    if (major != 10 || minor != 0)
        return bail(fail(CST_ERR_CUDA, "this library is built for sm_100a (B200); device %d is sm_%d%d", device,
                         major, minor));
    if (route_pack_init_attributes() != cudaSuccess || grouped_ffn_init_attributes() != cudaSuccess ||
        grouped_prefill_init_attributes() != cudaSuccess)
        return bail(fail(CST_ERR_CUDA, "cudaFuncSetAttribute failed: %s", cudaGetErrorString(cudaGetLastError())));
    const size_t arena = size_t(f.n_slots) * size_t(c->geo.slot_bytes);
    if (cudaMalloc(&c->arena, arena) != cudaSuccess)
        return bail(fail(CST_ERR_CUDA, "cannot allocate the %zu-byte expert arena", arena));
    if (cudaMalloc(&c->staging, size_t(3) * f.inter_dim * f.hidden_dim) != cudaSuccess)
        return bail(fail(CST_ERR_CUDA, "cannot allocate the upload staging buffer"));
    if (cudaMalloc(&c->d_slot_of_expert, size_t(f.n_routed_experts) * 4) != cudaSuccess)
        return bail(fail(CST_ERR_CUDA, "cannot allocate the slot table"));
    if (cudaMemcpy(c->d_slot_of_expert, c->slot_of_expert.data(), size_t(f.n_routed_experts) * 4,
                   cudaMemcpyHostToDevice) != cudaSuccess)
        return bail(fail(CST_ERR_CUDA, "slot table copy failed"));
    rc = alloc_workspace(c);
    if (rc != CST_OK) return bail(rc);
    *out = c;
    return CST_OK;
}

void cst_destroy(cst_ctx* c) {
    if (c == nullptr) return;
    if (c->device >= 0) {
        cudaSetDevice(c->device);
        cudaDeviceSynchronize();
    }
    for (auto& ev : c->prof_calls)
        for (auto e : ev) cudaEventDestroy(e);
    for (auto e : c->ev_pool) cudaEventDestroy(e);
    cudaFree(c->arena);
    cudaFree(c->staging);
    cudaFree(c->d_slot_of_expert);
    cudaFree(c->ws_base);
    cudaFree(c->serve_io);
    delete c;
}

int cst_upload_expert(cst_ctx* c, int32_t slot, int32_t expert_id, const cst_expert_weights* w, void* stream) {
    g_last_error.clear();
    if (int rc = check_ctx(c)) return rc;
    if (w == nullptr) return fail(CST_ERR_INVALID_ARG, "null weights");
    const int H = c->cfg.hidden_dim, I = c->cfg.inter_dim;
    if (slot < 0 || slot >= c->cfg.n_slots) return fail(CST_ERR_INVALID_ARG, "slot %d out of [0, %d)", slot, c->cfg.n_slots);
    if (expert_id < -1 || expert_id >= c->cfg.n_routed_experts)
        return fail(CST_ERR_UNKNOWN_EXPERT, "expert_id %d out of [-1, %d)", expert_id, c->cfg.n_routed_experts);
    // BuildExpertWeightsViewV2 rules (expert_format_v2.cc:68-175) for this context's shape
    if (w->rows != I || w->cols != H)
        return fail(CST_ERR_INVALID_ARG, "expert shape [%d, %d] does not match the context [%d, %d]", w->rows,
                    w->cols, I, H);
    if (w->row_block != kBlock || w->col_block != kBlock)
        return fail(CST_ERR_INVALID_ARG, "block (%d, %d) must be (128, 128)", w->row_block, w->col_block);
    if (!w->w_up || !w->w_gate || !w->w_down || !w->w_up_scale || !w->w_gate_scale || !w->w_down_scale)
        return fail(CST_ERR_INVALID_ARG, "null tensor pointer");
    if (int rc = ensure_device(c)) return rc;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const size_t mat = size_t(I) * H;
    CST_CUDA(cudaMemcpyAsync(c->staging, w->w_up, mat, cudaMemcpyDefault, s));
    CST_CUDA(cudaMemcpyAsync(c->staging + mat, w->w_gate, mat, cudaMemcpyDefault, s));
    CST_CUDA(cudaMemcpyAsync(c->staging + 2 * mat, w->w_down, mat, cudaMemcpyDefault, s));
    uint8_t* dst = c->arena + int64_t(slot) * c->geo.slot_bytes;
    CST_CUDA(launch_relayout(c->staging, c->staging + mat, c->staging + 2 * mat, dst, I, H, c->num_sms, s));
    const size_t grid = size_t(I / kBlock) * (H / kBlock) * 4;
    CST_CUDA(cudaMemcpyAsync(dst + c->geo.su_off, w->w_up_scale, grid, cudaMemcpyDefault, s));
    CST_CUDA(cudaMemcpyAsync(dst + c->geo.sg_off, w->w_gate_scale, grid, cudaMemcpyDefault, s));
    CST_CUDA(cudaMemcpyAsync(dst + c->geo.sd_off, w->w_down_scale, grid, cudaMemcpyDefault, s));
    // bookkeeping: a slot holds one expert; re-uploading replaces it (ExpertRegistryV2::Update)
    const int old = c->expert_of_slot[slot];
    if (old >= 0) c->slot_of_expert[old] = -1;
    if (old == -1 && c->shared_slot == slot) c->shared_slot = -1;
    if (expert_id >= 0) {
        const int prev = c->slot_of_expert[expert_id];
        if (prev >= 0 && prev != slot) c->expert_of_slot[prev] = -2;
        c->slot_of_expert[expert_id] = slot;
        c->expert_of_slot[slot] = expert_id;
    } else {
        c->expert_of_slot[slot] = -1;
        c->shared_slot = slot;
    }
    CST_CUDA(upload_slot_table(c, s));
    // upload is a load-time path: finish it before the staging buffer is reused
    CST_CUDA(cudaStreamSynchronize(s));
    return CST_OK;
}

int cst_free_expert(cst_ctx* c, int32_t slot) {
    g_last_error.clear();
    if (int rc = check_ctx(c)) return rc;
    if (slot < 0 || slot >= c->cfg.n_slots) return fail(CST_ERR_INVALID_ARG, "slot %d out of range", slot);
    if (int rc = ensure_device(c)) return rc;
    const int e = c->expert_of_slot[slot];
    if (e >= 0) c->slot_of_expert[e] = -1;
    if (c->shared_slot == slot) c->shared_slot = -1;
    c->expert_of_slot[slot] = -2;
    CST_CUDA(cudaDeviceSynchronize());
    CST_CUDA(upload_slot_table(c, nullptr));
    CST_CUDA(cudaDeviceSynchronize());
    return CST_OK;
}

int cst_set_expert_own_tokens_only(cst_ctx* c, int32_t expert_id, int32_t own_tokens_only) {
    g_last_error.clear();
    if (int rc = check_ctx(c)) return rc;
    if (expert_id < 0 || expert_id >= c->cfg.n_routed_experts)
        return fail(CST_ERR_UNKNOWN_EXPERT, "expert_id %d out of [0, %d)", expert_id, c->cfg.n_routed_experts);
    if (int rc = ensure_device(c)) return rc;
    c->own_tokens_only[expert_id] = own_tokens_only ? 1 : 0;
    CST_CUDA(cudaDeviceSynchronize());
    CST_CUDA(upload_slot_table(c, nullptr));
    CST_CUDA(cudaDeviceSynchronize());
    return CST_OK;
}

int32_t cst_find_slot(const cst_ctx* c, int32_t expert_id) {
    if (c == nullptr || expert_id < 0 || expert_id >= c->cfg.n_routed_experts) return -1;
    return c->slot_of_expert[expert_id];
}

int cst_set_gemm_mode(cst_ctx* c, int32_t mode) {
    g_last_error.clear();
    if (int rc = check_ctx(c)) return rc;
    if (mode != CST_GEMM_AUTO && mode != CST_GEMM_DECODE && mode != CST_GEMM_PREFILL)
        return fail(CST_ERR_INVALID_ARG, "gemm mode %d is not one of 0 (auto), 1 (decode), 2 (prefill)", mode);
    c->gemm_mode = mode;
    return CST_OK;
}

int cst_set_shared_slot(cst_ctx* c, int32_t slot) {
    g_last_error.clear();
    if (int rc = check_ctx(c)) return rc;
    if (slot < -1 || slot >= c->cfg.n_slots) return fail(CST_ERR_INVALID_ARG, "slot %d out of range", slot);
    c->shared_slot = slot;
    return CST_OK;
}

int cst_route(cst_ctx* c, const void* x, int32_t x_dtype, int32_t T, const float* gate_weight, const float* bias,
              const uint8_t* resident, int32_t top_k, int32_t* topk_idx, float* topk_weight, float* logits,
              float* group_scores, void* stream) {
    g_last_error.clear();
    if (int rc = check_ctx(c)) return rc;
    if (!valid_dtype(x_dtype)) return fail(CST_ERR_INVALID_ARG, "bad x_dtype %d", x_dtype);
    if (T < 0 || T > c->cfg.max_tokens) return fail(CST_ERR_INVALID_ARG, "T=%d exceeds max_tokens=%d", T, c->cfg.max_tokens);
    if (top_k <= 0 || top_k > c->cfg.top_k) return fail(CST_ERR_INVALID_ARG, "top_k=%d out of [1, %d]", top_k, c->cfg.top_k);
    if (T == 0) return CST_OK;  // empty batch: no work, pointers may be null
    if (!x || !gate_weight || !bias || !topk_idx || !topk_weight) return fail(CST_ERR_INVALID_ARG, "null pointer");
    if (!aligned16(x) || !aligned16(gate_weight))
        return fail(CST_ERR_INVALID_ARG, "x and gate_weight must be 16-byte aligned");
    if (int rc = ensure_device(c)) return rc;
    const cst_config& f = c->cfg;
    CST_CUDA(launch_router(x, x_dtype, gate_weight, bias, resident, T, f.n_routed_experts, f.hidden_dim, f.n_group,
                           f.topk_group, top_k, f.norm_topk_prob, f.routed_scaling_factor, c->ws.router_logits,
                           c->ws.router_cap, topk_idx, topk_weight, group_scores, c->ws.err,
                           static_cast<cudaStream_t>(stream), true, logits));
    return CST_OK;
}

static int moe_routed_impl(cst_ctx* c, const void* x, int x_dtype, int T, const int32_t* topk_idx,
                           const float* topk_w, int K, uint32_t flags, const void* residual, void* out,
                           int out_dtype, cudaStream_t s, int shared_begin = 0, int shared_end = -1,
                           const PeerSet* push = nullptr) {
    const bool shared = (flags & CST_FLAG_ADD_SHARED) != 0;
    if (shared && c->shared_slot < 0) return fail(CST_ERR_NOT_RESIDENT, "no shared expert is resident");
    if (shared_end < 0) shared_end = T;
    if (int64_t(T) * (K + 1) > c->max_rows)
        return fail(CST_ERR_INVALID_ARG, "T*(top_k+1)=%d exceeds the workspace (%d rows)", T * (K + 1), c->max_rows);
    PackArgs pa{};
    pa.topk_idx = topk_idx;
    pa.topk_w = topk_w;
    pa.slot_of_expert = c->d_slot_of_expert;
    pa.E = c->cfg.n_routed_experts;
    pa.K = K;
    pa.shared_slot = shared ? c->shared_slot : -1;
    pa.shared_t_begin = shared_begin;
    pa.shared_t_end = shared_end;
    pa.row_slot = nullptr;
    pa.single_slot = -1;
    pa.row_weight_in = nullptr;
    pa.T = T;
    if (int rc = run_experts(c, pa, x, x_dtype, s)) return rc;
    if (push != nullptr) {
        PushArgs pu{c->ws.y, c->cfg.hidden_dim, c->ws.tk_row, K + 1, T, c->cfg.hidden_dim, push->tl, *push};
        CST_CUDA(launch_combine_push(pu, s));
    } else {
        CombineArgs ca{c->ws.y, c->cfg.hidden_dim, c->ws.tk_row, K + 1, T, c->cfg.hidden_dim,
                       residual, x_dtype, out, out_dtype, nullptr};
        CST_CUDA(launch_combine(ca, s));
    }
    prof_mark(c, 6, s);
    return CST_OK;
}

static int peer_set_from(const cst_peer_set* p, PeerSet* out) {
    if (p == nullptr) return fail(CST_ERR_INVALID_ARG, "null peer set");
    if (p->world < 1 || p->world > CST_MAX_PEERS || p->rank < 0 || p->rank >= p->world)
        return fail(CST_ERR_INVALID_ARG, "peer set: world=%d rank=%d", p->world, p->rank);
    if (p->tl <= 0 || p->tl > p->tl_cap) return fail(CST_ERR_INVALID_ARG, "peer set: tl=%d tl_cap=%d", p->tl, p->tl_cap);
    if (!p->epoch || !p->done) return fail(CST_ERR_INVALID_ARG, "peer set: null epoch/counter");
    PeerSet q{};
    q.world = p->world;
    q.rank = p->rank;
    q.tl = p->tl;
    q.tl_cap = p->tl_cap;
    for (int r = 0; r < p->world; ++r) {
        if (!p->recv[r] || !p->flags[r] || !aligned16(p->recv[r]))
            return fail(CST_ERR_INVALID_ARG, "peer set: rank %d buffers missing or unaligned", r);
        q.recv[r] = p->recv[r];
        q.flags[r] = p->flags[r];
    }
    q.epoch = p->epoch;
    q.done = p->done;
    if (p->x_offset < 0 || p->x_offset % 16 || (p->x_offset > 0 && !p->gather_epoch))
        return fail(CST_ERR_INVALID_ARG, "peer set: bad gathered-row region (offset %lld)",
                    static_cast<long long>(p->x_offset));
    q.x_off = p->x_offset;
    q.gather_epoch = p->gather_epoch;
    if (p->presence_offset < 0 || p->presence_offset % 16)
        return fail(CST_ERR_INVALID_ARG, "peer set: bad presence offset %lld",
                    static_cast<long long>(p->presence_offset));
    q.pres_off = p->presence_offset;
    *out = q;
    return CST_OK;
}

int cst_moe_routed(cst_ctx* c, const void* x, int32_t x_dtype, int32_t T, const int32_t* topk_idx,
                   const float* topk_weight, int32_t top_k, uint32_t flags, void* out, int32_t out_dtype,
                   void* stream) {
    g_last_error.clear();
    if (int rc = check_ctx(c)) return rc;
    if (!valid_dtype(x_dtype) || !valid_dtype(out_dtype)) return fail(CST_ERR_INVALID_ARG, "bad dtype");
    if (T < 0 || T > c->cfg.max_tokens) return fail(CST_ERR_INVALID_ARG, "T=%d out of range", T);
    if (top_k <= 0 || top_k > 15) return fail(CST_ERR_INVALID_ARG, "top_k=%d out of range", top_k);
    if (T == 0) return CST_OK;
    if (!x || !out || !topk_idx || !topk_weight) return fail(CST_ERR_INVALID_ARG, "null pointer");
    if (!aligned16(x) || !aligned16(out)) return fail(CST_ERR_INVALID_ARG, "x and out must be 16-byte aligned");
    if (int rc = ensure_device(c)) return rc;
    prof_begin(c, static_cast<cudaStream_t>(stream));
    prof_fill_skipped(c, 0, static_cast<cudaStream_t>(stream));
    return moe_routed_impl(c, x, x_dtype, T, topk_idx, topk_weight, top_k, flags, nullptr, out, out_dtype,
                           static_cast<cudaStream_t>(stream));
}

int cst_moe_routed_range(cst_ctx* c, const void* x, int32_t x_dtype, int32_t T, const int32_t* topk_idx,
                         const float* topk_weight, int32_t top_k, int32_t shared_begin, int32_t shared_end,
                         void* out, int32_t out_dtype, void* stream) {
    g_last_error.clear();
    if (int rc = check_ctx(c)) return rc;
    if (!valid_dtype(x_dtype) || !valid_dtype(out_dtype)) return fail(CST_ERR_INVALID_ARG, "bad dtype");
    if (T < 0 || T > c->cfg.max_tokens) return fail(CST_ERR_INVALID_ARG, "T=%d out of range", T);
    if (top_k <= 0 || top_k > 15) return fail(CST_ERR_INVALID_ARG, "top_k=%d out of range", top_k);
    if (shared_begin < 0 || shared_end < shared_begin || shared_end > T)
        return fail(CST_ERR_INVALID_ARG, "shared token range [%d, %d) outside [0, %d)", shared_begin, shared_end, T);
    if (T == 0) return CST_OK;
    if (!x || !out || !topk_idx || !topk_weight) return fail(CST_ERR_INVALID_ARG, "null pointer");
    if (!aligned16(x) || !aligned16(out)) return fail(CST_ERR_INVALID_ARG, "x and out must be 16-byte aligned");
    if (int rc = ensure_device(c)) return rc;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    prof_begin(c, s);
    prof_fill_skipped(c, 0, s);
    const uint32_t flags = shared_end > shared_begin ? CST_FLAG_ADD_SHARED : 0u;
    return moe_routed_impl(c, x, x_dtype, T, topk_idx, topk_weight, top_k, flags, nullptr, out, out_dtype, s,
                           shared_begin, shared_end);
}

int cst_moe_layer(cst_ctx* c, const void* x, int32_t x_dtype, int32_t T, const float* gate_weight, const float* bias,
                  const uint8_t* resident, int32_t top_k, uint32_t flags, const void* residual, void* out,
                  int32_t out_dtype, int32_t* topk_idx, float* topk_weight, void* stream) {
    g_last_error.clear();
    if (int rc = check_ctx(c)) return rc;
    if (!valid_dtype(x_dtype) || !valid_dtype(out_dtype)) return fail(CST_ERR_INVALID_ARG, "bad dtype");
    if (T < 0 || T > c->cfg.max_tokens) return fail(CST_ERR_INVALID_ARG, "T=%d exceeds max_tokens=%d", T, c->cfg.max_tokens);
    if (top_k <= 0 || top_k > c->cfg.top_k) return fail(CST_ERR_INVALID_ARG, "top_k=%d out of range", top_k);
    if (T == 0) return CST_OK;
    if (!x || !out || !gate_weight || !bias) return fail(CST_ERR_INVALID_ARG, "null pointer");
    if (!aligned16(x) || !aligned16(out) || !aligned16(gate_weight) || (residual && !aligned16(residual)))
        return fail(CST_ERR_INVALID_ARG, "x, out, gate_weight and residual must be 16-byte aligned");
    if (int rc = ensure_device(c)) return rc;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    int32_t* idx = topk_idx ? topk_idx : c->ws.topk_idx;
    float* wts = topk_weight ? topk_weight : c->ws.topk_w;
    const cst_config& f = c->cfg;
    prof_begin(c, s);
    CST_CUDA(launch_router(x, x_dtype, gate_weight, bias, resident, T, f.n_routed_experts, f.hidden_dim, f.n_group,
                           f.topk_group, top_k, f.norm_topk_prob, f.routed_scaling_factor, c->ws.router_logits,
                           c->ws.router_cap, idx, wts, nullptr, c->ws.err, s));
    prof_mark(c, 0, s);
    return moe_routed_impl(c, x, x_dtype, T, idx, wts, top_k, flags, residual, out, out_dtype, s);
}

int cst_grouped_ffn(cst_ctx* c, const void* x, int32_t x_dtype, int32_t R, const int32_t* row_slot,
                    const float* row_weight, void* y, int32_t y_dtype, void* stream) {
    g_last_error.clear();
    if (int rc = check_ctx(c)) return rc;
    if (!valid_dtype(x_dtype) || !valid_dtype(y_dtype)) return fail(CST_ERR_INVALID_ARG, "bad dtype");
    if (R < 0 || R > c->max_rows) return fail(CST_ERR_INVALID_ARG, "R=%d exceeds the workspace (%d rows)", R, c->max_rows);
    if (R > kMaxRowsModeRows) return fail(CST_ERR_INVALID_ARG, "R=%d exceeds %d rows per call", R, kMaxRowsModeRows);
    if (R == 0) return CST_OK;
    if (!x || !y || !row_slot) return fail(CST_ERR_INVALID_ARG, "null pointer");
    if (!aligned16(x) || !aligned16(y)) return fail(CST_ERR_INVALID_ARG, "x and y must be 16-byte aligned");
    if (int rc = ensure_device(c)) return rc;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    PackArgs pa{};
    pa.row_slot = row_slot;
    pa.single_slot = -1;
    pa.row_weight_in = row_weight;
    pa.T = R;
    pa.shared_slot = -1;
    prof_begin(c, s);
    prof_fill_skipped(c, 0, s);
    if (int rc = run_experts(c, pa, x, x_dtype, s)) return rc;
    CombineArgs ca{c->ws.y, c->cfg.hidden_dim, c->ws.tk_row, 1, R, c->cfg.hidden_dim, nullptr, 0, y, y_dtype, nullptr};
    CST_CUDA(launch_combine(ca, s));
    prof_mark(c, 6, s);
    return CST_OK;
}

int cst_expert_forward(cst_ctx* c, int32_t expert_id, const void* x, int32_t in_dtype, int32_t batch, void* y,
                       int32_t out_dtype, void* stream) {
    g_last_error.clear();
    if (int rc = check_ctx(c)) return rc;
    if (expert_id < 0 || expert_id >= c->cfg.n_routed_experts)
        return fail(CST_ERR_UNKNOWN_EXPERT, "unknown expert %d", expert_id);
    const int slot = c->slot_of_expert[expert_id];
    if (slot < 0) return fail(CST_ERR_NOT_RESIDENT, "expert %d is not resident on this device", expert_id);
    // the reference serves fp16/bf16 in x fp16/bf16 out; fp32 output is an extension that
    // returns the unrounded expert result
    if ((in_dtype != CST_DTYPE_FP16 && in_dtype != CST_DTYPE_BF16) || !valid_dtype(out_dtype))
        return fail(CST_ERR_BACKEND, "unsupported dtype pair (%d, %d)", in_dtype, out_dtype);
    if (batch <= 0 || batch > c->max_rows) return fail(CST_ERR_BACKEND, "batch %d out of [1, %d]", batch, c->max_rows);
    if (!x || !y) return fail(CST_ERR_INVALID_ARG, "null pointer");
    if (batch > kMaxRowsModeRows) return fail(CST_ERR_BACKEND, "batch %d exceeds %d", batch, kMaxRowsModeRows);
    if (!aligned16(x) || !aligned16(y)) return fail(CST_ERR_INVALID_ARG, "x and y must be 16-byte aligned");
    if (int rc = ensure_device(c)) return rc;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    PackArgs pa{};
    pa.row_slot = nullptr;
    pa.single_slot = slot;
    pa.row_weight_in = nullptr;
    pa.T = batch;
    pa.shared_slot = -1;
    prof_begin(c, s);
    prof_fill_skipped(c, 0, s);
    if (int rc = run_experts(c, pa, x, in_dtype, s)) return rc;
    CombineArgs ca{c->ws.y, c->cfg.hidden_dim, c->ws.tk_row, 1, batch, c->cfg.hidden_dim, nullptr, 0, y, out_dtype,
                   nullptr};
    CST_CUDA(launch_combine(ca, s));
    prof_mark(c, 6, s);
    return CST_OK;
}

}  // extern "C"

namespace {

// The device half of one request: activation in, expert run, output back into the host
// response, stream synchronised (the reference worker copies synchronously too,
// backend_workspace_cuda_v2.cc:64-105).
int serve_run(cst_ctx* c, int32_t local_id, const cst_infer_request& m, uint8_t* out_host, void* stream) {
    if (int rc = ensure_device(c)) return rc;
    if (c->serve_io == nullptr) {
        const int64_t rows = std::min<int64_t>(c->max_rows, kMaxRowsModeRows);
        const size_t half = (size_t(rows) * c->cfg.hidden_dim * 2 + 255) & ~size_t(255);
        CST_CUDA(cudaMalloc(&c->serve_io, 2 * half));
        c->serve_half = half;
    }
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const size_t nbytes = m.activation_bytes;  // batch * hidden * 2, checked by the caller
    uint8_t* din = c->serve_io;
    uint8_t* dout = c->serve_io + c->serve_half;
    CST_CUDA(cudaMemcpyAsync(din, m.activation, nbytes, cudaMemcpyHostToDevice, s));
    if (int rc = cst_expert_forward(c, local_id, din, int32_t(m.input_dtype), m.batch_size, dout,
                                    int32_t(m.output_dtype), stream))
        return rc;
    CST_CUDA(cudaMemcpyAsync(out_host, dout, nbytes, cudaMemcpyDeviceToHost, s));
    CST_CUDA(cudaStreamSynchronize(s));
    return CST_OK;
}

}  // namespace

extern "C" {

int cst_serve_infer_request(cst_ctx* const* layers, int32_t n_layers, int32_t experts_per_layer,
                            const uint8_t* req_body, int64_t req_len, uint8_t* resp_body, int64_t resp_cap,
                            int64_t* resp_len, void* stream) {
    g_last_error.clear();
    if (resp_len == nullptr) return fail(CST_ERR_INVALID_ARG, "null resp_len");
    *resp_len = 0;
    if (n_layers < 0 || (n_layers > 0 && layers == nullptr) || experts_per_layer <= 0)
        return fail(CST_ERR_INVALID_ARG, "bad layer table (n_layers=%d, experts_per_layer=%d)", n_layers,
                    experts_per_layer);
    cst_infer_request m{};
    if (int rc = cst_decode_infer_request(req_body, req_len, &m)) return rc;  // no reply (worker.cc:92-97)
    // the worker's lookup (worker.cc:112-130): no entry -> 1, not on this device -> 2
    int32_t status = CST_ERR_BACKEND;
    cst_ctx* c = nullptr;
    int32_t local_id = -1;
    const int32_t layer = m.expert_id >= 0 ? m.expert_id / experts_per_layer : -1;
    if (layer < 0 || layer >= n_layers || layers[layer] == nullptr) {
        status = CST_ERR_UNKNOWN_EXPERT;
    } else {
        c = layers[layer];
        if (c->cfg.n_routed_experts != experts_per_layer)
            return fail(CST_ERR_INVALID_ARG, "experts_per_layer=%d, but the layer-%d context routes %d experts",
                        experts_per_layer, layer, c->cfg.n_routed_experts);
        local_id = m.expert_id % experts_per_layer;
        if (c->slot_of_expert[local_id] < 0) status = CST_ERR_NOT_RESIDENT;
    }
    // RunExpertRequest's checks (backend_workspace_cuda_v2.cc:139-181, :33-39), batch >= 1
    int64_t out_bytes = 0;
    bool usable = false;
    if (c != nullptr && status == CST_ERR_BACKEND) {
        const int64_t H = c->cfg.hidden_dim;
        const int64_t max_batch = std::min<int64_t>(c->max_rows, kMaxRowsModeRows);
        const auto wire = [](uint32_t d) { return d == CST_DTYPE_FP16 || d == CST_DTYPE_BF16; };
        if (m.batch_size < 1 || m.batch_size > max_batch)
            fail(CST_ERR_BACKEND, "batch %d outside [1, %lld]", m.batch_size, static_cast<long long>(max_batch));
        else if (m.hidden_dim != H)
            fail(CST_ERR_BACKEND, "hidden_dim %d, the context has %lld", m.hidden_dim, static_cast<long long>(H));
        else if (!wire(m.input_dtype) || !wire(m.output_dtype))
            fail(CST_ERR_BACKEND, "unsupported dtype pair (%u, %u)", m.input_dtype, m.output_dtype);
        else if (int64_t(m.activation_bytes) != int64_t(m.batch_size) * H * 2)
            fail(CST_ERR_BACKEND, "activation holds %u bytes, batch x hidden x 2 = %lld", m.activation_bytes,
                 static_cast<long long>(int64_t(m.batch_size) * H * 2));
        else {
            usable = true;
            out_bytes = int64_t(m.batch_size) * H * 2;
        }
    }
    const int64_t need = kInferResponseFixedBytes + out_bytes;
    if (resp_body == nullptr || resp_cap < need) {
        *resp_len = need;
        return fail(CST_ERR_INVALID_ARG, "the response needs %lld bytes, the buffer holds %lld",
                    static_cast<long long>(need), static_cast<long long>(resp_body ? resp_cap : 0));
    }
    if (usable) {
        if (serve_run(c, local_id, m, resp_body + kInferResponseFixedBytes, stream) == CST_OK) {
            status = CST_OK;
        } else {
            out_bytes = 0;  // the worker's failed run: status 4, no output (worker.cc:124-128)
        }
    }
    put_infer_response_fixed(resp_body, status, m.batch_size, m.hidden_dim, m.output_dtype, uint32_t(out_bytes));
    *resp_len = kInferResponseFixedBytes + out_bytes;
    return CST_OK;
}

int cst_shared_combine(cst_ctx* c, const void* x, int32_t x_dtype, int32_t T, const float* extra,
                       const void* residual, void* out, int32_t out_dtype, void* stream) {
    g_last_error.clear();
    if (int rc = check_ctx(c)) return rc;
    if (!valid_dtype(x_dtype) || !valid_dtype(out_dtype)) return fail(CST_ERR_INVALID_ARG, "bad dtype");
    if (T < 0 || T > c->max_rows || T > kMaxRowsModeRows) return fail(CST_ERR_INVALID_ARG, "T=%d out of range", T);
    if (T == 0) return CST_OK;
    if (!x || !out) return fail(CST_ERR_INVALID_ARG, "null pointer");
    if (!aligned16(x) || !aligned16(out) || (extra && !aligned16(extra)) || (residual && !aligned16(residual)))
        return fail(CST_ERR_INVALID_ARG, "x, extra, residual and out must be 16-byte aligned");
    if (int rc = ensure_device(c)) return rc;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    prof_begin(c, s);
    prof_fill_skipped(c, 0, s);
    if (c->shared_slot >= 0) {
        PackArgs pa{};
        pa.row_slot = nullptr;
        pa.single_slot = c->shared_slot;
        pa.row_weight_in = nullptr;
        pa.T = T;
        pa.shared_slot = -1;
        if (int rc = run_experts(c, pa, x, x_dtype, s)) return rc;
    } else {
        // no shared expert: only extra + residual; tk_row = -1 everywhere
        CST_CUDA(cudaMemsetAsync(c->ws.tk_row, 0xff, size_t(T) * sizeof(int32_t), s));
        prof_fill_skipped(c, 5, s);
    }
    CombineArgs ca{c->ws.y, c->cfg.hidden_dim, c->ws.tk_row, 1, T, c->cfg.hidden_dim, residual, x_dtype, out,
                   out_dtype, extra};
    CST_CUDA(launch_combine(ca, s));
    prof_mark(c, 6, s);
    return CST_OK;
}

int cst_combine_rows(cst_ctx* c, const float* rows, int64_t ld_rows, const int32_t* tk_row, int32_t k1, int32_t T,
                     const float* extra, const void* residual, int32_t residual_dtype, void* out, int32_t out_dtype,
                     void* stream) {
    g_last_error.clear();
    if (int rc = check_ctx(c)) return rc;
    if (!valid_dtype(out_dtype) || (residual && !valid_dtype(residual_dtype)))
        return fail(CST_ERR_INVALID_ARG, "bad dtype");
    if (T < 0 || k1 < 0 || k1 > 16) return fail(CST_ERR_INVALID_ARG, "bad arguments (T=%d, k1=%d; k1 must be <= 16)", T, k1);
    if (T == 0) return CST_OK;
    if ((k1 > 0 && (!rows || !tk_row)) || !out) return fail(CST_ERR_INVALID_ARG, "null pointer");
    if ((rows && (!aligned16(rows) || ld_rows % 4)) || !aligned16(out) || (extra && !aligned16(extra)) ||
        (residual && !aligned16(residual)))
        return fail(CST_ERR_INVALID_ARG, "rows, extra, residual and out must be 16-byte aligned");
    if (int rc = ensure_device(c)) return rc;
    CombineArgs ca{rows, ld_rows, tk_row, k1, T, c->cfg.hidden_dim, residual, residual_dtype, out, out_dtype, extra};
    CST_CUDA(launch_combine(ca, static_cast<cudaStream_t>(stream)));
    return CST_OK;
}

int cst_dequant_fp8(const uint8_t* w, const float* scale_inv, int32_t rows, int32_t cols, int32_t block, float* out,
                    void* stream) {
    g_last_error.clear();
    if (!w || !scale_inv || !out) return fail(CST_ERR_INVALID_ARG, "null pointer");
    if (rows <= 0 || cols <= 0 || block <= 0) return fail(CST_ERR_INVALID_ARG, "bad shape (%d, %d, %d)", rows, cols, block);
    if (!aligned16(w) || !aligned16(out)) return fail(CST_ERR_INVALID_ARG, "w and out must be 16-byte aligned");
    int dev = 0, sms = 0;
    CST_CUDA(cudaGetDevice(&dev));
    CST_CUDA(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
    CST_CUDA(launch_dequant_fp8(w, scale_inv, out, rows, cols, block, sms, static_cast<cudaStream_t>(stream)));
    return CST_OK;
}

int cst_rmsnorm(const void* x, int32_t x_dtype, int32_t T, int32_t H, const float* weight, float eps, void* out,
                int32_t out_dtype, void* stream) {
    g_last_error.clear();
    if (!valid_dtype(x_dtype) || !valid_dtype(out_dtype)) return fail(CST_ERR_INVALID_ARG, "bad dtype");
    if (T < 0 || H <= 0 || H % 8) return fail(CST_ERR_INVALID_ARG, "bad shape (T=%d, H=%d; H must be a multiple of 8)", T, H);
    if (!(eps >= 0.0f)) return fail(CST_ERR_INVALID_ARG, "eps must be >= 0");
    if (T == 0) return CST_OK;
    if (!x || !out) return fail(CST_ERR_INVALID_ARG, "null pointer");
    if (!aligned16(x) || !aligned16(out)) return fail(CST_ERR_INVALID_ARG, "x and out must be 16-byte aligned");
    CST_CUDA(launch_rmsnorm(x, x_dtype, T, H, weight, eps, out, out_dtype, static_cast<cudaStream_t>(stream)));
    return CST_OK;
}

int cst_moe_routed_push(cst_ctx* c, const void* x, int32_t x_dtype, const int32_t* topk_idx,
                        const float* topk_weight, int32_t top_k, const cst_peer_set* peers, void* stream) {
    g_last_error.clear();
    if (int rc = check_ctx(c)) return rc;
    PeerSet ps{};
    if (int rc = peer_set_from(peers, &ps)) return rc;
    const int T = ps.world * ps.tl;
    if (!valid_dtype(x_dtype)) return fail(CST_ERR_INVALID_ARG, "bad dtype");
    if (T > c->cfg.max_tokens) return fail(CST_ERR_INVALID_ARG, "T=%d exceeds max_tokens=%d", T, c->cfg.max_tokens);
    if (top_k <= 0 || top_k > 15) return fail(CST_ERR_INVALID_ARG, "top_k=%d out of range", top_k);
    if (!x || !topk_idx || !topk_weight) return fail(CST_ERR_INVALID_ARG, "null pointer");
    if (!aligned16(x)) return fail(CST_ERR_INVALID_ARG, "x must be 16-byte aligned");
    if (c->cfg.hidden_dim % 4) return fail(CST_ERR_INVALID_ARG, "hidden_dim must be a multiple of 4");
    if (int rc = ensure_device(c)) return rc;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    prof_begin(c, s);
    prof_fill_skipped(c, 0, s);
    const int lo = ps.rank * ps.tl;
    const uint32_t flags = c->shared_slot >= 0 ? CST_FLAG_ADD_SHARED : 0u;
    return moe_routed_impl(c, x, x_dtype, T, topk_idx, topk_weight, top_k, flags, nullptr, nullptr, CST_DTYPE_FP32,
                           s, lo, lo + ps.tl, &ps);
}

int cst_gather_rows(cst_ctx* c, const cst_peer_set* peers, const void* x, int32_t x_dtype, void* stream) {
    g_last_error.clear();
    if (int rc = check_ctx(c)) return rc;
    PeerSet ps{};
    if (int rc = peer_set_from(peers, &ps)) return rc;
    if (ps.x_off == 0) return fail(CST_ERR_INVALID_ARG, "the peer set has no gathered-row slots");
    if (x_dtype != CST_DTYPE_FP16 && x_dtype != CST_DTYPE_BF16)
        return fail(CST_ERR_INVALID_ARG, "gathered rows must be fp16 or bf16, got dtype %d", x_dtype);
    if (!x || !aligned16(x)) return fail(CST_ERR_INVALID_ARG, "x must be non-null and 16-byte aligned");
    if (int rc = ensure_device(c)) return rc;
    GatherArgs ga{ps, x, ps.tl, c->cfg.hidden_dim, c->ws.err};
    CST_CUDA(launch_gather_rows(ga, static_cast<cudaStream_t>(stream)));
    return CST_OK;
}

int cst_reduce_pushed(cst_ctx* c, const cst_peer_set* peers, const void* residual, int32_t residual_dtype,
                      void* out, int32_t out_dtype, void* stream) {
    g_last_error.clear();
    if (int rc = check_ctx(c)) return rc;
    PeerSet ps{};
    if (int rc = peer_set_from(peers, &ps)) return rc;
    if (!valid_dtype(out_dtype) || (residual && !valid_dtype(residual_dtype)))
        return fail(CST_ERR_INVALID_ARG, "bad dtype");
    if (!out || !aligned16(out) || (residual && !aligned16(residual)))
        return fail(CST_ERR_INVALID_ARG, "out (and residual) must be non-null and 16-byte aligned");
    if (int rc = ensure_device(c)) return rc;
    ReduceArgs ra{ps, ps.tl, c->cfg.hidden_dim, push_chunks(c->cfg.hidden_dim), residual, residual_dtype, out,
                  out_dtype, c->ws.err};
    CST_CUDA(launch_reduce_cast(ra, static_cast<cudaStream_t>(stream)));
    return CST_OK;
}

int cst_ipc_alloc(int64_t bytes, void** ptr, cst_ipc_handle* handle) {
    g_last_error.clear();
    if (bytes <= 0 || !ptr || !handle) return fail(CST_ERR_INVALID_ARG, "bad arguments");
    static_assert(sizeof(cudaIpcMemHandle_t) <= sizeof(cst_ipc_handle), "IPC handle does not fit");
    void* p = nullptr;
    CST_CUDA(cudaMalloc(&p, size_t(bytes)));
    cudaError_t e = cudaMemset(p, 0, size_t(bytes));
    cudaIpcMemHandle_t h;
    if (e == cudaSuccess) e = cudaIpcGetMemHandle(&h, p);
    if (e != cudaSuccess) {
        cudaFree(p);
        return fail(CST_ERR_CUDA, "cst_ipc_alloc: %s", cudaGetErrorString(e));
    }
    std::memset(handle, 0, sizeof(*handle));
    std::memcpy(handle->bytes, &h, sizeof(h));
    *ptr = p;
    return CST_OK;
}

int cst_ipc_open(const cst_ipc_handle* handle, void** ptr) {
    g_last_error.clear();
    if (!handle || !ptr) return fail(CST_ERR_INVALID_ARG, "null argument");
    cudaIpcMemHandle_t h;
    std::memcpy(&h, handle->bytes, sizeof(h));
    void* p = nullptr;
    CST_CUDA(cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess));
    *ptr = p;
    return CST_OK;
}

int cst_ipc_close(void* ptr) {
    g_last_error.clear();
    if (!ptr) return CST_OK;
    CST_CUDA(cudaIpcCloseMemHandle(ptr));
    return CST_OK;
}

int cst_ipc_free(void* ptr) {
    g_last_error.clear();
    if (!ptr) return CST_OK;
    CST_CUDA(cudaFree(ptr));
    return CST_OK;
}

int cst_device_error(cst_ctx* c) {
    g_last_error.clear();
    if (int rc = check_ctx(c)) return rc;
    if (int rc = ensure_device(c)) return rc;
    CST_CUDA(cudaDeviceSynchronize());
    int v = 0;
    CST_CUDA(cudaMemcpy(&v, c->ws.err, sizeof(int), cudaMemcpyDeviceToHost));
    if (v != CST_DEV_OK) {
        CST_CUDA(cudaMemset(c->ws.err, 0, sizeof(int)));
        return fail(CST_ERR_DEVICE_TIMEOUT, "a device-side wait gave up (code %d)", v);
    }
    return CST_OK;
}

int cst_profile_enable(cst_ctx* c, int32_t enable) {
    g_last_error.clear();
    if (int rc = check_ctx(c)) return rc;
    c->prof = enable != 0;
    return CST_OK;
}

int cst_profile_read(cst_ctx* c, float* stage_ms, int32_t max_calls) {
    g_last_error.clear();
    if (c == nullptr) return -fail(CST_ERR_INVALID_ARG, "null context");
    if (ensure_device(c) != CST_OK) return -CST_ERR_CUDA;
    int n = 0;
    for (auto& ev : c->prof_calls) {
        if (cudaEventSynchronize(ev.back()) != cudaSuccess) return -fail(CST_ERR_CUDA, "event sync failed");
        if (stage_ms != nullptr && n < max_calls) {
            for (int st = 0; st < CST_N_STAGES; ++st) {
                float ms = 0.0f;
                cudaEventElapsedTime(&ms, ev[st], ev[st + 1]);
                stage_ms[n * CST_N_STAGES + st] = ms;
            }
            ++n;
        }
        for (auto e : ev) c->ev_pool.push_back(e);
    }
    c->prof_calls.clear();
    return n;
}

int cst_ctx_info(const cst_ctx* c, int64_t* out, int32_t n) {
    if (c == nullptr || out == nullptr) return 0;
    int resident = 0;
    for (int v : c->slot_of_expert) resident += v >= 0;
    const int64_t vals[] = {int64_t(c->cfg.n_slots) * c->geo.slot_bytes, c->geo.slot_bytes, int64_t(c->ws_bytes),
                            c->num_sms, resident, c->shared_slot,
                            static_cast<int64_t>(reinterpret_cast<uintptr_t>(c->arena))};
    const int m = std::min<int>(n, int(sizeof(vals) / sizeof(vals[0])));
    for (int i = 0; i < m; ++i) out[i] = vals[i];
    return m;
}

}  // extern "C"
