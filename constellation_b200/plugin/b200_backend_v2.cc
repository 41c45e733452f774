// B200 backend of the reference expert node over the constellation_b200 C ABI (see the
// header for the interfaces it implements and how residency is kept).
#include "b200_backend_v2.h"

#include <cuda_runtime.h>

#include <array>
#include <cstdio>
#include <mutex>
#include <vector>

namespace expert_node_v2 {
namespace {

constexpr int kMaxGpus = 64;

struct GpuNode {
    cst_ctx* ctx = nullptr;
    B200NodeConfigV2 cfg{};
    std::uintptr_t arena = 0;   // device address of slot 0
    std::int64_t slot_bytes = 0;
    std::vector<int> free_slots;
};

std::mutex g_mu;
std::array<GpuNode, kMaxGpus> g_nodes;

// Slot of an arena address of GPU `gpu`, or -1.  Caller holds g_mu.
int slot_of(const GpuNode& n, const void* p) {
    const std::uintptr_t a = reinterpret_cast<std::uintptr_t>(p);
    if (n.ctx == nullptr || a < n.arena) return -1;
    const std::uintptr_t off = a - n.arena;
    if (off % static_cast<std::uintptr_t>(n.slot_bytes) != 0) return -1;
    const std::uintptr_t slot = off / static_cast<std::uintptr_t>(n.slot_bytes);
    return slot < static_cast<std::uintptr_t>(n.cfg.slots) ? static_cast<int>(slot) : -1;
}

void reset_storage(ExpertDeviceStorageV2* s) {
    s->w_up_weight.data = nullptr;
    s->w_up_weight.size = 0;
    s->w_up_scale.data = nullptr;
    s->w_up_scale.size = 0;
    s->w_gate_weight.data = nullptr;
    s->w_gate_weight.size = 0;
    s->w_gate_scale.data = nullptr;
    s->w_gate_scale.size = 0;
    s->w_down_weight.data = nullptr;
    s->w_down_weight.size = 0;
    s->w_down_scale.data = nullptr;
    s->w_down_scale.size = 0;
    s->w_up_meta = MatrixMetaV2{};
    s->w_gate_meta = MatrixMetaV2{};
    s->w_down_meta = MatrixMetaV2{};
    s->w_up_scale_meta = BlockScaleMetaV2{};
    s->w_gate_scale_meta = BlockScaleMetaV2{};
    s->w_down_scale_meta = BlockScaleMetaV2{};
}

}  // namespace

bool InitB200GpuV2(int local_gpu_id, const B200NodeConfigV2& cfg) {
    if (local_gpu_id < 0 || local_gpu_id >= kMaxGpus) return false;
    if (cfg.slots < 1 || cfg.slots > 1024 || cfg.max_batch < 1) return false;
    std::lock_guard<std::mutex> lock(g_mu);
    GpuNode& n = g_nodes[local_gpu_id];
    if (n.ctx != nullptr) return false;
    // A private router width: expert id == slot.  Requests never route; they name a slot.
    cst_config c{};
    c.hidden_dim = cfg.hidden_dim;
    c.inter_dim = cfg.inter_dim;
    c.n_routed_experts = cfg.slots;
    c.n_group = 1;
    c.topk_group = 1;
    c.top_k = 1;
    c.norm_topk_prob = 1;
    c.routed_scaling_factor = 1.0f;
    c.block_size = 128;
    c.n_slots = cfg.slots;
    c.max_tokens = cfg.max_batch;
    c.max_rows = cfg.max_batch;
    cst_ctx* ctx = nullptr;
    if (cst_create(local_gpu_id, &c, &ctx) != CST_OK) {
        std::fprintf(stderr, "[b200_backend] InitB200GpuV2(%d): %s\n", local_gpu_id, cst_last_error());
        return false;
    }
    std::int64_t info[7] = {};
    if (cst_ctx_info(ctx, info, 7) < 7 || info[6] == 0) {
        cst_destroy(ctx);
        return false;
    }
    n.ctx = ctx;
    n.cfg = cfg;
    n.slot_bytes = info[1];
    n.arena = static_cast<std::uintptr_t>(info[6]);
    n.free_slots.clear();
    for (int s = cfg.slots - 1; s >= 0; --s) n.free_slots.push_back(s);
    return true;
}

void ShutdownB200GpuV2(int local_gpu_id) {
    if (local_gpu_id < 0 || local_gpu_id >= kMaxGpus) return;
    std::lock_guard<std::mutex> lock(g_mu);
    GpuNode& n = g_nodes[local_gpu_id];
    if (n.ctx != nullptr) cst_destroy(n.ctx);
    n = GpuNode{};
}

bool UploadExpertB200V2(int local_gpu_id, const ExpertTensorBundleV2& host_bundle,
                        ExpertDeviceStorageV2* out_storage) {
    if (out_storage == nullptr) return false;
    reset_storage(out_storage);
    if (local_gpu_id < 0 || local_gpu_id >= kMaxGpus) return false;
    ExpertWeightsViewV2 v;
    if (!BuildExpertWeightsViewV2(host_bundle, &v)) {
        std::fprintf(stderr, "[b200_backend] upload: the bundle fails BuildExpertWeightsViewV2\n");
        return false;
    }
    std::lock_guard<std::mutex> lock(g_mu);
    GpuNode& n = g_nodes[local_gpu_id];
    if (n.ctx == nullptr) return false;
    if (v.w_up.matrix.rows != n.cfg.inter_dim || v.w_up.matrix.cols != n.cfg.hidden_dim) return false;
    if (n.free_slots.empty()) {
        std::fprintf(stderr, "[b200_backend] upload: all %d slots of GPU %d are in use\n", n.cfg.slots,
                     local_gpu_id);
        return false;
    }
    const int slot = n.free_slots.back();
    cst_expert_weights w{};
    w.w_up = v.w_up.weight.data.data();
    w.w_up_scale = v.w_up.scale.data.data();
    w.w_gate = v.w_gate.weight.data.data();
    w.w_gate_scale = v.w_gate.scale.data.data();
    w.w_down = v.w_down.weight.data.data();
    w.w_down_scale = v.w_down.scale.data.data();
    w.rows = v.w_up.matrix.rows;
    w.cols = v.w_up.matrix.cols;
    w.row_block = v.w_up.scale_meta.row_block;
    w.col_block = v.w_up.scale_meta.col_block;
    if (cst_upload_expert(n.ctx, slot, slot, &w, nullptr) != CST_OK) {
        std::fprintf(stderr, "[b200_backend] upload: %s\n", cst_last_error());
        return false;
    }
    n.free_slots.pop_back();
    // handles: addresses inside the slot (its first byte identifies it), sizes in elements
    std::uint8_t* base = reinterpret_cast<std::uint8_t*>(n.arena + std::uintptr_t(slot) * n.slot_bytes);
    const std::size_t mat = std::size_t(w.rows) * std::size_t(w.cols);
    const std::size_t grid = v.w_up.scale.data.size();
    out_storage->w_up_meta = v.w_up.matrix;
    out_storage->w_gate_meta = v.w_gate.matrix;
    out_storage->w_down_meta = v.w_down.matrix;
    out_storage->w_up_scale_meta = v.w_up.scale_meta;
    out_storage->w_gate_scale_meta = v.w_gate.scale_meta;
    out_storage->w_down_scale_meta = v.w_down.scale_meta;
    out_storage->w_up_weight.data = base;
    out_storage->w_up_weight.size = mat;
    out_storage->w_gate_weight.data = base + mat;
    out_storage->w_gate_weight.size = mat;
    out_storage->w_down_weight.data = base + 2 * mat;
    out_storage->w_down_weight.size = mat;
    float* sbase = reinterpret_cast<float*>(base + 3 * mat);
    out_storage->w_up_scale.data = sbase;
    out_storage->w_up_scale.size = grid;
    out_storage->w_gate_scale.data = sbase + grid;
    out_storage->w_gate_scale.size = grid;
    out_storage->w_down_scale.data = sbase + 2 * grid;
    out_storage->w_down_scale.size = v.w_down.scale.data.size();
    return true;
}

void FreeExpertWeightsB200V2(ExpertDeviceStorageV2* storage) {
    if (storage == nullptr) return;
    {
        std::lock_guard<std::mutex> lock(g_mu);
        for (int g = 0; g < kMaxGpus && storage->w_up_weight.data != nullptr; ++g) {
            GpuNode& n = g_nodes[g];
            const int slot = slot_of(n, storage->w_up_weight.data);
            if (slot < 0) continue;
            if (cst_free_expert(n.ctx, slot) == CST_OK) n.free_slots.push_back(slot);
            break;
        }
    }
    reset_storage(storage);
}

BackendRegistryEntryV2 B200RegistryEntryV2(BuildStaticGpuInfosFnV2 build_static,
                                           BuildDynamicGpuInfosFnV2 build_dynamic) {
    BackendRegistryEntryV2 e{};
    e.vendor = common::GpuVendor::Nvidia;
    e.build_static = build_static;
    e.build_dynamic = build_dynamic;
    e.upload_expert = &UploadExpertB200V2;
    e.free_expert_weights = &FreeExpertWeightsB200V2;
    return e;
}

BackendWorkspaceB200V2::BackendWorkspaceB200V2(int local_gpu_id, const ExpertWorkspaceConfigV2& config)
    : BackendWorkspaceV2(config), gpu_(local_gpu_id) {
    if (local_gpu_id < 0 || local_gpu_id >= kMaxGpus) return;
    B200NodeConfigV2 cfg;
    {
        std::lock_guard<std::mutex> lock(g_mu);
        const GpuNode& n = g_nodes[local_gpu_id];
        if (n.ctx == nullptr) return;
        cfg = n.cfg;
    }
    if (config.hidden_dim != cfg.hidden_dim || config.inter_dim != cfg.inter_dim) return;
    if (cudaSetDevice(local_gpu_id) != cudaSuccess) return;
    cap_bytes_ = std::size_t(cfg.max_batch) * std::size_t(cfg.hidden_dim) * 2;
    cudaStream_t s = nullptr;
    if (cudaStreamCreateWithFlags(&s, cudaStreamNonBlocking) != cudaSuccess) return;
    stream_ = s;
    if (cudaMalloc(&d_in_, cap_bytes_) != cudaSuccess || cudaMalloc(&d_out_, cap_bytes_) != cudaSuccess) return;
    ok_ = true;
}

BackendWorkspaceB200V2::~BackendWorkspaceB200V2() {
    if (gpu_ >= 0 && (d_in_ || d_out_ || stream_)) cudaSetDevice(gpu_);
    if (stream_) cudaStreamSynchronize(static_cast<cudaStream_t>(stream_));
    if (d_in_) cudaFree(d_in_);
    if (d_out_) cudaFree(d_out_);
    if (stream_) cudaStreamDestroy(static_cast<cudaStream_t>(stream_));
}

bool BackendWorkspaceB200V2::RunExpertRequest(const ExpertDeviceStorageV2& storage,
                                              const common::InferRequestMsg& req,
                                              common::InferResponseMsg* resp) {
    if (!ok_ || resp == nullptr) return false;
    if (req.hidden_dim != config_.hidden_dim || req.batch_size < 1) return false;
    const auto code = [](common::ActivationDType d) {
        return d == common::ActivationDType::FP16 ? CST_DTYPE_FP16
               : d == common::ActivationDType::BF16 ? CST_DTYPE_BF16 : 0;
    };
    const int in_dt = code(req.input_dtype), out_dt = code(req.output_dtype);
    if (in_dt == 0 || out_dt == 0) return false;
    const std::size_t bytes = std::size_t(req.batch_size) * std::size_t(req.hidden_dim) * 2;
    if (req.activation.size() != bytes || bytes > cap_bytes_) return false;
    cst_ctx* ctx = nullptr;
    int slot = -1;
    {
        std::lock_guard<std::mutex> lock(g_mu);
        const GpuNode& n = g_nodes[gpu_];
        slot = slot_of(n, storage.w_up_weight.data);
        ctx = n.ctx;
    }
    if (slot < 0 || ctx == nullptr) return false;
    if (cudaSetDevice(gpu_) != cudaSuccess) return false;
    cudaStream_t s = static_cast<cudaStream_t>(stream_);
    if (cudaMemcpyAsync(d_in_, req.activation.data(), bytes, cudaMemcpyHostToDevice, s) != cudaSuccess) return false;
    if (cst_expert_forward(ctx, slot, d_in_, in_dt, req.batch_size, d_out_, out_dt, s) != CST_OK) {
        cudaStreamSynchronize(s);
        return false;
    }
    resp->output.resize(bytes);
    if (cudaMemcpyAsync(resp->output.data(), d_out_, bytes, cudaMemcpyDeviceToHost, s) != cudaSuccess ||
        cudaStreamSynchronize(s) != cudaSuccess) {
        resp->output.clear();
        return false;
    }
    resp->status_code = 0;
    resp->batch_size = req.batch_size;
    resp->hidden_dim = req.hidden_dim;
    resp->output_dtype = req.output_dtype;
    return true;
}

std::unique_ptr<BackendWorkspaceV2> CreateBackendWorkspaceB200V2(const common::VendorWorkerSpan& vendor_span,
                                                                 int worker_id) {
    const int gpu = worker_id - vendor_span.worker_id_begin;
    if (gpu < 0 || gpu >= kMaxGpus || worker_id >= vendor_span.worker_id_begin + vendor_span.worker_count)
        return nullptr;
    ExpertWorkspaceConfigV2 cfg;
    {
        std::lock_guard<std::mutex> lock(g_mu);
        const GpuNode& n = g_nodes[gpu];
        if (n.ctx == nullptr) return nullptr;
        cfg.hidden_dim = n.cfg.hidden_dim;
        cfg.inter_dim = n.cfg.inter_dim;
    }
    auto ws = std::make_unique<BackendWorkspaceB200V2>(gpu, cfg);
    if (!ws->ok()) return nullptr;
    return ws;
}

}  // namespace expert_node_v2
