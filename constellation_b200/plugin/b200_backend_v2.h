// B200 backend of the reference expert node (expert_node_v2), over the constellation_b200
// C ABI: the backend registry's upload / free hooks and the request workspace.
//
// Reference interfaces implemented here:
//   BackendWorkspaceV2::RunExpertRequest      expert_node_v2/backend/backend_workspace_v2.h:11-29
//   UploadExpertFnV2 / FreeExpertWeightsFnV2  expert_node_v2/backend/backend_registry_v2.h:20-28
//   BackendRegistryEntryV2 (vendor Nvidia)    expert_node_v2/backend/backend_registry_v2.h:30-36
//   CreateBackendWorkspaceV2's role           expert_node_v2/backend/backend_workspace_v2.h:31-34
//
// Build inside the node's tree: include roots = the node repository's root and this
// repository's include/ and constellation_b200/plugin/; link with -lconstellation_b200
// -lcudart.  The node keeps its own GPU-info builders (build_static / build_dynamic of the
// CUDA backend) and passes them to B200RegistryEntryV2.
//
// Residency: the registry's upload hook is given no expert id -- the node's registry maps
// (expert_id, worker_id) to an ExpertDeviceStorageV2 itself (expert_registry_v2.cc:158-304)
// and passes the matching storage to RunExpertRequest (worker.cc:118-131).  This backend
// therefore keeps ONE expert arena per GPU (one cst_ctx of `slots` slots), puts each
// uploaded expert in a free slot and records the slot in the storage it fills: the storage's
// device pointers point into that slot of the arena (which holds the kernels' tile layout,
// not the row-major views of the CUDA backend).  A request runs on the slot of the storage
// the registry found, so experts of any number of layers share the arena and an expert is
// never looked up by a layer-local id.
#pragma once

#include <cstdint>
#include <memory>

#include "constellation_b200.h"
#include "expert_node_v2/backend/backend_registry_v2.h"
#include "expert_node_v2/backend/backend_workspace_v2.h"

namespace expert_node_v2 {

struct B200NodeConfigV2 {
    int hidden_dim = 7168;
    int inter_dim = 2048;
    int slots = 64;      // experts resident on this GPU, any layers (<= 1024)
    int max_batch = 64;  // rows per request (the CUDA backend serves batch 1 only)
};

// Creates GPU `local_gpu_id`'s arena and workspace (before the first upload to it).
// Returns false when the device cannot be used (no device, not sm_100, out of memory).
bool InitB200GpuV2(int local_gpu_id, const B200NodeConfigV2& cfg);
// Releases GPU `local_gpu_id`'s arena; every storage uploaded to it must be freed first.
void ShutdownB200GpuV2(int local_gpu_id);

// UploadExpertFnV2: validates the bundle with BuildExpertWeightsViewV2 (the node's own
// rules, expert_format_v2.cc:141-176), checks its shape against the GPU's config, and
// uploads it into a free arena slot.  On failure *out_storage is left empty.
bool UploadExpertB200V2(int local_gpu_id, const ExpertTensorBundleV2& host_bundle,
                        ExpertDeviceStorageV2* out_storage);
// FreeExpertWeightsFnV2: returns the storage's slot and resets the storage's handles (the
// DeviceBufferV2 destructors require it).
void FreeExpertWeightsB200V2(ExpertDeviceStorageV2* storage);

BackendRegistryEntryV2 B200RegistryEntryV2(BuildStaticGpuInfosFnV2 build_static,
                                           BuildDynamicGpuInfosFnV2 build_dynamic);

class BackendWorkspaceB200V2 final : public BackendWorkspaceV2 {
public:
    BackendWorkspaceB200V2(int local_gpu_id, const ExpertWorkspaceConfigV2& config);
    ~BackendWorkspaceB200V2() override;
    BackendWorkspaceB200V2(const BackendWorkspaceB200V2&) = delete;
    BackendWorkspaceB200V2& operator=(const BackendWorkspaceB200V2&) = delete;

    bool ok() const { return ok_; }

    // The request on the storage's expert: batch >= 1 (up to max_batch), fp16 / bf16 in
    // either pair, status 0 and the output on success.  Returns false (the worker then
    // answers status 4, worker.cc:126-130) for a storage that is not in this GPU's arena, a
    // malformed request or a device error -- the CUDA workspace's rules
    // (backend_workspace_cuda_v2.cc:139-181) without its batch_size == 1 limit.
    bool RunExpertRequest(const ExpertDeviceStorageV2& storage, const common::InferRequestMsg& req,
                          common::InferResponseMsg* resp) override;

private:
    int gpu_ = -1;
    bool ok_ = false;
    void* stream_ = nullptr;    // cudaStream_t
    void* d_in_ = nullptr;      // [max_batch, hidden] 16-bit rows
    void* d_out_ = nullptr;
    std::size_t cap_bytes_ = 0;
};

// The workspace for worker `worker_id` of the Nvidia span (local GPU = worker_id -
// span.worker_id_begin), as CreateBackendWorkspaceV2 builds one per worker thread.
std::unique_ptr<BackendWorkspaceV2> CreateBackendWorkspaceB200V2(const common::VendorWorkerSpan& vendor_span,
                                                                 int worker_id);

}  // namespace expert_node_v2
