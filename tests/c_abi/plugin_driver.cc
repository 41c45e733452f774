// Drives the B200 expert-node backend (constellation_b200/plugin) through the reference
// node's own interfaces: the registry hooks and BackendWorkspaceV2::RunExpertRequest.
//   plugin_driver cpu        status-only paths (no GPU needed); prints "cpu-ok"
//   plugin_driver gpu DIR    uploads the experts in DIR, serves requests, writes outputs
// Used by tests/test_expert_node_plugin.py.
#include <cstdio>
#include <cstring>
#include <fstream>
#include <iterator>
#include <memory>
#include <string>
#include <vector>

#include "b200_backend_v2.h"

using namespace expert_node_v2;

namespace {

int g_fail = 0;
#define CHECK(cond)                                                        \
    do {                                                                   \
        if (!(cond)) {                                                     \
            std::printf("FAIL %s:%d %s\n", __FILE__, __LINE__, #cond);      \
            ++g_fail;                                                      \
        }                                                                  \
    } while (0)

std::vector<std::uint8_t> read_file(const std::string& p) {
    std::ifstream f(p, std::ios::binary);
    return std::vector<std::uint8_t>((std::istreambuf_iterator<char>(f)), std::istreambuf_iterator<char>());
}

void write_file(const std::string& p, const std::string& bytes) {
    std::ofstream f(p, std::ios::binary);
    f.write(bytes.data(), static_cast<std::streamsize>(bytes.size()));
}

void set_tensor(HostTensorV2* t, std::vector<std::uint8_t> bytes, std::uint64_t d0, std::uint64_t d1,
                const char* dtype) {
    t->bytes = std::move(bytes);
    t->meta.shape = {d0, d1};
    t->meta.dtype = dtype;
    t->meta.row_block = 128;
    t->meta.col_block = 128;
    t->ready = true;
}

// The six tensors of expert `e` as the node receives them (LoadWeights messages).
void load_bundle(const std::string& dir, int e, int H, int I, ExpertTensorBundleV2* b) {
    const std::string p = dir + "/e" + std::to_string(e) + "_";
    const std::uint64_t gi = (I + 127) / 128, gh = (H + 127) / 128;
    set_tensor(&b->w_up, read_file(p + "w_up.bin"), I, H, "float8_e4m3fn");
    set_tensor(&b->w_up_scale, read_file(p + "s_up.bin"), gi, gh, "float32");
    set_tensor(&b->w_gate, read_file(p + "w_gate.bin"), I, H, "float8_e4m3fn");
    set_tensor(&b->w_gate_scale, read_file(p + "s_gate.bin"), gi, gh, "float32");
    set_tensor(&b->w_down, read_file(p + "w_down.bin"), H, I, "float8_e4m3fn");
    set_tensor(&b->w_down_scale, read_file(p + "s_down.bin"), gh, gi, "float32");
}

common::InferRequestMsg request(const std::string& dir, const char* name, int batch, int H,
                                common::ActivationDType in, common::ActivationDType out) {
    common::InferRequestMsg r;
    r.expert_id = 0;  // the registry's key; the backend runs the storage it is handed
    r.batch_size = batch;
    r.hidden_dim = H;
    r.input_dtype = in;
    r.output_dtype = out;
    const auto x = read_file(dir + "/" + name);
    r.activation.assign(x.begin(), x.end());
    return r;
}

int run_cpu() {
    B200NodeConfigV2 cfg;
    // no device here: the arena cannot be created, and nothing else may succeed
    CHECK(!InitB200GpuV2(0, cfg));
    CHECK(!InitB200GpuV2(-1, cfg));
    ExpertTensorBundleV2 b;  // nothing ready
    {
        ExpertDeviceStorageV2 st;
        CHECK(!UploadExpertB200V2(0, b, &st));
        CHECK(st.w_up_weight.data == nullptr && st.w_up_weight.size == 0);
        FreeExpertWeightsB200V2(&st);  // an empty storage frees to empty
    }  // no leak abort from DeviceBufferV2
    CHECK(!UploadExpertB200V2(0, b, nullptr));
    BackendWorkspaceB200V2 ws(0, ExpertWorkspaceConfigV2{7168, 2048});
    CHECK(!ws.ok());
    ExpertDeviceStorageV2 st;
    common::InferRequestMsg req;
    req.batch_size = 1;
    req.hidden_dim = 7168;
    req.input_dtype = req.output_dtype = common::ActivationDType::BF16;
    req.activation.assign(7168 * 2, '\0');
    common::InferResponseMsg resp;
    CHECK(!ws.RunExpertRequest(st, req, &resp));  // the worker answers status 4
    common::VendorWorkerSpan span{0, 1};
    CHECK(CreateBackendWorkspaceB200V2(span, 0) == nullptr);
    const BackendRegistryEntryV2 e = B200RegistryEntryV2(nullptr, nullptr);
    CHECK(e.vendor == common::GpuVendor::Nvidia);
    CHECK(e.upload_expert == &UploadExpertB200V2 && e.free_expert_weights == &FreeExpertWeightsB200V2);
    if (g_fail == 0) std::printf("cpu-ok\n");
    return g_fail == 0 ? 0 : 1;
}

void serve(BackendWorkspaceV2& ws, const ExpertDeviceStorageV2& st, const common::InferRequestMsg& req,
           const std::string& out_path, const char* tag) {
    common::InferResponseMsg resp;
    resp.status_code = 4;
    const bool ok = ws.RunExpertRequest(st, req, &resp);
    std::printf("%s ok=%d status=%d batch=%d hidden=%d dtype=%u bytes=%zu\n", tag, int(ok), resp.status_code,
                resp.batch_size, resp.hidden_dim, static_cast<unsigned>(resp.output_dtype), resp.output.size());
    if (ok) write_file(out_path, resp.output);
}

int run_gpu(const std::string& dir) {
    const int H = 256, I = 128;
    B200NodeConfigV2 cfg;
    cfg.hidden_dim = H;
    cfg.inter_dim = I;
    cfg.slots = 2;
    cfg.max_batch = 8;
    CHECK(InitB200GpuV2(0, cfg));
    CHECK(!InitB200GpuV2(0, cfg));  // once per GPU
    const BackendRegistryEntryV2 reg = B200RegistryEntryV2(nullptr, nullptr);
    ExpertTensorBundleV2 b0, b1;
    load_bundle(dir, 0, H, I, &b0);
    load_bundle(dir, 1, H, I, &b1);
    ExpertDeviceStorageV2 sa, sb, sc;
    CHECK(reg.upload_expert(0, b0, &sa));
    CHECK(reg.upload_expert(0, b1, &sb));
    CHECK(!reg.upload_expert(0, b1, &sc));  // both slots in use
    CHECK(sc.w_up_weight.data == nullptr);
    CHECK(sa.w_up_meta.rows == I && sa.w_up_meta.cols == H && sa.w_down_meta.rows == H);
    CHECK(sa.w_up_scale_meta.num_row_blocks == I / 128 && sa.w_up_scale_meta.num_col_blocks == H / 128);
    ExpertTensorBundleV2 bad;
    load_bundle(dir, 0, H, I, &bad);
    bad.w_down_scale.meta.dtype = "bfloat16";
    CHECK(!reg.upload_expert(0, bad, &sc));

    common::VendorWorkerSpan span{3, 1};  // worker 3 = the first Nvidia worker = GPU 0
    std::unique_ptr<BackendWorkspaceV2> ws = CreateBackendWorkspaceB200V2(span, 3);
    CHECK(ws != nullptr);
    if (!ws) return 1;
    using D = common::ActivationDType;
    serve(*ws, sa, request(dir, "x3_bf16.bin", 3, H, D::BF16, D::BF16), dir + "/out1.bin", "req1");
    serve(*ws, sb, request(dir, "x1_fp16.bin", 1, H, D::FP16, D::BF16), dir + "/out2.bin", "req2");
    serve(*ws, sb, request(dir, "x5_bf16.bin", 5, H, D::BF16, D::FP16), dir + "/out3.bin", "req3");
    // replacement, as ExpertRegistryV2::Update does it: free, then upload into the storage
    reg.free_expert_weights(&sa);
    CHECK(sa.w_up_weight.data == nullptr && sa.w_up_meta.rows == 0);
    CHECK(reg.upload_expert(0, b1, &sa));
    serve(*ws, sa, request(dir, "x3_bf16.bin", 3, H, D::BF16, D::BF16), dir + "/out4.bin", "req4");
    // malformed requests and a storage this backend did not fill
    serve(*ws, sa, request(dir, "x3_bf16.bin", 2, H, D::BF16, D::BF16), dir + "/bad.bin", "bad_bytes");
    serve(*ws, sa, request(dir, "x3_bf16.bin", 3, H, D::Unknown, D::BF16), dir + "/bad.bin", "bad_dtype");
    common::InferRequestMsg big = request(dir, "x3_bf16.bin", 9, H, D::BF16, D::BF16);
    big.activation.assign(std::size_t(9) * H * 2, '\0');
    serve(*ws, sa, big, dir + "/bad.bin", "bad_batch");
    ExpertDeviceStorageV2 foreign;
    serve(*ws, foreign, request(dir, "x3_bf16.bin", 3, H, D::BF16, D::BF16), dir + "/bad.bin", "foreign");
    reg.free_expert_weights(&sa);
    reg.free_expert_weights(&sb);
    ws.reset();
    ShutdownB200GpuV2(0);
    std::printf("gpu-done fails=%d\n", g_fail);
    return g_fail == 0 ? 0 : 1;
}

}  // namespace

int main(int argc, char** argv) {
    if (argc >= 2 && std::strcmp(argv[1], "cpu") == 0) return run_cpu();
    if (argc >= 3 && std::strcmp(argv[1], "gpu") == 0) return run_gpu(argv[2]);
    std::printf("usage: plugin_driver cpu | gpu DIR\n");
    return 2;
}
