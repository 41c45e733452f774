// C entry points over the reference node's own C++ expert code -- TEST INFRASTRUCTURE ONLY.
//
// Compiled (by oracle/Makefile) together with the reference's unmodified sources
//   expert_node_v2/expert_format_v2.cc, backend/fp8_lut_v2.cc,
//   backend/expert_reference_v2.cc, backend/dummy_expert_data_v2.cc,
//   backend/cpu/fused_up_gate_cpu_v2.cc, backend/cpu/down_cpu_v2.cc
// into oracle/_ref/libref_expert.so.  It lets Python call:
//   * FillDummyExpertBundleV2 / FillDummyInputActivationV2 (dummy_expert_data_v2.cc:9-150),
//     the reference's deterministic fixture;
//   * RunExpertReferenceV2 (expert_reference_v2.cc:146-176), the scalar oracle every
//     reference kernel test compares against;
//   * RunFusedUpGateCpuV2 + RunDownCpuV2 (cpu/fused_up_gate_cpu_v2.cc:12-178,
//     cpu/down_cpu_v2.cc:10-119), the reference's OpenMP CPU backend, which is the
//     timed CPU baseline (the thread count is passed explicitly instead of the
//     hard-coded 12 in backend_cpu_v2.cc:245-246);
//   * the activation codec (activation_codec_v2.h) and the FP8 LUT (fp8_lut_v2.cc);
//   * the node's InferRequest / InferResponse body codec (common/infer_codec.cc:7-76 over
//     common/protocol.cc), compiled from its sources too.
// Views are built over caller-owned memory, so nothing is copied per call.
#include <cstdint>
#include <cstring>
#include <span>
#include <vector>

#include "common/infer_codec.h"
#include "expert_node_v2/backend/activation_codec_v2.h"
#include "expert_node_v2/backend/cpu/down_cpu_v2.h"
#include "expert_node_v2/backend/cpu/fused_up_gate_cpu_v2.h"
#include "expert_node_v2/backend/dummy_expert_data_v2.h"
#include "expert_node_v2/backend/expert_reference_v2.h"
#include "expert_node_v2/backend/fp8_lut_v2.h"
#include "expert_node_v2/expert_format_v2.h"

namespace {

MatrixBlockScaleViewV2 make_view(const std::uint8_t* w, const float* s, int rows, int cols,
                                 int rblk, int cblk) {
    MatrixBlockScaleViewV2 v{};
    v.matrix.rows = rows;
    v.matrix.cols = cols;
    v.matrix.fp8_format = Fp8Format::TORCH_E4M3FN;
    v.weight.data = std::span<const std::uint8_t>(w, static_cast<std::size_t>(rows) * cols);
    v.scale_meta.row_block = rblk;
    v.scale_meta.col_block = cblk;
    v.scale_meta.num_row_blocks = ceil_div_int(rows, rblk);
    v.scale_meta.num_col_blocks = ceil_div_int(cols, cblk);
    v.scale.data = std::span<const float>(
        s, static_cast<std::size_t>(v.scale_meta.num_row_blocks) * v.scale_meta.num_col_blocks);
    return v;
}

ExpertWeightsViewV2 make_expert(const std::uint8_t* wu, const float* su, const std::uint8_t* wg,
                                const float* sg, const std::uint8_t* wd, const float* sd,
                                int inter, int hidden, int rblk, int cblk) {
    ExpertWeightsViewV2 e{};
    e.w_up = make_view(wu, su, inter, hidden, rblk, cblk);
    e.w_gate = make_view(wg, sg, inter, hidden, rblk, cblk);
    e.w_down = make_view(wd, sd, hidden, inter, rblk, cblk);
    return e;
}

void copy_tensor(const HostTensorV2& t, void* dst) {
    std::memcpy(dst, t.bytes.data(), t.bytes.size());
}

}  // namespace

extern "C" {

int ref_fill_dummy(int hidden, int inter, int rblk, int cblk, std::uint8_t* wu, float* su,
                   std::uint8_t* wg, float* sg, std::uint8_t* wd, float* sd) {
    ExpertTensorBundleV2 b;
    DummyExpertShapeV2 shape;
    shape.hidden_dim = hidden;
    shape.inter_dim = inter;
    shape.row_block = rblk;
    shape.col_block = cblk;
    FillDummyExpertBundleV2(&b, shape);
    copy_tensor(b.w_up, wu);
    copy_tensor(b.w_up_scale, su);
    copy_tensor(b.w_gate, wg);
    copy_tensor(b.w_gate_scale, sg);
    copy_tensor(b.w_down, wd);
    copy_tensor(b.w_down_scale, sd);
    ExpertWeightsViewV2 v;
    return BuildExpertWeightsViewV2(b, &v) ? 0 : 1;
}

void ref_dummy_input(int hidden, int dtype, float* x_float, std::uint16_t* x_encoded) {
    std::vector<float> f;
    std::vector<std::uint16_t> e;
    FillDummyInputActivationV2(hidden, static_cast<common::ActivationDType>(dtype), &f, &e);
    std::memcpy(x_float, f.data(), f.size() * sizeof(float));
    std::memcpy(x_encoded, e.data(), e.size() * sizeof(std::uint16_t));
}

// One batch-1 call of the reference scalar oracle; y gets `hidden` 16-bit words.
int ref_expert_reference(const std::uint8_t* wu, const float* su, const std::uint8_t* wg,
                         const float* sg, const std::uint8_t* wd, const float* sd, int inter,
                         int hidden, int rblk, int cblk, const std::uint16_t* x, int in_dtype,
                         int out_dtype, std::uint16_t* y, float* h_out) {
    const ExpertWeightsViewV2 e = make_expert(wu, su, wg, sg, wd, sd, inter, hidden, rblk, cblk);
    std::vector<std::uint8_t> yb;
    std::vector<float> h;
    if (!RunExpertReferenceV2(e, x, static_cast<common::ActivationDType>(in_dtype),
                              static_cast<common::ActivationDType>(out_dtype), &yb, &h)) {
        return 4;
    }
    std::memcpy(y, yb.data(), yb.size());
    if (h_out != nullptr) std::memcpy(h_out, h.data(), h.size() * sizeof(float));
    return 0;
}

// One batch-1 call of the reference OpenMP CPU backend; h_scratch holds `inter` floats.
int ref_expert_cpu(const std::uint8_t* wu, const float* su, const std::uint8_t* wg,
                   const float* sg, const std::uint8_t* wd, const float* sd, int inter,
                   int hidden, int rblk, int cblk, const std::uint16_t* x, int in_dtype,
                   std::uint16_t* y, int out_dtype, float* h_scratch, int threads) {
    const ExpertWeightsViewV2 e = make_expert(wu, su, wg, sg, wd, sd, inter, hidden, rblk, cblk);
    if (!RunFusedUpGateCpuV2(e.w_up, e.w_gate, x, static_cast<common::ActivationDType>(in_dtype),
                             h_scratch, threads)) {
        return 4;
    }
    if (!RunDownCpuV2(e.w_down, h_scratch, y, static_cast<common::ActivationDType>(out_dtype),
                      threads)) {
        return 4;
    }
    return 0;
}

float ref_decode_fp8(int fmt, int byte) {
    return DecodeFp8ByteV2(static_cast<Fp8Format>(fmt), static_cast<std::uint8_t>(byte));
}

std::uint16_t ref_encode_bf16(float x) { return EncodeFloatToBf16V2(x); }
std::uint16_t ref_encode_fp16(float x) { return EncodeFloatToFp16V2(x); }
float ref_decode_bf16(std::uint16_t b) { return DecodeBf16ToFloatV2(b); }
float ref_decode_fp16(std::uint16_t b) { return DecodeFp16ToFloatV2(b); }

// EncodeInferRequestBody: the body's length, or -1 if `cap` is short.
long long ref_encode_infer_request(std::int32_t expert_id, std::int32_t batch, std::int32_t hidden,
                                   std::uint32_t in_dtype, std::uint32_t out_dtype, const std::uint8_t* act,
                                   long long n, std::uint8_t* out, long long cap) {
    common::InferRequestMsg m;
    m.expert_id = expert_id;
    m.batch_size = batch;
    m.hidden_dim = hidden;
    m.input_dtype = static_cast<common::ActivationDType>(in_dtype);
    m.output_dtype = static_cast<common::ActivationDType>(out_dtype);
    m.activation.assign(reinterpret_cast<const char*>(act), static_cast<std::size_t>(n));
    const std::string body = common::EncodeInferRequestBody(m);
    if (static_cast<long long>(body.size()) > cap) return -1;
    std::memcpy(out, body.data(), body.size());
    return static_cast<long long>(body.size());
}

// DecodeInferRequestBody: 1 and the fields (expert, batch, hidden, in dtype, out dtype) and
// payload, or 0 when the reference rejects the body.
int ref_decode_infer_request(const std::uint8_t* body, long long len, long long* fields,
                             std::uint8_t* payload, long long cap, long long* n) {
    common::InferRequestMsg m;
    if (!common::DecodeInferRequestBody(std::string(reinterpret_cast<const char*>(body), len), &m)) return 0;
    fields[0] = m.expert_id;
    fields[1] = m.batch_size;
    fields[2] = m.hidden_dim;
    fields[3] = static_cast<long long>(m.input_dtype);
    fields[4] = static_cast<long long>(m.output_dtype);
    *n = static_cast<long long>(m.activation.size());
    if (*n > cap) return 0;
    std::memcpy(payload, m.activation.data(), m.activation.size());
    return 1;
}

long long ref_encode_infer_response(std::int32_t status, std::int32_t batch, std::int32_t hidden,
                                    std::uint32_t out_dtype, const std::uint8_t* output, long long n,
                                    std::uint8_t* out, long long cap) {
    common::InferResponseMsg m;
    m.status_code = status;
    m.batch_size = batch;
    m.hidden_dim = hidden;
    m.output_dtype = static_cast<common::ActivationDType>(out_dtype);
    m.output.assign(reinterpret_cast<const char*>(output), static_cast<std::size_t>(n));
    const std::string body = common::EncodeInferResponseBody(m);
    if (static_cast<long long>(body.size()) > cap) return -1;
    std::memcpy(out, body.data(), body.size());
    return static_cast<long long>(body.size());
}

// DecodeInferResponseBody: 1 and (status, batch, hidden, out dtype) + payload, or 0.
int ref_decode_infer_response(const std::uint8_t* body, long long len, long long* fields,
                              std::uint8_t* payload, long long cap, long long* n) {
    common::InferResponseMsg m;
    if (!common::DecodeInferResponseBody(std::string(reinterpret_cast<const char*>(body), len), &m)) return 0;
    fields[0] = m.status_code;
    fields[1] = m.batch_size;
    fields[2] = m.hidden_dim;
    fields[3] = static_cast<long long>(m.output_dtype);
    *n = static_cast<long long>(m.output.size());
    if (*n > cap) return 0;
    std::memcpy(payload, m.output.data(), m.output.size());
    return 1;
}

}  // extern "C"
