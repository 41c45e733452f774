// Wire codec of the expert node's InferRequest / InferResponse bodies (host code only).
//
// The format is the reference's (common/infer_codec.cc:7-76 over the little-endian helpers of
// common/protocol.cc:13-80, mirrored by common/protocol.py:503-577 on the coordinator side):
//
//   request   i32 expert_id | i32 batch_size | i32 hidden_dim | u32 input_dtype |
//             u32 output_dtype | u32 n | n activation bytes
//   response  i32 status_code | i32 batch_size | i32 hidden_dim | u32 output_dtype |
//             u32 n | n output bytes
//
// A body decodes only if every field is present, the byte run fits, and nothing trails it.
// Fields are assembled from bytes, so the code does not depend on the host's byte order.
#include <cstdint>
#include <cstring>

#include "../../include/constellation_b200.h"
#include "kernels.h"

namespace cst {

namespace {

void put_u32(uint8_t* p, uint32_t v) {
    p[0] = uint8_t(v);
    p[1] = uint8_t(v >> 8);
    p[2] = uint8_t(v >> 16);
    p[3] = uint8_t(v >> 24);
}

uint32_t get_u32(const uint8_t* p) {
    return uint32_t(p[0]) | (uint32_t(p[1]) << 8) | (uint32_t(p[2]) << 16) | (uint32_t(p[3]) << 24);
}

// The five (request: six) fixed words, then the byte run whose length is the last word.
int decode_body(const uint8_t* body, int64_t len, int n_words, uint32_t* words, const uint8_t** run,
                const char* what) {
    if (len < 0 || (len > 0 && body == nullptr)) return set_last_error(CST_ERR_INVALID_ARG, "%s: bad buffer", what);
    if (len < int64_t(4) * n_words)
        return set_last_error(CST_ERR_INVALID_ARG, "%s: buffer too short while reading the fixed fields", what);
    for (int i = 0; i < n_words; ++i) words[i] = get_u32(body + 4 * i);
    const int64_t off = int64_t(4) * n_words;
    const int64_t n = words[n_words - 1];
    if (off + n > len) return set_last_error(CST_ERR_INVALID_ARG, "%s: buffer too short while reading the payload", what);
    if (off + n != len)
        return set_last_error(CST_ERR_INVALID_ARG, "%s has trailing bytes: parsed %lld, total %lld", what,
                              static_cast<long long>(off + n), static_cast<long long>(len));
    *run = body + off;
    return CST_OK;
}

int encode_body(const uint32_t* words, int n_words, const uint8_t* run, uint8_t* body, int64_t cap, int64_t* len,
                const char* what) {
    const int64_t n = words[n_words - 1];
    const int64_t need = int64_t(4) * n_words + n;
    if (len) *len = need;
    if (n > 0 && run == nullptr) return set_last_error(CST_ERR_INVALID_ARG, "%s: null payload", what);
    if (body == nullptr || cap < need)
        return set_last_error(CST_ERR_INVALID_ARG, "%s needs %lld bytes, buffer holds %lld", what,
                              static_cast<long long>(need), static_cast<long long>(body ? cap : 0));
    for (int i = 0; i < n_words; ++i) put_u32(body + 4 * i, words[i]);
    if (n > 0) std::memmove(body + 4 * n_words, run, size_t(n));
    return CST_OK;
}

}  // namespace

void put_infer_response_fixed(uint8_t* body, int32_t status, int32_t batch, int32_t hidden, uint32_t out_dtype,
                              uint32_t nbytes) {
    put_u32(body + 0, uint32_t(status));
    put_u32(body + 4, uint32_t(batch));
    put_u32(body + 8, uint32_t(hidden));
    put_u32(body + 12, out_dtype);
    put_u32(body + 16, nbytes);
}

}  // namespace cst

using namespace cst;

extern "C" int cst_encode_infer_request(const cst_infer_request* m, uint8_t* body, int64_t cap, int64_t* len) {
    clear_last_error();
    if (m == nullptr) return set_last_error(CST_ERR_INVALID_ARG, "null request");
    const uint32_t w[6] = {uint32_t(m->expert_id), uint32_t(m->batch_size), uint32_t(m->hidden_dim),
                           m->input_dtype,         m->output_dtype,         m->activation_bytes};
    return encode_body(w, 6, m->activation, body, cap, len, "infer_request");
}

extern "C" int cst_decode_infer_request(const uint8_t* body, int64_t len, cst_infer_request* out) {
    clear_last_error();
    if (out == nullptr) return set_last_error(CST_ERR_INVALID_ARG, "null output");
    uint32_t w[6];
    const uint8_t* run = nullptr;
    if (int rc = decode_body(body, len, 6, w, &run, "infer_request")) return rc;
    out->expert_id = int32_t(w[0]);
    out->batch_size = int32_t(w[1]);
    out->hidden_dim = int32_t(w[2]);
    out->input_dtype = w[3];
    out->output_dtype = w[4];
    out->activation_bytes = w[5];
    out->activation = run;
    return CST_OK;
}

extern "C" int cst_encode_infer_response(const cst_infer_response* m, uint8_t* body, int64_t cap, int64_t* len) {
    clear_last_error();
    if (m == nullptr) return set_last_error(CST_ERR_INVALID_ARG, "null response");
    const uint32_t w[5] = {uint32_t(m->status_code), uint32_t(m->batch_size), uint32_t(m->hidden_dim),
                           m->output_dtype, m->output_bytes};
    return encode_body(w, 5, m->output, body, cap, len, "infer_response");
}

extern "C" int cst_decode_infer_response(const uint8_t* body, int64_t len, cst_infer_response* out) {
    clear_last_error();
    if (out == nullptr) return set_last_error(CST_ERR_INVALID_ARG, "null output");
    uint32_t w[5];
    const uint8_t* run = nullptr;
    if (int rc = decode_body(body, len, 5, w, &run, "infer_response")) return rc;
    out->status_code = int32_t(w[0]);
    out->batch_size = int32_t(w[1]);
    out->hidden_dim = int32_t(w[2]);
    out->output_dtype = w[3];
    out->output_bytes = w[4];
    out->output = run;
    return CST_OK;
}
