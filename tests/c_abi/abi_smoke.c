/* A plain C (and C++) client of include/constellation_b200.h: checks that the header
 * compiles standalone, that the library links, and round-trips an expert-node request and
 * response body through the codec.  Touches no GPU; tests/test_c_abi.py builds and runs it. */
#include <stdint.h>
#include <stdio.h>
#include <string.h>

#include "constellation_b200.h"

static int fail(const char* what) {
    printf("FAIL %s: %s\n", what, cst_last_error());
    return 1;
}

int main(void) {
    if (cst_abi_version() < 100) return fail("abi version");
    uint8_t act[2 * 8];
    for (int i = 0; i < (int)sizeof(act); ++i) act[i] = (uint8_t)(3 * i + 1);
    cst_infer_request req;
    memset(&req, 0, sizeof(req));
    req.expert_id = 61 * 256 + 17;
    req.batch_size = 2;
    req.hidden_dim = 4;
    req.input_dtype = CST_DTYPE_BF16;
    req.output_dtype = CST_DTYPE_FP16;
    req.activation_bytes = sizeof(act);
    req.activation = act;
    uint8_t body[64];
    int64_t len = 0;
    if (cst_encode_infer_request(&req, body, sizeof(body), &len) != CST_OK) return fail("encode request");
    if (len != CST_INFER_REQUEST_FIXED_BYTES + (int64_t)sizeof(act)) return fail("request length");
    /* little-endian fixed fields */
    if (body[0] != ((61 * 256 + 17) & 0xff) || body[1] != ((61 * 256 + 17) >> 8) || body[20] != sizeof(act))
        return fail("request bytes");
    cst_infer_request back;
    if (cst_decode_infer_request(body, len, &back) != CST_OK) return fail("decode request");
    if (back.expert_id != req.expert_id || back.batch_size != 2 || back.hidden_dim != 4 ||
        back.input_dtype != CST_DTYPE_BF16 || back.output_dtype != CST_DTYPE_FP16 ||
        back.activation_bytes != sizeof(act) || memcmp(back.activation, act, sizeof(act)) != 0)
        return fail("request fields");
    if (cst_decode_infer_request(body, len - 1, &back) != CST_ERR_INVALID_ARG) return fail("short body accepted");

    /* an expert whose layer has no context here: status 1, echoed fields, no device use */
    uint8_t resp[64];
    int64_t n = 0;
    if (cst_serve_infer_request(NULL, 0, 256, body, len, resp, sizeof(resp), &n, NULL) != CST_OK)
        return fail("serve");
    cst_infer_response r;
    if (cst_decode_infer_response(resp, n, &r) != CST_OK) return fail("decode response");
    if (r.status_code != CST_ERR_UNKNOWN_EXPERT || r.batch_size != 2 || r.hidden_dim != 4 ||
        r.output_dtype != CST_DTYPE_FP16 || r.output_bytes != 0 || n != CST_INFER_RESPONSE_FIXED_BYTES)
        return fail("response fields");
    printf("OK\n");
    return 0;
}
