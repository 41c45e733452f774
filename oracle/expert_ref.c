/*
 * Scalar FP8 block-scaled SwiGLU expert in plain C -- CPU ORACLE, TEST INFRASTRUCTURE ONLY.
 *
 * Restates the reference node's scalar oracle:
 *   - RunFusedUpGateReferenceV2  expert_node_v2/backend/expert_reference_v2.cc:11-90
 *       h[r] = silu(sum_k LUT[Wg[r,k]] * Sg[r/rb, k/cb] * x[k]) * sum_k LUT[Wu[r,k]] * Su[..] * x[k]
 *       fp32 running sums in k order, silu(g) = g / (1 + exp(-g))           (:85)
 *   - RunDownReferenceV2         expert_reference_v2.cc:92-144
 *       y[r] = sum_k LUT[Wd[r,k]] * Sd[r/rb, k/cb] * h[k]
 *   - the LUT of fp8_lut_v2.cc:47-66 (torch e4m3fn with 0x7F/0xFF -> +-448).
 * Ragged blocks (rows/cols not multiples of the block) follow the reference's
 * ceil-div scale grids.  Tokens are independent: the n input rows are processed
 * one after the other exactly like n batch-1 calls.
 *
 * Only tests/, the smoke check and bench.py's CPU-baseline leg load this file's
 * shared library (oracle/_ref/libexpert_oracle.so, built by oracle/refbuild.py).
 */
#include <math.h>
#include <stddef.h>
#include <stdint.h>

static float g_lut[256];
static int g_lut_ready = 0;

static float decode_e4m3fn_ref(uint8_t v) {
    const int sign = (v >> 7) & 1;
    const int e = (v >> 3) & 0xF;
    const int m = v & 7;
    const float s = sign ? -1.0f : 1.0f;
    if (e == 0) return s * ldexpf((float)m / 8.0f, -6);
    if (e == 0xF && m == 7) return s * 448.0f;
    return s * ldexpf(1.0f + (float)m / 8.0f, e - 7);
}

static void build_lut(void) {
    if (g_lut_ready) return;
    for (int i = 0; i < 256; ++i) g_lut[i] = decode_e4m3fn_ref((uint8_t)i);
    g_lut_ready = 1;
}

float oracle_decode_e4m3fn_ref(int byte) {
    build_lut();
    return g_lut[byte & 0xFF];
}

/* x: [n, H] fp32 (already decoded activations); h_out: [n, I]; y_out: [n, H] (fp32, pre-encode). */
int oracle_expert_lut(const uint8_t* wu, const float* su, const uint8_t* wg, const float* sg,
                      const uint8_t* wd, const float* sd, int inter, int hidden, int rblk, int cblk,
                      const float* x, int n, float* h_out, float* y_out) {
    if (!wu || !su || !wg || !sg || !wd || !sd || !x || !h_out || !y_out) return 3;
    if (inter <= 0 || hidden <= 0 || rblk <= 0 || cblk <= 0 || n < 0) return 3;
    build_lut();
    const int up_ncb = (hidden + cblk - 1) / cblk;
    const int dn_ncb = (inter + cblk - 1) / cblk;
    for (int t = 0; t < n; ++t) {
        const float* xt = x + (size_t)t * hidden;
        float* ht = h_out + (size_t)t * inter;
        float* yt = y_out + (size_t)t * hidden;
        for (int r = 0; r < inter; ++r) {
            const int rb = r / rblk;
            float up = 0.0f, gate = 0.0f;
            for (int k = 0; k < hidden; ++k) {
                const size_t wi = (size_t)r * hidden + k;
                const size_t si = (size_t)rb * up_ncb + (size_t)(k / cblk);
                const float xv = xt[k];
                up += (g_lut[wu[wi]] * su[si]) * xv;
                gate += (g_lut[wg[wi]] * sg[si]) * xv;
            }
            const float silu = gate / (1.0f + expf(-gate));
            ht[r] = silu * up;
        }
        for (int r = 0; r < hidden; ++r) {
            const int rb = r / rblk;
            float acc = 0.0f;
            for (int k = 0; k < inter; ++k) {
                const size_t wi = (size_t)r * inter + k;
                const size_t si = (size_t)rb * dn_ncb + (size_t)(k / cblk);
                acc += (g_lut[wd[wi]] * sd[si]) * ht[k];
            }
            yt[r] = acc;
        }
    }
    return 0;
}
