/*
 * TEST INFRASTRUCTURE ONLY — the CPU restatement ("oracle") of glm.c's
 * mixture-of-experts FFN hot path. Only tests/, __graft_entry__.smoke() and
 * bench.py's cpu_baseline / --impl reference legs may load it, and only as a
 * checker or a timed baseline; the product library never links it.
 *
 * Parity pin: this restatement is checked against glm.c's own code compiled
 * from its sources (oracle/ref_harness.c -> oracle/_ref/libglmref.so) on
 * seeded inputs, and against the golden fixtures in tests/golden/ that were
 * produced by that compiled reference (tests/golden/make_golden.py).
 *
 * Arithmetic contract (what must match the reference bit for bit):
 *  - rmsnorm sums x^2 in double, left to right (infer.c:746-752);
 *  - router logits are a left-to-right fp32 sum of separately rounded fp32
 *    products (dot_f32, infer.c:920-926) -- build with -ffp-contract=off;
 *  - sigmoid is 1/(1+expf(-l)) in fp32 (infer.c:1104-1107);
 *  - top-k keeps the K largest sel = p + bias, ties to the lower expert id,
 *    NaN and -inf never selected, stores unbiased p (infer.c:1110-1135);
 *  - weights are normalised by max(sum, 6.103515625e-5) (infer.c:1136-1145)
 *    and scaled by 1.8 when applied (infer.c:1171,1175).
 * The Q8 matvec inner sums are reassociated by the reference's `omp simd`
 * (infer.c:778-780), so expert outputs agree to rounding, not bit for bit.
 */
#include <math.h>
#include <stddef.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#include "moe_oracle.h"

/* infer.c:746-752 */
void orc_rmsnorm(float *out, const float *x, const float *w, int n) {
    double acc = 0.0;
    for (int i = 0; i < n; i++) acc += (double)x[i] * (double)x[i];
    const float mean_sq = (float)(acc / (double)n);
    const float scale = 1.0f / sqrtf(mean_sq + 1e-5f);
    for (int i = 0; i < n; i++) out[i] = x[i] * scale * w[i];
}

/* infer.c:765-786: y[r] = sum_g s[r,g] * (sum_{k<gs} q[r, g*gs+k] * x[g*gs+k]) */
void orc_matvec_q80(const int8_t *q, const float *s, const float *x, float *y,
                    int rows, int cols, int gs) {
    const int groups = cols / gs;
    for (int r = 0; r < rows; r++) {
        const int8_t *qr = q + (size_t)r * (size_t)cols;
        const float *sr = s + (size_t)r * (size_t)groups;
        float total = 0.0f;
        for (int g = 0; g < groups; g++) {
            float part = 0.0f;
            for (int k = 0; k < gs; k++) part += (float)qr[g * gs + k] * x[g * gs + k];
            total += sr[g] * part;
        }
        y[r] = total;
    }
}

/* infer.c:916-938 without CBLAS: one left-to-right fp32 dot per row. */
void orc_router_logits(const float *w, const float *xn, float *logits, int n_experts, int dim) {
    for (int e = 0; e < n_experts; e++) {
        const float *row = w + (size_t)e * (size_t)dim;
        float acc = 0.0f;
        for (int i = 0; i < dim; i++) {
            float prod = row[i] * xn[i];
            acc = acc + prod;
        }
        logits[e] = acc;
    }
}

float orc_sigmoid(float logit) { return 1.0f / (1.0f + expf(-logit)); }

float orc_silu(float v) { return v / (1.0f + expf(-v)); }

/* Selection of infer.c:1110-1135, restated as "K best by (sel desc, id asc)
 * among experts whose sel compares greater than -inf"; unused slots keep
 * id -1 / weight -1e30 as the reference leaves them. */
void orc_topk(const float *probs, const float *bias, int n_experts, int k_used,
              int32_t *idx, float *weight) {
    for (int k = 0; k < k_used; k++) {
        idx[k] = -1;
        weight[k] = -1e30f;
    }
    for (int k = 0; k < k_used; k++) {
        int best = -1;
        float best_sel = -INFINITY;
        for (int e = 0; e < n_experts; e++) {
            int taken = 0;
            for (int j = 0; j < k; j++) taken |= (idx[j] == e);
            if (taken) continue;
            const float sel = probs[e] + bias[e];
            if (sel > best_sel) { /* strict: first (lowest) id wins ties; NaN never wins */
                best_sel = sel;
                best = e;
            }
        }
        if (best < 0) break;
        idx[k] = best;
        weight[k] = probs[best];
    }
}

/* infer.c:1136-1145 */
void orc_normalize_topk(const int32_t *idx, float *weight, int k_used) {
    float sum = 0.0f;
    for (int k = 0; k < k_used; k++)
        if (idx[k] >= 0) sum += weight[k];
    if (sum > 0.0f) {
        const float floor_v = 6.103515625e-5f;
        const float inv = 1.0f / (sum < floor_v ? floor_v : sum);
        for (int k = 0; k < k_used; k++) weight[k] *= inv;
    }
}

/* One SwiGLU expert: out = down . (silu(gate . xn) * (up . xn)) */
static void swiglu_expert(const OrcQ8 *gate, const OrcQ8 *up, const OrcQ8 *down,
                          const float *xn, float *hid, float *tmp, float *out,
                          int dim, int ffn, int gs) {
    orc_matvec_q80(gate->q, gate->s, xn, hid, ffn, dim, gs);
    orc_matvec_q80(up->q, up->s, xn, tmp, ffn, dim, gs);
    for (int i = 0; i < ffn; i++) hid[i] = orc_silu(hid[i]) * tmp[i];
    orc_matvec_q80(down->q, down->s, hid, out, dim, ffn, gs);
}

/* infer.c:1087-1216 for one token; x is updated in place. */
int orc_moe_layer(const OrcMoeLayer *L, float *x, int32_t *topk_idx, float *topk_w, int routed_enabled) {
    const int D = L->dim, F = L->ffn, E = L->n_experts, K = L->k_used, gs = L->gs;
    float *xn = (float *)malloc(sizeof(float) * (size_t)D);
    float *probs = (float *)malloc(sizeof(float) * (size_t)E);
    float *hid = (float *)malloc(sizeof(float) * (size_t)F);
    float *tmp = (float *)malloc(sizeof(float) * (size_t)F);
    float *yk = (float *)malloc(sizeof(float) * (size_t)D);
    float *acc = (float *)calloc((size_t)D, sizeof(float));
    if (!xn || !probs || !hid || !tmp || !yk || !acc) {
        free(xn); free(probs); free(hid); free(tmp); free(yk); free(acc);
        return -1;
    }

    orc_rmsnorm(xn, x, L->ffn_norm, D);
    orc_router_logits(L->router, xn, probs, E, D);
    for (int e = 0; e < E; e++) probs[e] = orc_sigmoid(probs[e]);
    orc_topk(probs, L->router_bias, E, K, topk_idx, topk_w);
    orc_normalize_topk(topk_idx, topk_w, K);

    if (routed_enabled && L->routed_gate.q) {
        const size_t up_q = (size_t)F * D, up_s = (size_t)F * (D / gs);
        const size_t dn_q = (size_t)D * F, dn_s = (size_t)D * (F / gs);
        for (int k = 0; k < K; k++) {
            const int e = topk_idx[k];
            if (e < 0) continue;
            const float scale = topk_w[k] * 1.8f;
            OrcQ8 g = {L->routed_gate.q + e * up_q, L->routed_gate.s + e * up_s};
            OrcQ8 u = {L->routed_up.q + e * up_q, L->routed_up.s + e * up_s};
            OrcQ8 d = {L->routed_down.q + e * dn_q, L->routed_down.s + e * dn_s};
            swiglu_expert(&g, &u, &d, xn, hid, tmp, yk, D, F, gs);
            for (int i = 0; i < D; i++) acc[i] += scale * yk[i];
        }
    }
    swiglu_expert(&L->shared_gate, &L->shared_up, &L->shared_down, xn, hid, tmp, yk, D, F, gs);
    for (int i = 0; i < D; i++) x[i] += yk[i] + acc[i];

    free(xn); free(probs); free(hid); free(tmp); free(yk); free(acc);
    return 0;
}

/* Flat-pointer convenience wrapper for ctypes: same 15-pointer order as the
 * reference harness (LayerMoeShared then LayerMoeRouted fields). */
int orc_moe_layer_ptrs(int dim, int ffn, int n_experts, int k_used, int gs,
                       const void *const *p, int n_tokens, float *x,
                       int32_t *topk_idx, float *topk_w, int routed_enabled) {
    OrcMoeLayer L;
    L.dim = dim; L.ffn = ffn; L.n_experts = n_experts; L.k_used = k_used; L.gs = gs;
    L.ffn_norm = (const float *)p[0];
    L.router = (const float *)p[1];
    L.router_bias = (const float *)p[2];
    L.shared_gate.q = (const int8_t *)p[3]; L.shared_gate.s = (const float *)p[4];
    L.shared_up.q = (const int8_t *)p[5];   L.shared_up.s = (const float *)p[6];
    L.shared_down.q = (const int8_t *)p[7]; L.shared_down.s = (const float *)p[8];
    L.routed_gate.q = (const int8_t *)p[9];  L.routed_gate.s = (const float *)p[10];
    L.routed_up.q = (const int8_t *)p[11];   L.routed_up.s = (const float *)p[12];
    L.routed_down.q = (const int8_t *)p[13]; L.routed_down.s = (const float *)p[14];
    for (int t = 0; t < n_tokens; t++) {
        int rc = orc_moe_layer(&L, x + (size_t)t * dim, topk_idx + (size_t)t * k_used,
                               topk_w + (size_t)t * k_used, routed_enabled);
        if (rc) return rc;
    }
    return 0;
}
