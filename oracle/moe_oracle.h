/* TEST INFRASTRUCTURE ONLY: CPU restatement of glm.c's MoE FFN hot path.
 * See moe_oracle.c for the reference citations and the arithmetic contract. */
#ifndef GLM_MOE_ORACLE_H
#define GLM_MOE_ORACLE_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct {
    const int8_t *q; /* int8 [rows][cols], row-major */
    const float *s;  /* fp32 [rows][cols/gs], row-major (planar scales) */
} OrcQ8;

typedef struct {
    int dim, ffn, n_experts, k_used, gs;
    const float *ffn_norm;    /* [dim] */
    const float *router;      /* [n_experts][dim] */
    const float *router_bias; /* [n_experts] */
    OrcQ8 shared_gate, shared_up, shared_down;
    OrcQ8 routed_gate, routed_up, routed_down; /* expert-major blocks */
} OrcMoeLayer;

void orc_rmsnorm(float *out, const float *x, const float *w, int n);
void orc_matvec_q80(const int8_t *q, const float *s, const float *x, float *y, int rows, int cols, int gs);
void orc_router_logits(const float *w, const float *xn, float *logits, int n_experts, int dim);
float orc_sigmoid(float logit);
float orc_silu(float v);
void orc_topk(const float *probs, const float *bias, int n_experts, int k_used, int32_t *idx, float *weight);
void orc_normalize_topk(const int32_t *idx, float *weight, int k_used);
int orc_moe_layer(const OrcMoeLayer *L, float *x, int32_t *topk_idx, float *topk_w, int routed_enabled);
int orc_moe_layer_ptrs(int dim, int ffn, int n_experts, int k_used, int gs, const void *const *p,
                       int n_tokens, float *x, int32_t *topk_idx, float *topk_w, int routed_enabled);

#ifdef __cplusplus
}
#endif

#endif
