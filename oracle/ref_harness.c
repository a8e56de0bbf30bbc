/*
 * TEST INFRASTRUCTURE ONLY — never linked into the product library.
 *
 * Thin C harness around glm.c's OWN CPU implementation of the MoE FFN hot
 * path. It is compiled from the reference sources where they lie (the
 * reference directory is passed with -I and infer.c is included textually so
 * that its `static` functions are reachable); nothing of the reference is
 * copied into this repository. The build recipe is oracle/Makefile and the
 * output goes to oracle/_ref/libglmref.so.
 *
 * Entry points (plain pointers, ctypes-friendly):
 *   ref_moe_layer    -> apply_moe_shared_ffn_layer   (infer.c:1087-1216)
 *   ref_matvec_q80   -> matvec_q80_rows              (infer.c:765-786)
 *   ref_rmsnorm      -> rmsnorm                      (infer.c:746-752)
 *   ref_time_moe_layer: wall-clock timing of the same call with the
 *                      reference's own clock (monotonic_ms, infer.c:1426)
 *
 * The Runtime/RunState objects are assembled in memory exactly as
 * runtime_open (infer.c:357-744) would leave them for one MoE layer: the
 * layer's weights sit at index 1 of moe_layers / moe_routed_layers
 * (layers 1..n_layers-1 are MoE, infer.c:641,699).
 */
#include "infer.c"

/* Order of the 15 weight pointers: LayerMoeShared fields (model.h:65-74)
 * followed by LayerMoeRouted fields (model.h:76-83). */
enum {
    RP_FFN_NORM = 0, RP_GATE_INP, RP_EXP_PROBS_B,
    RP_GATE_SH_Q, RP_GATE_SH_S, RP_UP_SH_Q, RP_UP_SH_S, RP_DOWN_SH_Q, RP_DOWN_SH_S,
    RP_GATE_Q, RP_GATE_S, RP_UP_Q, RP_UP_S, RP_DOWN_Q, RP_DOWN_S,
    RP_COUNT
};

typedef struct {
    Runtime rt;
    LayerMoeShared shared[2];
    LayerMoeRouted routed[2];
    RunState st;
} RefMoeCtx;

static void ref_ctx_build(RefMoeCtx *c, int dim, int moe_dim, int n_experts, int n_used, int gs,
                          const void *const *p) {
    memset(c, 0, sizeof(*c));
    c->rt.cfg.dim = dim;
    c->rt.cfg.hidden_dim = moe_dim;
    c->rt.cfg.vocab_size = 1;
    c->rt.cfg.n_layers = 2;
    c->rt.cfg.n_routed_experts = n_experts;
    c->rt.cfg.n_experts_used = n_used;
    c->rt.cfg.group_size = (uint64_t)gs;
    c->rt.cfg.moe_ffn_dim = moe_dim;

    LayerMoeShared *w = &c->shared[1];
    w->ffn_norm = (const float *)p[RP_FFN_NORM];
    w->gate_inp = (const float *)p[RP_GATE_INP];
    w->exp_probs_b = (const float *)p[RP_EXP_PROBS_B];
    w->gate_sh_q = (const int8_t *)p[RP_GATE_SH_Q];
    w->gate_sh_s = (const float *)p[RP_GATE_SH_S];
    w->up_sh_q = (const int8_t *)p[RP_UP_SH_Q];
    w->up_sh_s = (const float *)p[RP_UP_SH_S];
    w->down_sh_q = (const int8_t *)p[RP_DOWN_SH_Q];
    w->down_sh_s = (const float *)p[RP_DOWN_SH_S];
    c->rt.moe_layers = c->shared;
    c->rt.has_moe_shared = 1;

    LayerMoeRouted *r = &c->routed[1];
    r->gate_q = (const int8_t *)p[RP_GATE_Q];
    r->gate_s = (const float *)p[RP_GATE_S];
    r->up_q = (const int8_t *)p[RP_UP_Q];
    r->up_s = (const float *)p[RP_UP_S];
    r->down_q = (const int8_t *)p[RP_DOWN_Q];
    r->down_s = (const float *)p[RP_DOWN_S];
    c->rt.moe_routed_layers = c->routed;
    c->rt.has_moe_routed = (r->gate_q != NULL);

    runstate_build(&c->st, &c->rt, 1);
}

/* One call of apply_moe_shared_ffn_layer per token; x is [n_tokens][dim]
 * updated in place; topk_idx/topk_w receive [n_tokens][n_used]. */
int ref_moe_layer(int dim, int moe_dim, int n_experts, int n_used, int gs,
                  const void *const *ptrs, int n_tokens,
                  float *x, int32_t *topk_idx, float *topk_w) {
    RefMoeCtx c;
    ref_ctx_build(&c, dim, moe_dim, n_experts, n_used, gs, ptrs);
    for (int t = 0; t < n_tokens; t++) {
        memcpy(c.st.x, x + (size_t)t * dim, (size_t)dim * sizeof(float));
        apply_moe_shared_ffn_layer(&c.rt, &c.st, gs, 1, 0, 0);
        memcpy(x + (size_t)t * dim, c.st.x, (size_t)dim * sizeof(float));
        for (int k = 0; k < n_used; k++) {
            if (topk_idx) topk_idx[(size_t)t * n_used + k] = c.st.moe_topk_idx[k];
            if (topk_w) topk_w[(size_t)t * n_used + k] = c.st.moe_topk_w[k];
        }
    }
    runstate_free(&c.st);
    return 0;
}

/* Times `iters` calls over the token rows of x (cycling), after `warmup`
 * untimed calls; returns total milliseconds via *ms_total. x is left holding
 * whatever the last calls produced (callers pass a scratch copy). */
int ref_time_moe_layer(int dim, int moe_dim, int n_experts, int n_used, int gs,
                       const void *const *ptrs, int n_tokens, float *x,
                       int warmup, int iters, double *ms_total) {
    RefMoeCtx c;
    ref_ctx_build(&c, dim, moe_dim, n_experts, n_used, gs, ptrs);
    double t0 = 0.0;
    for (int i = 0; i < warmup + iters; i++) {
        if (i == warmup) t0 = monotonic_ms();
        int t = i % (n_tokens > 0 ? n_tokens : 1);
        memcpy(c.st.x, x + (size_t)t * dim, (size_t)dim * sizeof(float));
        apply_moe_shared_ffn_layer(&c.rt, &c.st, gs, 1, 0, 0);
    }
    *ms_total = monotonic_ms() - t0;
    runstate_free(&c.st);
    return 0;
}

void ref_matvec_q80(const int8_t *q, const float *s, const float *x, float *y, int rows, int dim, int gs) {
    matvec_q80_rows(q, s, x, y, rows, dim, gs);
}

int ref_time_matvec_q80(const int8_t *q, const float *s, const float *x, float *y, int rows, int dim, int gs,
                        int warmup, int iters, double *ms_total) {
    double t0 = 0.0;
    for (int i = 0; i < warmup + iters; i++) {
        if (i == warmup) t0 = monotonic_ms();
        matvec_q80_rows(q, s, x, y, rows, dim, gs);
    }
    *ms_total = monotonic_ms() - t0;
    return 0;
}

void ref_rmsnorm(float *o, const float *x, const float *w, int n) {
    rmsnorm(o, x, w, n);
}

int ref_omp_max_threads(void) {
#if defined(_OPENMP)
    return omp_get_max_threads();
#else
    return 1;
#endif
}
