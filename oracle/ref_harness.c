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
 *   ref_time_moe_stack: the same clock around one token passed through a
 *                      stack of distinct MoE layers per step, as the
 *                      decoder's layer loop calls them (infer.c:1819-1845)
 *   ref_decode       -> greedy generation with glm_cpu_forward_token
 *                      (infer.c:1903) and argmax (infer.c:1218), fed as
 *                      glm_app_main's loop feeds it (infer.c:2190-2228)
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

/* Times `steps` steps after `warmup` untimed ones; a step takes the next
 * token row of x (cycling) through layers 0..n_layers-1 of `tables`
 * ([n_layers][RP_COUNT] weight pointers), each layer's output feeding the
 * next, as glm_cpu_forward_token's layer loop does. *ms_total: the steps'
 * total milliseconds. */
int ref_time_moe_stack(int dim, int moe_dim, int n_experts, int n_used, int gs,
                       const void *const *tables, int n_layers, int n_tokens, const float *x,
                       int warmup, int steps, double *ms_total) {
    RefMoeCtx c;
    ref_ctx_build(&c, dim, moe_dim, n_experts, n_used, gs, tables);
    double t0 = 0.0;
    for (int i = 0; i < warmup + steps; i++) {
        if (i == warmup) t0 = monotonic_ms();
        int t = i % (n_tokens > 0 ? n_tokens : 1);
        memcpy(c.st.x, x + (size_t)t * dim, (size_t)dim * sizeof(float));
        for (int l = 0; l < n_layers; l++) {
            const void *const *p = tables + (size_t)l * RP_COUNT;
            LayerMoeShared *w = &c.shared[1];
            LayerMoeRouted *r = &c.routed[1];
            w->ffn_norm = (const float *)p[RP_FFN_NORM];
            w->gate_inp = (const float *)p[RP_GATE_INP];
            w->exp_probs_b = (const float *)p[RP_EXP_PROBS_B];
            w->gate_sh_q = (const int8_t *)p[RP_GATE_SH_Q];
            w->gate_sh_s = (const float *)p[RP_GATE_SH_S];
            w->up_sh_q = (const int8_t *)p[RP_UP_SH_Q];
            w->up_sh_s = (const float *)p[RP_UP_SH_S];
            w->down_sh_q = (const int8_t *)p[RP_DOWN_SH_Q];
            w->down_sh_s = (const float *)p[RP_DOWN_SH_S];
            r->gate_q = (const int8_t *)p[RP_GATE_Q];
            r->gate_s = (const float *)p[RP_GATE_S];
            r->up_q = (const int8_t *)p[RP_UP_Q];
            r->up_s = (const float *)p[RP_UP_S];
            r->down_q = (const int8_t *)p[RP_DOWN_Q];
            r->down_s = (const float *)p[RP_DOWN_S];
            apply_moe_shared_ffn_layer(&c.rt, &c.st, gs, 1, 0, 0);
        }
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

/* OpenMP team size of later calls (the 1-thread baseline line). */
void ref_set_omp_threads(int n) {
#ifdef _OPENMP
    omp_set_num_threads(n > 0 ? n : 1);
#else
    (void)n;
#endif
}

int ref_omp_max_threads(void) {
#if defined(_OPENMP)
    return omp_get_max_threads();
#else
    return 1;
#endif
}

/* Full decoder described by plain tables, assembled in memory as
 * runtime_open would leave it (infer.c:357-744):
 *   icfg[16]: dim, hidden_dim, n_layers, n_heads, vocab_size, rope_dim,
 *             q_lora_rank, kv_lora_rank, qk_nope_dim, head_k_dim, v_head_dim,
 *             n_routed_experts, n_experts_used, group_size, moe_ffn_dim,
 *             cache_cap
 *   glob[12]: output_norm, tok_q, tok_s, out_q, out_s, l0_ffn_norm,
 *             l0 gate q/s, up q/s, down q/s
 *   attn[n_layers*15]: LayerAttnWeights fields per layer (model.h:46-62)
 *   moe[n_layers*15]:  the 15 MoE pointers per layer (layer 0 unused)
 * The prompt ids are fed one per position; then n_gen tokens are picked
 * with argmax (temperature 0) and fed back. out_ids receives them; if
 * logits_out is not NULL it receives the logits of every generating step
 * ([n_gen][vocab]). Returns 0 or the failing forward's status. Built over
 * the cuda-patched glm.c (GLM_ENABLE_CUDA, oracle/glm_cuda_patch.py), the
 * loop runs with the cuda backend started, as glm_app_main starts it
 * (infer.c:2174, 2258). */
int ref_decode(const int32_t *icfg, const void *const *glob, const void *const *attn, const void *const *moe,
               const int32_t *prompt, int n_prompt, int n_gen, int32_t *out_ids, float *logits_out) {
    Runtime rt;
    memset(&rt, 0, sizeof(rt));
    RuntimeConfig *c = &rt.cfg;
    c->dim = icfg[0];
    c->hidden_dim = icfg[1];
    c->n_layers = icfg[2];
    c->n_heads = icfg[3];
    c->n_kv_heads = icfg[3];
    c->vocab_size = icfg[4];
    c->rope_dim = icfg[5];
    c->q_lora_rank = icfg[6];
    c->kv_lora_rank = icfg[7];
    c->l0_qk_nope_dim = icfg[8];
    c->l0_head_k_dim = icfg[9];
    c->l0_v_head_dim = icfg[10];
    c->n_routed_experts = icfg[11];
    c->n_experts_used = icfg[12];
    c->group_size = (uint64_t)icfg[13];
    c->moe_ffn_dim = icfg[14];
    c->seq_len = icfg[15];
    c->bos_id = -1;
    c->eos_id = -1;
    const int L = c->n_layers, gs = icfg[13];

    rt.output_norm = (const float *)glob[0];
    rt.tok_q = (const int8_t *)glob[1];
    rt.tok_s = (const float *)glob[2];
    rt.out_q = (const int8_t *)glob[3];
    rt.out_s = (const float *)glob[4];
    rt.has_l0_ffn = 1;
    rt.l0_ffn_norm = (const float *)glob[5];
    rt.l0_ffn_gate_q = (const int8_t *)glob[6];
    rt.l0_ffn_gate_s = (const float *)glob[7];
    rt.l0_ffn_up_q = (const int8_t *)glob[8];
    rt.l0_ffn_up_s = (const float *)glob[9];
    rt.l0_ffn_down_q = (const int8_t *)glob[10];
    rt.l0_ffn_down_s = (const float *)glob[11];

    LayerAttnWeights *aw = (LayerAttnWeights *)calloc((size_t)L, sizeof(LayerAttnWeights));
    LayerMoeShared *ms = (LayerMoeShared *)calloc((size_t)L, sizeof(LayerMoeShared));
    LayerMoeRouted *mr = (LayerMoeRouted *)calloc((size_t)L, sizeof(LayerMoeRouted));
    if (!aw || !ms || !mr) return -1;
    for (int l = 0; l < L; l++) {
        const void *const *a = attn + (size_t)l * 15;
        aw[l].attn_norm = (const float *)a[0];
        aw[l].q_a_norm = (const float *)a[1];
        aw[l].kv_a_norm = (const float *)a[2];
        aw[l].q_a_q = (const int8_t *)a[3];
        aw[l].q_a_s = (const float *)a[4];
        aw[l].q_b_q = (const int8_t *)a[5];
        aw[l].q_b_s = (const float *)a[6];
        aw[l].kv_a_q = (const int8_t *)a[7];
        aw[l].kv_a_s = (const float *)a[8];
        aw[l].k_b_q = (const int8_t *)a[9];
        aw[l].k_b_s = (const float *)a[10];
        aw[l].v_b_q = (const int8_t *)a[11];
        aw[l].v_b_s = (const float *)a[12];
        aw[l].attn_out_q = (const int8_t *)a[13];
        aw[l].attn_out_s = (const float *)a[14];
        if (l == 0) continue;
        const void *const *p = moe + (size_t)l * 15;
        ms[l].ffn_norm = (const float *)p[RP_FFN_NORM];
        ms[l].gate_inp = (const float *)p[RP_GATE_INP];
        ms[l].exp_probs_b = (const float *)p[RP_EXP_PROBS_B];
        ms[l].gate_sh_q = (const int8_t *)p[RP_GATE_SH_Q];
        ms[l].gate_sh_s = (const float *)p[RP_GATE_SH_S];
        ms[l].up_sh_q = (const int8_t *)p[RP_UP_SH_Q];
        ms[l].up_sh_s = (const float *)p[RP_UP_SH_S];
        ms[l].down_sh_q = (const int8_t *)p[RP_DOWN_SH_Q];
        ms[l].down_sh_s = (const float *)p[RP_DOWN_SH_S];
        mr[l].gate_q = (const int8_t *)p[RP_GATE_Q];
        mr[l].gate_s = (const float *)p[RP_GATE_S];
        mr[l].up_q = (const int8_t *)p[RP_UP_Q];
        mr[l].up_s = (const float *)p[RP_UP_S];
        mr[l].down_q = (const int8_t *)p[RP_DOWN_Q];
        mr[l].down_s = (const float *)p[RP_DOWN_S];
    }
    rt.has_all_attn = 1;
    rt.attn_layers = aw;
    rt.has_moe_shared = 1;
    rt.moe_layers = ms;
    rt.has_moe_routed = 1;
    rt.moe_routed_layers = mr;

    RunState st;
    runstate_build(&st, &rt, icfg[15]);
#if defined(GLM_ENABLE_CUDA)
    glm_backend_init(BACKEND_CUDA, &rt, &st);
#endif
    int token = prompt[0];
    if (token < 0 || token >= c->vocab_size) token = 0;
    int prompt_index = 1, generated = 0, rc = 0;
    for (int pos = 0; pos < icfg[15]; pos++) {
        rc = glm_cpu_forward_token(&rt, &st, token, pos, 0);
        if (rc != 0) break;
        int next;
        if (prompt_index < n_prompt) {
            next = prompt[prompt_index++];
            if (next < 0 || next >= c->vocab_size) next = 0;
        } else {
            next = argmax(st.logits, c->vocab_size);
            if (logits_out)
                memcpy(logits_out + (size_t)generated * c->vocab_size, st.logits, (size_t)c->vocab_size * sizeof(float));
            out_ids[generated++] = next;
            if (generated >= n_gen) break;
        }
        token = next;
    }
#if defined(GLM_ENABLE_CUDA)
    glm_backend_free(0);
#endif
    runstate_free(&st);
    free(aw);
    free(ms);
    free(mr);
    (void)gs;
    return rc;
}

/* glm.c's own loader on a .bin checkpoint (runtime_open, infer.c:357-744),
 * then the same greedy loop as ref_decode (glm_cpu_forward_token per
 * position, argmax at temperature 0, infer.c:2190-2228). runtime_open exits
 * the process on a malformed file, as glm.c does. */
int ref_decode_bin(const char *path, const int32_t *prompt, int n_prompt, int n_gen, int cache_cap,
                   int32_t *out_ids) {
    Runtime rt;
    memset(&rt, 0, sizeof(rt));
    runtime_open(&rt, path);
    RuntimeConfig *c = &rt.cfg;
    c->bos_id = -1;
    c->eos_id = -1;
    RunState st;
    runstate_build(&st, &rt, cache_cap);
    int token = prompt[0];
    if (token < 0 || token >= c->vocab_size) token = 0;
    int prompt_index = 1, generated = 0, rc = 0;
    for (int pos = 0; pos < cache_cap; pos++) {
        rc = glm_cpu_forward_token(&rt, &st, token, pos, 0);
        if (rc != 0) break;
        int next;
        if (prompt_index < n_prompt) {
            next = prompt[prompt_index++];
            if (next < 0 || next >= c->vocab_size) next = 0;
        } else {
            next = argmax(st.logits, c->vocab_size);
            out_ids[generated++] = next;
            if (generated >= n_gen) break;
        }
        token = next;
    }
    runstate_free(&st);
    runtime_close(&rt);
    return rc;
}
