/*
 * glm_cuda.h -- C-ABI of the B200 (sm_100a) backend for glm.c's
 * mixture-of-experts FFN hot path (GLM-4.7-Flash).
 *
 * Plain pointers and sizes only; no CUDA or C++ types cross this boundary
 * (streams are passed as void*). Every entry point returns 0 on success and a
 * negative GLM_CUDA_ERR_* code on failure; glm_cuda_last_error() returns the
 * message. There is no CPU fallback behind any of these calls: if the device
 * path cannot run, the call fails.
 *
 * Weight layout is glm.c's planar Q8 format, unchanged: int8 q[rows][cols]
 * row-major plus fp32 s[rows][cols/gs] row-major (infer.c:765-786), routed
 * experts stored expert-major (infer.c:697-742). Supported: gs == 32 or 16
 * (glm.c's own export uses 16, glm47_flash_export.py:36), dim % 128 == 0,
 * moe_ffn_dim % 64 == 0 (% 128 for gs == 16), 1 <= n_experts_used <= 8.
 * Both group sizes run on the integer tensor cores; per-token MoE calls take
 * the persistent kernel at either size (the three-kernel chain, which the
 * allocation-free entry point uses, takes gs == 32 only).
 *
 * Threading: like glm.c's backends (one instance per process, infer.m:18-37)
 * the library keeps one global device context; calls are serialised by an
 * internal mutex.
 */
#ifndef GLM_CUDA_H
#define GLM_CUDA_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define GLM_CUDA_OK 0
#define GLM_CUDA_ERR_ARG (-1)      /* bad argument or unsupported shape */
#define GLM_CUDA_ERR_STATE (-2)    /* not initialised / layer not uploaded */
#define GLM_CUDA_ERR_CUDA (-3)     /* a CUDA call failed */
#define GLM_CUDA_ERR_NOMEM (-4)    /* device allocation failed */

/* Device bring-up and per-process state for `n_layers` layer slots.
 * Replaces the device part of glm_backend_init (backend.h:7, backend.c:73-86;
 * Metal counterpart glm_metal_init, infer.m:847-929). The glm.c glue treats a
 * nonzero return the way backend.c:79-82 treats a Metal init failure. */
int glm_cuda_init(int device, int dim, int moe_ffn_dim, int n_routed_experts, int n_experts_used,
                  int group_size, int n_layers);

/* Copy one MoE layer's weights to HBM, preserving the planar Q8 layout.
 * Arguments are the fields of LayerMoeShared (model.h:65-74) followed by
 * LayerMoeRouted (model.h:76-83) for layer `layer` as runtime_open leaves
 * them (infer.c:640-743); host pointers. gate_q == NULL uploads no routed
 * block (has_moe_routed == 0). Replaces the weight-upload step of
 * glm_metal_prepare (infer.m:932-1010), which never uploaded routed experts. */
int glm_cuda_upload_moe_layer(int layer, const float *ffn_norm, const float *gate_inp, const float *exp_probs_b,
                              const int8_t *gate_sh_q, const float *gate_sh_s, const int8_t *up_sh_q,
                              const float *up_sh_s, const int8_t *down_sh_q, const float *down_sh_s,
                              const int8_t *gate_q, const float *gate_s, const int8_t *up_q, const float *up_s,
                              const int8_t *down_q, const float *down_s);

/* As glm_cuda_upload_moe_layer, but the pointers are device memory that the
 * caller owns and keeps alive (16-byte aligned); nothing is copied. */
int glm_cuda_bind_moe_layer_device(int layer, const float *ffn_norm, const float *gate_inp,
                                   const float *exp_probs_b, const int8_t *gate_sh_q, const float *gate_sh_s,
                                   const int8_t *up_sh_q, const float *up_sh_s, const int8_t *down_sh_q,
                                   const float *down_sh_s, const int8_t *gate_q, const float *gate_s,
                                   const int8_t *up_q, const float *up_s, const int8_t *down_q,
                                   const float *down_s);

/* The MoE FFN of layer `layer` applied in place to x[n_tokens][dim] (host
 * memory): rmsnorm, sigmoid router with biased top-k, K routed SwiGLU experts
 * weighted by 1.8 * normalised probability, shared expert, residual add.
 * Replaces apply_moe_shared_ffn_layer (infer.c:1087-1216), called from the
 * layer loop at infer.c:1845. topk_idx / topk_w (may be NULL) receive
 * [n_tokens][n_experts_used] as RunState.moe_topk_idx / moe_topk_w hold them
 * (model.h:157-158). GLM_DISABLE_MOE_ROUTED is honoured per call as at
 * infer.c:1161-1165. Synchronous: returns after x is back in host memory. */
int glm_cuda_moe_layer(int layer, float *x, int n_tokens, int32_t *topk_idx, float *topk_w);

/* Stream-ordered variant on device memory (x_dev in place, topk outputs
 * optional device arrays); `stream` is a cudaStream_t or NULL for the
 * library's own stream. Returns after enqueueing. */
int glm_cuda_moe_layer_async(int layer, float *x_dev, int n_tokens, int32_t *topk_idx_dev, float *topk_w_dev,
                             void *stream);

/* Decode kernels behind glm_cuda_moe_layer / _async. PERSISTENT: one
 * launch per token and layer, one CTA per SM (all resident) streaming every
 * weight tile through shared memory with TMA (needs n_routed_experts <= SM
 * count and a multiple of 4, dim <= 2048, moe_ffn_dim % 128 == 0 and <= 3840).
 * CHAIN: three dependent kernels per token and layer (router, gate/up, down).
 * AUTO (the default) picks PERSISTENT when the sizes allow. Both give the
 * same expert ids and agree on x to fp32 rounding. */
#define GLM_CUDA_PATH_AUTO 0
#define GLM_CUDA_PATH_PERSISTENT 1
#define GLM_CUDA_PATH_CHAIN 2
#define GLM_CUDA_PATH_BATCHED 3  /* sizes outside the per-token kernels: every call runs the batched kernels */

/* Select the decode kernels (GLM_CUDA_PATH_*). No counterpart in glm.c. */
int glm_cuda_set_decode_path(int path);

/* ---- expert parallelism (no counterpart in glm.c, which runs every expert
 * on one host): the routed experts are split over n_shards ranks (one
 * process per GPU), n_routed_experts / n_shards consecutive experts each;
 * every rank routes its own tokens, the (token, slot) rows travel to the
 * rank holding their expert and the expert outputs travel back (the caller
 * moves the buffers, e.g. with an NCCL all-to-all), the shared expert runs
 * where the tokens are. Per layer: ep_dispatch -> exchange -> ep_experts ->
 * exchange back -> ep_combine; one layer at a time. */

/* Make this rank shard `shard` of n_shards; max_tokens bounds n_tokens of
 * ep_dispatch. Call after glm_cuda_init and before uploading layers: the
 * routed arrays of later uploads / binds hold only this shard's experts
 * (gate/up [n_routed_experts / n_shards][moe_ffn_dim][dim] ...), the router
 * and the shared expert stay whole. The single-rank MoE entry points then
 * return GLM_CUDA_ERR_STATE. Allocates the exchange scratch. */
int glm_cuda_ep_setup(int n_shards, int shard, int max_tokens);

/* Route x_dev[n_tokens][dim] (device) exactly as apply_moe_shared_ffn_layer
 * (infer.c:1098-1145) and lay out the send buffer: for every (token, slot)
 * pair with a valid expert, its normalised row (rmsnorm(x) * ffn_norm, fp32
 * [dim]) in send_rows_dev, grouped by destination shard (shard order; pairs
 * in (token, slot) order within a shard), the expert id local to that shard
 * in send_expert_dev, and send_counts_dev[n_shards] rows per shard. Buffers
 * hold n_tokens * n_experts_used rows. Stream-ordered. */
int glm_cuda_ep_dispatch(int layer, const float *x_dev, int n_tokens, float *send_rows_dev,
                         int32_t *send_expert_dev, int32_t *send_counts_dev, void *stream);

/* This shard's experts on n_recv received rows (recv_expert_dev: local
 * expert ids) plus the shared expert on this rank's tokens of the last
 * dispatch; out_rows_dev[n_recv][dim] receives each row's expert output
 * (SwiGLU FFN, not yet weighted) in the received order. */
int glm_cuda_ep_experts(int layer, const float *recv_rows_dev, const int32_t *recv_expert_dev, int n_recv,
                        float *out_rows_dev, void *stream);

/* x_dev += shared + sum_k 1.8 w_k y_k in rank order (infer.c:1175-1214), with
 * y_k read from back_rows_dev laid out as the send buffer of the last
 * dispatch; topk outputs (may be NULL) as in glm_cuda_moe_layer. */
int glm_cuda_ep_combine(int layer, float *x_dev, const float *back_rows_dev, int32_t *topk_idx_dev,
                        float *topk_w_dev, void *stream);

/* Synchronise and report a bounded wait that gave up in the ep kernels. */
int glm_cuda_ep_status(void);

/* ---- Expert parallelism over peer memory (NVLink), no host round trip.
 * Same layer as glm_cuda_ep_dispatch / _experts / _combine with the exchange
 * done by the kernels: every rank holds one "peer region" of the same layout
 * (sized by glm_cuda_ep_setup's arguments, which must agree on every rank);
 * the sender writes each (token, slot) row, its local expert id and the row
 * counts straight into the receiver's region and raises a per-pair flag; the
 * receiver's expert kernels wait for every sender's flag, and send the
 * outputs back the same way. Flags carry the layer-call count, so the three
 * calls below must be made in the same order on every rank, and no call is
 * ever skipped on one rank. A peer that does not answer within 4 s makes the
 * waiting kernel give up (glm_cuda_ep_status then returns GLM_CUDA_ERR_CUDA).
 * The reference has no multi-GPU path; this replaces the all-to-all of the
 * calls above (infer.c:1166-1195 per token, with the expert products on the
 * rank that holds the expert). */

#define GLM_CUDA_IPC_HANDLE_BYTES 64

/* Allocate (once) this rank's peer region; *region_dev_out receives its
 * device address, ipc_handle_out (may be NULL) GLM_CUDA_IPC_HANDLE_BYTES of
 * cudaIpcMemHandle_t for the other ranks' glm_cuda_ep_peer_open. */
int glm_cuda_ep_peer_region(void **region_dev_out, void *ipc_handle_out);

/* Map another rank's region (its IPC handle) into this process. */
int glm_cuda_ep_peer_open(const void *ipc_handle, void **region_dev_out);

/* regions[n_shards]: every rank's region as this process addresses it
 * (regions[shard] = this rank's own). Two library instances in one process
 * may pass each other's region addresses directly. */
int glm_cuda_ep_peer_connect(void *const *regions);

/* Route x_dev[n_tokens][dim], pack, push the rows to their experts' ranks. */
int glm_cuda_ep_p2p_dispatch(int layer, const float *x_dev, int n_tokens, void *stream);

/* Wait for every rank's rows, run this rank's experts (and the shared
 * expert on its own tokens), push the outputs back to their senders. */
int glm_cuda_ep_p2p_experts(int layer, void *stream);

/* Wait for every rank's outputs; x_dev += shared + sum_k 1.8 w_k y_k in rank
 * order (infer.c:1175-1214); topk outputs (may be NULL) as in
 * glm_cuda_moe_layer. */
int glm_cuda_ep_p2p_combine(int layer, float *x_dev, int32_t *topk_idx_dev, float *topk_w_dev, void *stream);

/* Host copies (synchronising the device) of the last dispatch's rows per
 * receiver and of the rows received from each sender, [n_shards] each. */
int glm_cuda_ep_p2p_counts(int32_t *send_counts, int32_t *recv_counts);

/* Calls of glm_cuda_moe_layer / _async with n_tokens >= min_tokens run the
 * batched prefill kernels instead of the per-token decode kernels: exact
 * routing of all tokens in one launch, then the routed and shared experts
 * as grouped GEMMs on the tensor cores (Q8 weights dequantised on chip to
 * bf16 pairs), then the weighted combine. Same expert ids; x agrees with
 * the decode kernels within ~1e-5 relative. 0 disables it (except with
 * gs == 16, where every call is batched). Default 32 where the sizes fit
 * (dim and moe_ffn_dim multiples of 128, n_routed_experts <= 256). The first call with a larger n_tokens
 * than before allocates the kernels' scratch. Returns the previous value,
 * or a negative error. No counterpart in glm.c, whose prefill runs the
 * token loop of glm_app_main (infer.c:2190-2228). */
int glm_cuda_set_prefill_tokens(int min_tokens);

/* The decode kernels the next call will use: GLM_CUDA_PATH_PERSISTENT or
 * GLM_CUDA_PATH_CHAIN (negative on error). */
int glm_cuda_decode_path(void);

/* One token through the MoE FFN of layers first_layer .. first_layer +
 * n_layers - 1 in turn (x_dev[dim] in place), as consecutive calls of
 * glm_cuda_moe_layer_async with n_tokens = 1 would do, in a single
 * persistent launch: glm.c's per-layer MoE call (apply_moe_shared_ffn_layer,
 * infer.c:1087-1216) repeated over a stack of MoE layers with nothing between
 * them. In the full decoder attention runs between MoE layers and
 * glm_cuda_moe_layer_async is the call to use. topk_idx_dev / topk_w_dev (may
 * be NULL) receive [n_layers][n_experts_used]. Fails with GLM_CUDA_ERR_ARG
 * when the sizes do not fit the persistent kernel. */
int glm_cuda_moe_layers_async(int first_layer, int n_layers, float *x_dev, int32_t *topk_idx_dev,
                              float *topk_w_dev, void *stream);

/* Instrumented single-token run of the CHAIN decode kernels on device
 * memory: CUDA events are recorded between the three decode kernels (router,
 * gate/up+SwiGLU, down+combine) and ms_out[0..2] receive their durations.
 * Synchronises the library stream. For profiling; no counterpart in glm.c
 * beyond its per-token bench timing (infer.c:2194-2196). */
int glm_cuda_moe_layer_profile(int layer, float *x_dev, float ms_out[3]);

/* No counterpart in glm.c: an addition for callers that must not allocate
 * device memory at call time (e.g. a server that plans all GPU memory at
 * start-up and forbids cudaMalloc on the request path, or an embedder that
 * only hands over pointers it already owns), and so cannot call
 * glm_cuda_init. Same computation as glm_cuda_moe_layer_async, on device
 * memory the caller owns: the 15 weight pointers in the order of
 * glm_cuda_upload_moe_layer, the shape, x_dev[n_tokens][dim] updated in place
 * and optional topk outputs. Allocates nothing: its scratch is a fixed
 * ~170 KB static device array per GPU (held until the process exits), so
 * dim <= 4096, moe_ffn_dim <= 4096, n_routed_experts <= 256 and
 * n_experts_used <= 8 (else GLM_CUDA_ERR_ARG), with gs == 32. The first call
 * on a device resolves that array's address; make it before any stream
 * capture. All calls share the array: calls that overlap on the GPU race and
 * must be ordered by the caller. Uses the current device; `stream` may be
 * NULL (legacy default stream). */
int glm_cuda_moe_layer_noalloc(const float *ffn_norm, const float *gate_inp, const float *exp_probs_b,
                               const int8_t *gate_sh_q, const float *gate_sh_s, const int8_t *up_sh_q,
                               const float *up_sh_s, const int8_t *down_sh_q, const float *down_sh_s,
                               const int8_t *gate_q, const float *gate_s, const int8_t *up_q, const float *up_s,
                               const int8_t *down_q, const float *down_s, int dim, int moe_ffn_dim,
                               int n_routed_experts, int n_experts_used, int group_size, float *x_dev,
                               int n_tokens, int32_t *topk_idx_dev, float *topk_w_dev, void *stream);

/* y[rows] = Q8(qmat, smat) . x[dim], host pointers. Same signature and
 * return convention as glm_backend_try_metal_matvec (backend.h:13,
 * backend.c:67-71; called by matvec_rows at infer.c:793): 0 = handled,
 * nonzero = not handled. The weight matrix is copied to HBM on first use and
 * cached by its host address, as infer.m:307-322 caches Metal buffers. */
int glm_cuda_matvec_q80(const int8_t *qmat, const float *smat, const float *x, float *y, int rows, int dim, int gs);

/* Stream-ordered matvec on device pointers. q_dev must be 16-byte aligned,
 * s_dev 8-byte (gs 32) or 4-byte (gs 16) aligned, dim a multiple of 64;
 * GLM_CUDA_ERR_CUDA (misaligned address) otherwise, before any launch. */
int glm_cuda_matvec_q80_async(const int8_t *q_dev, const float *s_dev, const float *x_dev, float *y_dev, int rows,
                              int dim, int gs, void *stream);

/* Wait for all work on the device (the library's stream and the streams
 * passed to the _async calls); GLM_CUDA_ERR_CUDA if a decode kernel's bounded
 * wait gave up since the last check. */
int glm_cuda_synchronize(void);

/* Router statistics since init: out[0] routed tokens, out[1] tokens whose
 * fast interval certification failed and took the exact recomputation,
 * out[2] tokens still not certified after it: a tie that only libm's last
 * bit of expf could decide (resolved with a correctly rounded exp), or
 * experts with bit-identical exact logits (ordered by id, as glm.c orders
 * them), out[3] rmsnorm means recomputed serially. */
int glm_cuda_route_stats(uint64_t out[4]);

/* Number of kernel launches the library has issued since init. */
uint64_t glm_cuda_launch_count(void);

/* Message of the most recent failure ("" if none). */
const char *glm_cuda_last_error(void);

/* ------------------------------------------------------------------------
 * Full batch-1 decoder (GLM-4.7-Flash: MLA attention in every layer, a dense
 * SwiGLU FFN in layer 0, MoE FFN in layers 1..n_layers-1), the device side of
 * glm_backend_forward_token (backend.h:8, backend.c:88-91).
 * ------------------------------------------------------------------------ */

/* Shapes, named after RuntimeConfig (model.h:7-45). cache_cap = KV-cache
 * positions (RunState.cache_cap, infer.c:2165-2170). */
typedef struct GlmCudaModelDims {
    int32_t dim, hidden_dim, n_layers, n_heads, vocab_size, rope_dim, q_lora_rank, kv_lora_rank;
    int32_t qk_nope_dim, head_k_dim, v_head_dim, n_routed_experts, n_experts_used, group_size, moe_ffn_dim;
    int32_t cache_cap;
} GlmCudaModelDims;

/* Device bring-up for the whole decoder; also does glm_cuda_init for the MoE
 * layers (then uploaded with glm_cuda_upload_moe_layer, layers 1..). Replaces
 * glm_backend_init's device part (backend.c:73-86). */
int glm_cuda_model_init(int device, const GlmCudaModelDims *dims);

/* Runtime's model-wide weights (model.h:87-103): output_norm, token
 * embedding tok_q/tok_s, LM head out_q/out_s, layer-0 dense FFN norm and
 * gate/up/down. Host pointers, copied to HBM (planar Q8 kept). */
int glm_cuda_upload_model_globals(const float *output_norm, const int8_t *tok_q, const float *tok_s,
                                  const int8_t *out_q, const float *out_s, const float *l0_ffn_norm,
                                  const int8_t *l0_gate_q, const float *l0_gate_s, const int8_t *l0_up_q,
                                  const float *l0_up_s, const int8_t *l0_down_q, const float *l0_down_s);

/* As above on caller-owned device memory (16-byte aligned); nothing copied. */
int glm_cuda_bind_model_globals_device(const float *output_norm, const int8_t *tok_q, const float *tok_s,
                                       const int8_t *out_q, const float *out_s, const float *l0_ffn_norm,
                                       const int8_t *l0_gate_q, const float *l0_gate_s, const int8_t *l0_up_q,
                                       const float *l0_up_s, const int8_t *l0_down_q, const float *l0_down_s);

/* One layer's attention weights in the order of LayerAttnWeights
 * (model.h:46-62); host pointers, copied to HBM. */
int glm_cuda_upload_attn_layer(int layer, const float *attn_norm, const float *q_a_norm, const float *kv_a_norm,
                               const int8_t *q_a_q, const float *q_a_s, const int8_t *q_b_q, const float *q_b_s,
                               const int8_t *kv_a_q, const float *kv_a_s, const int8_t *k_b_q, const float *k_b_s,
                               const int8_t *v_b_q, const float *v_b_s, const int8_t *attn_out_q,
                               const float *attn_out_s);

/* As above on caller-owned device memory (16-byte aligned). */
int glm_cuda_bind_attn_layer_device(int layer, const float *attn_norm, const float *q_a_norm,
                                    const float *kv_a_norm, const int8_t *q_a_q, const float *q_a_s,
                                    const int8_t *q_b_q, const float *q_b_s, const int8_t *kv_a_q,
                                    const float *kv_a_s, const int8_t *k_b_q, const float *k_b_s,
                                    const int8_t *v_b_q, const float *v_b_s, const int8_t *attn_out_q,
                                    const float *attn_out_s);

/* One decode step of token `token` at position `pos` (writing the KV cache
 * at pos): glm_cpu_forward_token (infer.c:1903) on the GPU. logits (host,
 * vocab_size floats, may be NULL) receive the LM-head output, as
 * RunState.logits. Replaces glm_backend_forward_token (backend.c:88-91). */
int glm_cuda_forward_token(int token, int pos, float *logits);

/* Greedy generation as glm.c's loop runs it at temperature 0
 * (infer.c:2190-2228; argmax infer.c:1218-1228): the prompt ids are fed one
 * per position, then n_gen tokens are picked by argmax and fed back; out_ids
 * receives them. The whole step runs from device memory (one CUDA graph per
 * call, replayed for every position). device_ms (may be NULL) receives the
 * device time of the n_prompt + n_gen - 1 steps. */
int glm_cuda_generate(const int32_t *prompt, int n_prompt, int n_gen, int32_t *out_ids, float *device_ms);

/* Batched prompt pass: positions start_pos .. start_pos + n_tokens - 1 with
 * ids tokens[0 .. n_tokens) (clamped to the vocabulary as infer.c:2219)
 * through every layer as one batch, writing their KV-cache rows: what
 * n_tokens calls of glm_backend_forward_token in glm.c's prompt loop
 * (infer.c:2190-2233) leave behind, with the layers taken one at a time.
 * Per layer, each token's attention runs in position order on the decode
 * kernels (the causal order: token t reads the rows written for the tokens
 * before it). Then the FFN of the whole batch runs at once on the batched
 * MoE kernels, which read each touched expert's weights once per layer.
 * Expert ids are glm.c's.
 * The residual rows agree with token-by-token decoding to ~1e-5 relative
 * (the grouped GEMMs' bf16-pair products). logits (host, vocab_size
 * floats, may be NULL) receive the last token's LM-head output. Needs the
 * batched MoE kernels (dim and moe_ffn_dim multiples of 128). */
int glm_cuda_prefill(const int32_t *tokens, int n_tokens, int start_pos, float *logits);

/* glm_cuda_generate runs prompts of n_prompt - 1 >= min_tokens through
 * glm_cuda_prefill's batched pass for positions 0 .. n_prompt - 2, then
 * decodes step by step from position n_prompt - 1. 0 (the default) keeps
 * the token-by-token prompt loop. */
int glm_cuda_set_model_prefill(int min_tokens);

/* Release all device memory and state. Replaces glm_backend_free's device
 * part (backend.c:93-95, glm_metal_free). Safe to call twice. */
/* glm.c's runtime checkpoint (.bin, format version 4 with every layer's
 * attention, as glm47_flash_export.py writes it) to the device: maps the
 * file, checks the header and offsets as runtime_open does (infer.c:357-744),
 * then glm_cuda_model_init(device, dims from the header, cache_cap) and the
 * upload calls for the globals, every attention layer and every MoE layer.
 * Replaces runtime_open + glm_backend_init (backend.c:73-86) for the cuda
 * backend; glm_cuda_forward_token / glm_cuda_generate follow. A malformed
 * file is GLM_CUDA_ERR_ARG (glm.c exits instead). */
int glm_cuda_load_checkpoint(const char *path, int device, int cache_cap);

void glm_cuda_free(void);

#ifdef __cplusplus
}
#endif

#endif /* GLM_CUDA_H */
