// Internal (non-exported) interfaces between the C-ABI layer (glm_cuda.cu)
// and the kernel translation units.
#pragma once

#include <cstdint>
#include <cuda_runtime.h>

namespace glmq {

// Device-resident weights of one MoE FFN layer, planar Q8 as in glm.c
// (LayerMoeShared model.h:65-74, LayerMoeRouted model.h:76-83).
struct MoeLayerDev {
    const float* ffn_norm = nullptr;     // [D]
    const float* router = nullptr;       // [E][D]   gate_inp
    const float* router_bias = nullptr;  // [E]      exp_probs_b
    const int8_t* gate_sh_q = nullptr;   // [F][D]
    const float* gate_sh_s = nullptr;    // [F][D/gs]
    const int8_t* up_sh_q = nullptr;
    const float* up_sh_s = nullptr;
    const int8_t* down_sh_q = nullptr;   // [D][F]
    const float* down_sh_s = nullptr;    // [D][F/gs]
    const int8_t* gate_q = nullptr;      // [E][F][D]
    const float* gate_s = nullptr;       // [E][F][D/gs]
    const int8_t* up_q = nullptr;
    const float* up_s = nullptr;
    const int8_t* down_q = nullptr;      // [E][D][F]
    const float* down_s = nullptr;       // [E][D][F/gs]
};

struct MoeDims {
    int D, F, E, K, gs;
};

// Per-device scratch of the decode path (all device pointers).
struct MoeScratch {
    float* xn;              // [D]
    float* h;               // [(K+1)][F]  SwiGLU activations, routed slots by rank, shared last
    double* center;         // [E] router logit estimates
    double* bound;          // [E] rigorous error bound of the reference's serial fp32 sum
    int32_t* topk_idx;      // [K]
    float* topk_w;          // [K]
    unsigned int* counter;  // [1] last-CTA election; kept at 0 between launches
    unsigned long long* stats;  // [4] calls, interval fallbacks, unresolved near-ties, mean fallbacks
    // Persistent kernel only:
    unsigned int* status = nullptr;    // [1] nonzero after one of its bounded waits gave up
    unsigned int* grid_bar = nullptr;  // [2] grid-barrier arrivals, exited CTAs (reset by the last CTA out)
};

// One decode token through one MoE layer: x_out = x_in + FFN(x_in).
// x_in may equal x_out. Returns a cudaError_t from the launches.
// `events` (optional, 4 entries) are recorded before K1, after K1, after K2
// and after K3 on `stream`, for per-kernel timing.
cudaError_t launch_moe_decode(const MoeLayerDev& w, const MoeDims& d, const MoeScratch& s, const float* x_in,
                              float* x_out, int routed_enabled, int num_sms, cudaStream_t stream,
                              cudaEvent_t* events = nullptr);

// Whether the persistent decode kernel supports these sizes on a device with
// `num_sms` SMs (and its dynamic shared memory size).
cudaError_t persistent_check(const MoeDims& d, int num_sms, size_t* smem_out);

// One token through the MoE FFN of layers [first, first + n_layers) of the
// device table `layers_dev`, in one launch of one CTA per SM (all resident):
// x <- x + FFN_l(x) for each layer in turn. topk_out / topkw_out (optional,
// [n_layers][K]) receive each layer's expert ids and weights. next_layer
// (table index or -1) names the layer expected after the last one: its
// routing-independent weights are pulled into L2 while the last layer runs.
cudaError_t launch_moe_persistent(const MoeLayerDev* layers_dev, int first, int n_layers, const MoeDims& d,
                                  const MoeScratch& s, float* x, int32_t* topk_out, float* topkw_out,
                                  int routed_enabled, int num_sms, cudaStream_t stream, int next_layer);

// y = Q8(q, s) . x for a rows x cols planar Q8 matrix (gs = 32, cols % 64 == 0);
// with `accumulate`, y += Q8(q, s) . x; with `norm`, x is first replaced by
// rmsnorm(x) * norm (glm.c's rmsnorm, infer.c:746-752). With `stage`, each
// CTA copies its weight rows into shared memory before the launch wait when
// they fit (~200 KB): faster when the launch follows a long kernel whose SMs
// free up one by one (the decoder), slower back to back with no work in
// between (each CTA then waits for its whole slice before computing).
cudaError_t launch_q80_matvec(const int8_t* q, const float* s, const float* x, float* y, int rows, int cols,
                              int gs, int num_sms, cudaStream_t stream, bool accumulate = false,
                              const float* norm = nullptr, bool stage = false);

// Two matrices with the same column count on the same (normed) x in one
// launch: y = Q8(q, s) . x (rows rows), y2 = Q8(q2, s2) . x (rows2 rows).
cudaError_t launch_q80_matvec2(const int8_t* q, const float* s, float* y, int rows, const int8_t* q2,
                               const float* s2, float* y2, int rows2, const float* x, int cols, int gs, int num_sms,
                               cudaStream_t stream, const float* norm, bool stage = false);

// ---- decoder around the MoE layers (decoder.cu)

struct MlaArgs {
    const float* q_full;      // [n_heads][head_k]
    const float* kv_a;        // [kv_lora + rope] this position's kv_a projection
    const float* kv_norm;     // [kv_lora] kv_a_norm
    float* cache_comp;        // this layer's [cap][kv_lora]; position pos is written
    float* cache_pe;          // this layer's [cap][rope]
    const int8_t* k_b_q;      // [n_heads][kv_lora][qk_nope]
    const float* k_b_s;
    const int8_t* v_b_q;      // [n_heads][v_head][kv_lora]
    const float* v_b_s;
    float* att_concat;        // [n_heads][v_head]
    const int* pos;           // device: current position
    int qk_nope, rope, head_k, kv_lora, v_head, gs, cache_cap;
    float kq_scale;
};

cudaError_t launch_embed(const int8_t* tok_q, const float* tok_s, const int* token, float* x, int D, int gs,
                         cudaStream_t st);
// MLA attention of every head with this position's cache write, one
// thread-block cluster of kMlaCluster CTAs per head (decoder.cu).
constexpr int kMlaCluster = 8;
constexpr int kMlaThreads = 256;
constexpr int kMlaStage = 4;      // staged q / kv_a floats per thread: head_k, kv_lora + rope <= 1024
constexpr int kMlaRowBlocks = 8;  // 128-float blocks of a cache row: kv_lora <= 1024
size_t mla_smem(const MlaArgs& a);
cudaError_t launch_mla(const MlaArgs& a, int n_heads, cudaStream_t st);
cudaError_t launch_silu_mul(float* g, const float* u, int n, int num_sms, cudaStream_t st);
// part: nblocks float2 scratch; counter: one word, zero between calls.
cudaError_t launch_argmax(const float* x, int n, float2* part, unsigned* counter, int nblocks, int* out,
                          cudaStream_t st);
cudaError_t launch_decode_advance(int* pos, int* token, const int* argmax, const int* prompt, int n_prompt,
                                  int* out_ids, int vocab, cudaStream_t st);

size_t q80_matvec_smem_bytes(int cols, bool norm = false, int gs = 32);

// ---- batched prefill (moe_prefill.cu)

struct PrefillRouteArgs {
    const float* x;        // [T][D]
    const float* norm;     // [D] ffn_norm
    const float* router;   // [E][D]
    const float* bias;     // [E]
    float* xn;             // [T][D] rmsnorm(x) * norm
    int32_t* topk_idx;     // [T][K]
    float* topk_w;         // [T][K]
    unsigned long long* stats;
    int T, D, E, K;
    double* cen;           // [T][E] router logit centres (scratch)
    double* bnd;           // [T][E] their error bounds (scratch)
};

struct PrefillDispatchArgs {
    const int32_t* topk_idx;  // [T][K]
    int T, K, E, routed;
    int mt1, mt2;             // weight-row tiles of gate/up (F / 128) and of down (D / 128)
    int* counts;              // [0] rows, [1] gate/up items, [2] down items
    int* row_tok;             // [rows] token of each row
    int* tok_row;             // [T][K + 1] row of each (token, slot); slot K = shared expert; -1 = none
    int4* items1;             // gate/up items {group, row0, nrows, m-tile}
    int4* items2;             // down items {group, row0, nrows, m-tile}
};

constexpr int kEpMaxShards = 8;  // most ranks the routed experts are split over

struct GroupGemmArgs {
    const int4* items1;
    const int4* items2;
    const int* counts;
    void* hhi;         // mode 0 output: h = SwiGLU(gate, up) [rows][Mtot] bf16 high part
    void* hlo;         //                                       low part
    float* y;          // mode 1 output [rows][Mtot]
    unsigned* status;  // bit 64: a bounded wait gave up
    int K, Mtot, E, mode;  // mode 0: gate/up (K = D, Mtot = F); 1: down (K = F, Mtot = D)
    int gs;                // weight scale group: 32 or 16
    // Mode 1 of expert parallelism over peer memory (row_src non-null): the
    // output row of a received slot q * cap + j goes straight into row
    // me * cap + j of back_rows in rank q's region; rows of this rank's own
    // tokens (sources n_slots + t) go to y. After the last CTA's stores,
    // flag_back[me] of every region is raised to `epoch`.
    const int* row_src = nullptr;  // grouped row -> source
    unsigned char* peer[kEpMaxShards] = {};
    size_t back_off = 0, flag_off = 0;
    int n_slots = 0, cap = 0, me = 0, n_shards = 0;
    unsigned* done = nullptr;      // last-CTA counter, zero between launches
    unsigned epoch = 0;
};

cudaError_t prefill_check(const MoeDims& d);
size_t prefill_workspace_bytes(const MoeDims& d, int T);
// T tokens (x [T][D] on the device, updated in place) through one MoE layer.
// ws: prefill_workspace_bytes() of device scratch. topk_idx / topk_w
// (optional, [T][K]) receive the routing.
// ---- expert parallelism (moe_prefill.cu): experts sharded over n_shards ranks

struct EpShape {
    int D, F, K;        // model dims (K = experts per token)
    int E;              // routed experts in total
    int n_shards;       // ranks the routed experts are split over
    int e_local;        // routed experts held by this rank (E / n_shards)
    int T_max;          // most tokens this rank routes per call
    int n_recv_cap;     // most (token, slot) rows this rank can receive per call
};

cudaError_t ep_check(const MoeDims& d, int n_shards);
size_t ep_workspace_bytes(const EpShape& s);
// Route T own tokens (global expert ids) and lay out the send buffer:
// send_rows [rows][D] (xn of each (token, slot) pair, grouped by destination
// rank), send_expert [rows] (expert id local to the destination),
// send_counts [n_shards]. Keeps xn, ids, weights and the send positions in ws.
cudaError_t launch_ep_dispatch(const MoeLayerDev& w, const MoeDims& d, const EpShape& s, unsigned char* ws,
                               const float* x, int T, float* send_rows, int32_t* send_expert, int32_t* send_counts,
                               int routed, int num_sms, unsigned long long* stats, cudaStream_t st);
// This rank's experts (w: routed arrays hold its e_local experts; dl.E =
// e_local) on n_recv received rows, plus the shared expert on its own T
// tokens of the last dispatch. out_rows [n_recv][D] in the received order.
cudaError_t launch_ep_experts(const MoeLayerDev& w, const MoeDims& dl, const EpShape& s, unsigned char* ws, int T,
                              const float* recv_rows, const int32_t* recv_expert, int n_recv, float* out_rows,
                              int routed, int num_sms, unsigned* status, cudaStream_t st);
// x[t] += shared + sum_k 1.8 w_k y_k with y_k = back_rows[send position].
cudaError_t launch_ep_combine(const MoeDims& d, const EpShape& s, unsigned char* ws, float* x, int T, int n_recv,
                              const float* back_rows, int num_sms, cudaStream_t st);
cudaError_t ep_copy_routing(const EpShape& s, unsigned char* ws, int T, int32_t* topk_idx, float* topk_w,
                            cudaStream_t st);

// ---- expert parallelism over peer memory: every rank holds one "peer
// region" of the same layout; senders write rows, ids and counts straight
// into the receiver's region and raise a flag per (sender, receiver) pair;
// the expert outputs go back the same way. Flags carry an epoch that grows
// by one per layer call, so they never need resetting.

struct EpRegion {
    int cap;                 // rows one sender may put in one receiver's region (T_max * min(K, e_local))
    size_t header;           // EpRegionHeader: the shape the region was laid out for (checked on connect)
    size_t recv_rows;        // [n_shards][cap][D] fp32: rows from sender s at [s][0 .. count)
    size_t recv_expert;      // [n_shards][cap] int32 local expert id of each received row
    size_t back_rows;        // [n_shards][cap][D] fp32: outputs of the rows this rank sent to d, at [d][j]
    size_t recv_cnt;         // [n_shards] int32 rows from each sender
    size_t flag_rows;        // [n_shards] u32: epoch of sender s's last completed row push
    size_t flag_back;        // [n_shards] u32: epoch of receiver d's last completed output push
    size_t bytes;
};

struct EpRegionHeader {
    uint32_t magic;          // kEpRegionMagic
    int32_t n_shards, cap, D, K, e_local, T_max;
    uint32_t pad;
    uint64_t bytes;
};
constexpr uint32_t kEpRegionMagic = 0x31525045u;  // "EPR1"

struct EpPeers {
    unsigned char* base[kEpMaxShards];  // every rank's region as this process addresses it
};

EpRegion ep_region_layout(const EpShape& s);
// Route, pack and push this rank's rows into the receivers' regions.
cudaError_t launch_ep_p2p_dispatch(const MoeLayerDev& w, const MoeDims& d, const EpShape& s, unsigned char* ws,
                                   const float* x, int T, int routed, int num_sms, unsigned long long* stats,
                                   const EpPeers& peers, int me, unsigned epoch, cudaStream_t st);
// Wait for every sender's rows, run this rank's experts (and the shared
// expert on its own tokens) and push the outputs back to their senders.
cudaError_t launch_ep_p2p_experts(const MoeLayerDev& w, const MoeDims& dl, const EpShape& s, unsigned char* ws,
                                  int T, int routed, int num_sms, unsigned* status, const EpPeers& peers, int me,
                                  unsigned epoch, cudaStream_t st);
// Wait for every receiver's outputs and combine them in rank order.
cudaError_t launch_ep_p2p_combine(const MoeDims& d, const EpShape& s, unsigned char* ws, float* x, int T,
                                  int num_sms, unsigned* status, const EpPeers& peers, int me, unsigned epoch,
                                  cudaStream_t st);
// Host copies of the last dispatch's per-destination send counts (ws) and
// of the per-sender receive counts (this rank's region).
cudaError_t ep_p2p_counts(const EpShape& s, unsigned char* ws, const unsigned char* region, int32_t* send_counts,
                          int32_t* recv_counts, cudaStream_t st);

cudaError_t launch_moe_prefill(const MoeLayerDev& w, const MoeDims& d, unsigned char* ws, float* x, int T,
                               int32_t* topk_idx, float* topk_w, int routed, int num_sms, unsigned* status,
                               unsigned long long* stats, cudaStream_t st);

// Record the message glm_cuda_last_error() returns for this thread.
void set_last_error(const char* msg);

// Raise kernel `fn`'s dynamic shared-memory limit to at least `bytes` on the
// current device. The attribute is per device, so the record is keyed on
// (kernel, device) under a mutex; a later call for the same pair and size
// makes no CUDA call (safe inside stream capture).
cudaError_t ensure_smem_attr(const void* fn, int bytes);

// Whether `grid` CTAs of kernel `fn` (threads per CTA, dynamic shared memory
// smem, its attribute already raised) fit the current device at once, i.e.
// every CTA of a grid-synchronising kernel can be resident together.
// cudaErrorCooperativeLaunchTooLarge if not. The occupancy query is made once
// per (kernel, device, threads, smem) under a mutex; later calls make no CUDA
// call (safe inside stream capture).
cudaError_t ensure_resident(const void* fn, int threads, int smem, int grid);

}  // namespace glmq
