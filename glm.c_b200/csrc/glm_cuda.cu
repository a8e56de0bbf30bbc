// C-ABI layer of the B200 backend (declarations and citations in
// include/glm_cuda.h). Owns the per-process device context: weights in HBM
// (planar Q8, unchanged layout), decode scratch, a private stream, and the
// host-pointer-keyed weight cache of the matvec hook.
#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <map>
#include <tuple>
#include <mutex>
#include <string>
#include <unordered_map>
#include <vector>

#include <cuda_runtime.h>

#include "glm_cuda.h"
#include "glm_internal.h"

namespace glmq {

cudaError_t ensure_smem_attr(const void* fn, int bytes) {
    static std::mutex mu;
    static std::map<std::pair<const void*, int>, int> set;
    int dev = 0;
    cudaError_t err = cudaGetDevice(&dev);
    if (err) return err;
    std::lock_guard<std::mutex> lk(mu);
    int& have = set[{fn, dev}];
    if (have >= bytes) return cudaSuccess;
    err = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
    if (!err) have = bytes;
    return err;
}

cudaError_t ensure_resident(const void* fn, int threads, int smem, int grid) {
    static std::mutex mu;
    static std::map<std::tuple<const void*, int, int, int>, int> ok;  // (fn, device, threads, smem) -> CTAs that fit
    int dev = 0, sms = 0;
    cudaError_t err = cudaGetDevice(&dev);
    if (err) return err;
    std::lock_guard<std::mutex> lk(mu);
    auto it = ok.find({fn, dev, threads, smem});
    if (it == ok.end()) {
        int per_sm = 0;
        if ((err = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, fn, threads, (size_t)smem))) return err;
        if ((err = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev))) return err;
        it = ok.emplace(std::make_tuple(fn, dev, threads, smem), per_sm * sms).first;
    }
    return it->second >= grid ? cudaSuccess : cudaErrorCooperativeLaunchTooLarge;
}

}  // namespace glmq

namespace {

struct LayerSlot {
    glmq::MoeLayerDev w;
    std::vector<void*> owned;  // device buffers this library allocated
    bool ready = false;
};

struct MatvecEntry {
    int8_t* q = nullptr;
    float* s = nullptr;
    int rows = 0, dim = 0, gs = 0;
};

// Non-MoE weights of one decoder layer (LayerAttnWeights, model.h:46-62).
struct AttnLayer {
    const float* attn_norm = nullptr;
    const float* q_a_norm = nullptr;
    const float* kv_a_norm = nullptr;
    const int8_t* q_a_q = nullptr;
    const float* q_a_s = nullptr;
    const int8_t* q_b_q = nullptr;
    const float* q_b_s = nullptr;
    const int8_t* kv_a_q = nullptr;
    const float* kv_a_s = nullptr;
    const int8_t* k_b_q = nullptr;
    const float* k_b_s = nullptr;
    const int8_t* v_b_q = nullptr;
    const float* v_b_s = nullptr;
    const int8_t* attn_out_q = nullptr;
    const float* attn_out_s = nullptr;
    std::vector<void*> owned;
    bool ready = false;
};

// The rest of the decoder (Runtime fields, model.h:87-124) and its device
// buffers (RunState, model.h:126-160).
struct Model {
    bool inited = false;
    GlmCudaModelDims d{};
    const float* output_norm = nullptr;
    const int8_t* tok_q = nullptr;
    const float* tok_s = nullptr;
    const int8_t* out_q = nullptr;
    const float* out_s = nullptr;
    const float* l0_norm = nullptr;
    const int8_t* l0_gate_q = nullptr;
    const float* l0_gate_s = nullptr;
    const int8_t* l0_up_q = nullptr;
    const float* l0_up_s = nullptr;
    const int8_t* l0_down_q = nullptr;
    const float* l0_down_s = nullptr;
    std::vector<void*> owned_globals;
    bool globals_ready = false;
    std::vector<AttnLayer> attn;
    float *x = nullptr, *xn = nullptr, *q_a = nullptr, *q_full = nullptr, *kv_a = nullptr, *att = nullptr,
          *ff_gate = nullptr, *ff_up = nullptr, *logits = nullptr, *cache_comp = nullptr, *cache_pe = nullptr;
    int *pos = nullptr, *token = nullptr, *argmax = nullptr, *prompt = nullptr, *out_ids = nullptr;
    float2* amax_part = nullptr;      // [num_sms] per-CTA argmax partials
    unsigned* amax_count = nullptr;   // argmax last-CTA counter
    int prompt_cap = 0, out_cap = 0;
    int* io_host = nullptr;  // pinned [2]: token, pos
    // batched prompt pass (glm_cuda_prefill)
    float* pf_x = nullptr;    // [pf_cap][dim] the batch's residual rows
    int* pf_pos = nullptr;    // [pf_cap] their positions
    int* pf_tok = nullptr;    // [pf_cap] their token ids (clamped as infer.c:2219)
    int* pf_host = nullptr;   // pinned [2 * pf_cap]: ids, then positions
    int pf_cap = 0;
};

struct State {
    bool inited = false;
    int device = 0;
    int num_sms = 0;
    glmq::MoeDims dims{};
    std::vector<LayerSlot> layers;
    glmq::MoeScratch scratch{};
    cudaStream_t stream = nullptr;
    // staging for the host-pointer entry points
    float* x_dev = nullptr;
    int32_t* idx_dev = nullptr;
    float* w_dev = nullptr;
    int stage_tokens = 0;
    float* mv_x = nullptr;
    float* mv_y = nullptr;
    size_t mv_x_cap = 0, mv_y_cap = 0;
    std::unordered_map<const void*, MatvecEntry> mv_cache;
    unsigned long long launches = 0;
    unsigned int* status_host = nullptr;      // pinned copy of scratch.status
    glmq::MoeLayerDev* layers_dev = nullptr;  // device copy of every slot's pointers (persistent kernel)
    bool persistent_ok = false;               // sizes fit the persistent kernel on this device
    int decode_path = GLM_CUDA_PATH_AUTO;
    // batched prefill (calls with n_tokens >= prefill_min_tokens)
    bool prefill_ok = false;   // sizes fit the prefill kernels
    int prefill_min_tokens = 32;
    int model_prefill_min = 0; // glm_cuda_generate: batched prompt pass from this many prompt tokens (0 = off)
    unsigned char* pf_ws = nullptr;
    size_t pf_ws_cap = 0;
    // expert parallelism (glm_cuda_ep_setup): routed weights hold this shard's experts
    int ep_shards = 1, ep_shard = 0;
    glmq::EpShape ep{};
    unsigned char* ep_ws = nullptr;
    int ep_layer = -1, ep_T = 0, ep_nrecv = -1;  // the layer in flight
    // expert parallelism over peer memory (glm_cuda_ep_peer_*, glm_cuda_ep_p2p_*)
    unsigned char* ep_region = nullptr;  // this rank's peer region (cudaMalloc, IPC-exportable)
    std::vector<void*> ep_opened;        // peers' regions opened with cudaIpcOpenMemHandle
    glmq::EpPeers ep_peers{};
    bool ep_connected = false;
    unsigned ep_epoch = 0;               // layer calls so far; flags carry it
    int ep_p2p_stage = 0;                // 0 idle, 1 dispatched, 2 experts done
    Model m;
};

State g;
std::mutex g_mu;
thread_local std::string g_err;

int fail(int code, const char* fmt, ...) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof buf, fmt, ap);
    va_end(ap);
    g_err = buf;
    fprintf(stderr, "[glm-cuda] %s\n", buf);
    return code;
}

#define CUDA_TRY(call)                                                                          \
    do {                                                                                        \
        cudaError_t e_ = (call);                                                                \
        if (e_ != cudaSuccess)                                                                  \
            return fail(e_ == cudaErrorMemoryAllocation ? GLM_CUDA_ERR_NOMEM : GLM_CUDA_ERR_CUDA, \
                        "%s failed: %s (%s:%d)", #call, cudaGetErrorString(e_), __FILE__, __LINE__); \
    } while (0)

template <typename T>
int dev_alloc(T** p, size_t count) {
    *p = nullptr;
    if (count == 0) return 0;
    CUDA_TRY(cudaMalloc(reinterpret_cast<void**>(p), count * sizeof(T)));
    return 0;
}

void release_layer(LayerSlot& L) {
    for (void* p : L.owned) cudaFree(p);
    L.owned.clear();
    L.w = glmq::MoeLayerDev{};
    L.ready = false;
}

void release_model() {
    Model& m = g.m;
    for (auto& A : m.attn)
        for (void* p : A.owned) cudaFree(p);
    for (void* p : m.owned_globals) cudaFree(p);
    void* bufs[] = {m.x,     m.xn,        m.q_a,      m.q_full, m.kv_a,   m.att,    m.ff_gate, m.ff_up,
                    m.logits, m.cache_comp, m.cache_pe, m.pos,    m.token,  m.argmax, m.prompt,  m.out_ids,
                    m.amax_part, m.amax_count, m.pf_x, m.pf_pos, m.pf_tok};
    for (void* p : bufs)
        if (p) cudaFree(p);
    if (m.io_host) cudaFreeHost(m.io_host);
    if (m.pf_host) cudaFreeHost(m.pf_host);
    g.m = Model{};
}

// Close the peers' regions and free this rank's (the peers must have
// stopped using it: the caller's process group agrees on that).
void release_ep_peers() {
    for (void* p : g.ep_opened) cudaIpcCloseMemHandle(p);
    g.ep_opened.clear();
    if (g.ep_region) cudaFree(g.ep_region);
    g.ep_region = nullptr;
    g.ep_peers = glmq::EpPeers{};
    g.ep_connected = false;
    g.ep_epoch = 0;
    g.ep_p2p_stage = 0;
}

void release_all() {
    release_model();
    for (auto& L : g.layers) release_layer(L);
    g.layers.clear();
    for (auto& kv : g.mv_cache) {
        cudaFree(kv.second.q);
        cudaFree(kv.second.s);
    }
    g.mv_cache.clear();
    void* bufs[] = {g.scratch.xn,     g.scratch.h,     g.scratch.center, g.scratch.bound,  g.scratch.topk_idx,
                    g.scratch.topk_w, g.scratch.counter, g.scratch.stats, g.scratch.status, g.scratch.grid_bar,
                    g.x_dev,          g.idx_dev,       g.w_dev,          g.mv_x,           g.mv_y,
                    g.layers_dev,     g.pf_ws,         g.ep_ws};
    for (void* p : bufs)
        if (p) cudaFree(p);
    release_ep_peers();
    g.ep_ws = nullptr;
    g.ep_shards = 1;
    g.ep_shard = 0;
    g.ep = glmq::EpShape{};
    g.ep_layer = -1;
    g.pf_ws = nullptr;
    g.pf_ws_cap = 0;
    g.prefill_ok = false;
    g.prefill_min_tokens = 32;
    g.model_prefill_min = 0;
    g.scratch = glmq::MoeScratch{};
    g.x_dev = nullptr;
    g.idx_dev = nullptr;
    g.w_dev = nullptr;
    g.mv_x = g.mv_y = nullptr;
    g.mv_x_cap = g.mv_y_cap = 0;
    g.stage_tokens = 0;
    g.layers_dev = nullptr;
    g.persistent_ok = false;
    g.decode_path = GLM_CUDA_PATH_AUTO;
    if (g.stream) cudaStreamDestroy(g.stream);
    g.stream = nullptr;
    if (g.status_host) cudaFreeHost(g.status_host);
    g.status_host = nullptr;
    g.inited = false;
}

// After a synchronisation that copied scratch.status into status_host: a
// nonzero word means one of the bounded waits gave up (persistent decode
// kernel: bit 2 grid barrier, 3 weight tile, 4 ring slot, 5 routing hand-off;
// prefill GEMM: bit 6 tensor-core commit).
int take_device_status() {
    const unsigned int st = g.status_host ? *g.status_host : 0u;
    if (st == 0) return 0;
    *g.status_host = 0;
    cudaMemsetAsync(g.scratch.status, 0, sizeof(unsigned int), g.stream);
    // a launch that gave up may have left its barrier words set: clear them
    cudaMemsetAsync(g.scratch.grid_bar, 0, 2 * sizeof(unsigned int), g.stream);
    if (st & 128u)
        return fail(GLM_CUDA_ERR_CUDA, "a peer rank did not answer within 4 s (expert-parallel exchange, status 0x%x)",
                    st);
    return fail(GLM_CUDA_ERR_CUDA, "the decode kernel gave up waiting (status 0x%x)", st);
}

// Mirror slot `layer`'s pointers into the device table the persistent kernel reads.
int publish_layer(int layer) {
    CUDA_TRY(cudaMemcpyAsync(g.layers_dev + layer, &g.layers[layer].w, sizeof(glmq::MoeLayerDev),
                             cudaMemcpyHostToDevice, g.stream));
    CUDA_TRY(cudaStreamSynchronize(g.stream));
    return 0;
}

bool use_persistent() { return g.persistent_ok && g.decode_path != GLM_CUDA_PATH_CHAIN; }

bool decode_kernels_ok();

// The layer glm.c's loop calls after `layer` (infer.c:1845), if it has weights.
int next_moe_layer(int layer) {
    return layer + 1 < (int)g.layers.size() && g.layers[layer + 1].ready ? layer + 1 : -1;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

bool routed_disabled_by_env() {
    // infer.c:1161-1165: set, non-empty and not starting with '0'.
    const char* v = getenv("GLM_DISABLE_MOE_ROUTED");
    return v && v[0] && v[0] != '0';
}

int check_layer(int layer, bool sharded_ok = false) {
    if (!g.inited) return fail(GLM_CUDA_ERR_STATE, "glm_cuda_init has not been called");
    if (g.ep_shards > 1 && !sharded_ok)
        return fail(GLM_CUDA_ERR_STATE, "experts are sharded (glm_cuda_ep_setup): use the glm_cuda_ep_* calls");
    if (layer < 0 || layer >= (int)g.layers.size())
        return fail(GLM_CUDA_ERR_ARG, "layer %d out of range [0,%zu)", layer, g.layers.size());
    if (!g.layers[layer].ready) return fail(GLM_CUDA_ERR_STATE, "layer %d has no weights", layer);
    return 0;
}

template <typename T>
int upload(LayerSlot& L, const T* host, size_t count, const T** out) {
    *out = nullptr;
    if (!host) return 0;
    T* d = nullptr;
    if (int rc = dev_alloc(&d, count)) return rc;
    L.owned.push_back(d);
    CUDA_TRY(cudaMemcpyAsync(d, host, count * sizeof(T), cudaMemcpyHostToDevice, g.stream));
    *out = d;
    return 0;
}

int ensure_stage(int n_tokens) {
    if (n_tokens <= g.stage_tokens) return 0;
    if (g.x_dev) cudaFree(g.x_dev);
    if (g.idx_dev) cudaFree(g.idx_dev);
    if (g.w_dev) cudaFree(g.w_dev);
    g.x_dev = nullptr;
    g.idx_dev = nullptr;
    g.w_dev = nullptr;
    g.stage_tokens = 0;
    if (int rc = dev_alloc(&g.x_dev, (size_t)n_tokens * g.dims.D)) return rc;
    if (int rc = dev_alloc(&g.idx_dev, (size_t)n_tokens * g.dims.K)) return rc;
    if (int rc = dev_alloc(&g.w_dev, (size_t)n_tokens * g.dims.K)) return rc;
    g.stage_tokens = n_tokens;
    return 0;
}

int ensure_prefill_ws(int n_tokens) {
    const size_t need = glmq::prefill_workspace_bytes(g.dims, n_tokens);
    if (need <= g.pf_ws_cap) return 0;
    if (g.pf_ws) cudaFree(g.pf_ws);
    g.pf_ws = nullptr;
    g.pf_ws_cap = 0;
    if (int rc = dev_alloc(&g.pf_ws, need)) return rc;
    g.pf_ws_cap = need;
    return 0;
}

// Per-token decode kernels: the persistent kernel takes gs = 32 and 16, the
// three-kernel chain gs = 32 only; where neither applies every call runs on
// the batched kernels.
bool chain_ok() { return g.dims.gs == 32; }
bool decode_kernels_ok() { return use_persistent() || chain_ok(); }

bool use_prefill(int n_tokens) {
    if (!g.prefill_ok) return false;
    return !decode_kernels_ok() || (g.prefill_min_tokens > 0 && n_tokens >= g.prefill_min_tokens);
}

int moe_enqueue(int layer, float* x_dev, int n_tokens, int32_t* idx_dev, float* w_dev, cudaStream_t st) {
    const LayerSlot& L = g.layers[layer];
    const int routed = routed_disabled_by_env() ? 0 : 1;
    const auto& d = g.dims;
    if (use_prefill(n_tokens)) {
        if (int rc = ensure_prefill_ws(n_tokens)) return rc;
        cudaError_t e = glmq::launch_moe_prefill(L.w, d, g.pf_ws, x_dev, n_tokens, idx_dev, w_dev, routed, g.num_sms,
                                                 g.scratch.status, g.scratch.stats, st);
        g.launches += 9;
        if (e != cudaSuccess) return fail(GLM_CUDA_ERR_CUDA, "moe prefill launch: %s", cudaGetErrorString(e));
        return 0;
    }
    if (use_persistent()) {
        for (int t = 0; t < n_tokens; ++t) {
            cudaError_t e = glmq::launch_moe_persistent(g.layers_dev, layer, 1, d, g.scratch, x_dev + (size_t)t * d.D,
                                                        idx_dev ? idx_dev + (size_t)t * d.K : nullptr,
                                                        w_dev ? w_dev + (size_t)t * d.K : nullptr, routed,
                                                        g.num_sms, st, t + 1 < n_tokens ? layer : next_moe_layer(layer));
            g.launches += 1;
            if (e != cudaSuccess)
                return fail(GLM_CUDA_ERR_CUDA, "moe persistent launch: %s", cudaGetErrorString(e));
        }
        return 0;
    }
    for (int t = 0; t < n_tokens; ++t) {
        float* xt = x_dev + (size_t)t * d.D;
        cudaError_t e = glmq::launch_moe_decode(L.w, d, g.scratch, xt, xt, routed, g.num_sms, st);
        g.launches += 3;
        if (e != cudaSuccess) return fail(GLM_CUDA_ERR_CUDA, "moe decode launch: %s", cudaGetErrorString(e));
        if (idx_dev)
            CUDA_TRY(cudaMemcpyAsync(idx_dev + (size_t)t * d.K, g.scratch.topk_idx, sizeof(int32_t) * d.K,
                                     cudaMemcpyDeviceToDevice, st));
        if (w_dev)
            CUDA_TRY(cudaMemcpyAsync(w_dev + (size_t)t * d.K, g.scratch.topk_w, sizeof(float) * d.K,
                                     cudaMemcpyDeviceToDevice, st));
    }
    return 0;
}

}  // namespace

void glmq::set_last_error(const char* msg) { g_err = msg ? msg : ""; }

namespace {

int init_locked(int device, int dim, int moe_ffn_dim, int n_routed_experts, int n_experts_used, int group_size,
                int n_layers) {
    if (g.inited) release_all();
    if (dim <= 0 || dim % 128 || moe_ffn_dim <= 0 || moe_ffn_dim % 64)
        return fail(GLM_CUDA_ERR_ARG, "unsupported dims dim=%d moe_ffn_dim=%d (need dim%%128==0, ffn%%64==0)", dim,
                    moe_ffn_dim);
    if (group_size != 32 && group_size != 16)
        return fail(GLM_CUDA_ERR_ARG, "unsupported group size %d (supported: 32, 16)", group_size);
    if (n_experts_used < 1 || n_experts_used > 8 || n_experts_used > n_routed_experts || n_routed_experts > 1024)
        return fail(GLM_CUDA_ERR_ARG, "unsupported expert counts E=%d K=%d", n_routed_experts, n_experts_used);
    if (n_layers <= 0) return fail(GLM_CUDA_ERR_ARG, "n_layers must be positive");
    int ndev = 0;
    CUDA_TRY(cudaGetDeviceCount(&ndev));
    if (device < 0 || device >= ndev) return fail(GLM_CUDA_ERR_ARG, "device %d not present (%d devices)", device, ndev);
    CUDA_TRY(cudaSetDevice(device));
    cudaDeviceProp prop{};
    CUDA_TRY(cudaGetDeviceProperties(&prop, device));
    if (prop.major < 10)
        return fail(GLM_CUDA_ERR_CUDA, "device %d is sm_%d%d; this library is built for sm_100a", device,
                    prop.major, prop.minor);
    g.device = device;
    g.num_sms = prop.multiProcessorCount;
    g.dims = glmq::MoeDims{dim, moe_ffn_dim, n_routed_experts, n_experts_used, group_size};
    CUDA_TRY(cudaStreamCreateWithFlags(&g.stream, cudaStreamNonBlocking));
    auto& s = g.scratch;
    int rc = 0;
    if ((rc = dev_alloc(&s.xn, dim)) || (rc = dev_alloc(&s.h, (size_t)(n_experts_used + 1) * moe_ffn_dim)) ||
        (rc = dev_alloc(&s.center, n_routed_experts)) || (rc = dev_alloc(&s.bound, n_routed_experts)) ||
        (rc = dev_alloc(&s.topk_idx, n_experts_used)) || (rc = dev_alloc(&s.topk_w, n_experts_used)) ||
        (rc = dev_alloc(&s.counter, 1)) || (rc = dev_alloc(&s.stats, 4)) || (rc = dev_alloc(&s.status, 1)) ||
        (rc = dev_alloc(&s.grid_bar, 2)) || (rc = dev_alloc(&g.layers_dev, n_layers))) {
        release_all();
        return rc;
    }
    CUDA_TRY(cudaMemset(s.counter, 0, sizeof(unsigned int)));
    CUDA_TRY(cudaMemset(s.stats, 0, 4 * sizeof(unsigned long long)));
    CUDA_TRY(cudaMemset(s.status, 0, sizeof(unsigned int)));
    CUDA_TRY(cudaMemset(s.grid_bar, 0, 2 * sizeof(unsigned int)));  // barrier arrivals, exited CTAs
    CUDA_TRY(cudaMemset(g.layers_dev, 0, sizeof(glmq::MoeLayerDev) * n_layers));
    CUDA_TRY(cudaHostAlloc(reinterpret_cast<void**>(&g.status_host), sizeof(unsigned int), cudaHostAllocDefault));
    *g.status_host = 0;
    g.persistent_ok = glmq::persistent_check(g.dims, g.num_sms, nullptr) == cudaSuccess;
    g.prefill_ok = glmq::prefill_check(g.dims) == cudaSuccess;
    if (group_size != 32 && !g.prefill_ok && !g.persistent_ok) {
        release_all();
        return fail(GLM_CUDA_ERR_ARG,
                    "group size %d needs the persistent or the batched kernels, and these sizes fit neither", group_size);
    }
    g.layers.assign(n_layers, LayerSlot{});
    g.launches = 0;
    g.inited = true;
    g_err.clear();
    return 0;
}

}  // namespace

extern "C" {

int glm_cuda_init(int device, int dim, int moe_ffn_dim, int n_routed_experts, int n_experts_used, int group_size,
                  int n_layers) {
    std::lock_guard<std::mutex> lk(g_mu);
    return init_locked(device, dim, moe_ffn_dim, n_routed_experts, n_experts_used, group_size, n_layers);
}

int glm_cuda_upload_moe_layer(int layer, const float* ffn_norm, const float* gate_inp, const float* exp_probs_b,
                              const int8_t* gate_sh_q, const float* gate_sh_s, const int8_t* up_sh_q,
                              const float* up_sh_s, const int8_t* down_sh_q, const float* down_sh_s,
                              const int8_t* gate_q, const float* gate_s, const int8_t* up_q, const float* up_s,
                              const int8_t* down_q, const float* down_s) {
    std::lock_guard<std::mutex> lk(g_mu);
    if (!g.inited) return fail(GLM_CUDA_ERR_STATE, "glm_cuda_init has not been called");
    if (layer < 0 || layer >= (int)g.layers.size()) return fail(GLM_CUDA_ERR_ARG, "layer %d out of range", layer);
    if (!ffn_norm || !gate_inp || !exp_probs_b || !gate_sh_q || !gate_sh_s || !up_sh_q || !up_sh_s || !down_sh_q ||
        !down_sh_s)
        return fail(GLM_CUDA_ERR_ARG, "layer %d: shared-expert/router pointers must be non-NULL", layer);
    const bool routed = gate_q != nullptr;
    if (routed && (!gate_s || !up_q || !up_s || !down_q || !down_s))
        return fail(GLM_CUDA_ERR_ARG, "layer %d: routed block is incomplete", layer);
    const auto& d = g.dims;
    const size_t D = d.D, F = d.F, gD = D / d.gs, gF = F / d.gs;
    const size_t E = d.E, Er = d.E / g.ep_shards;  // router: all experts; routed block: this shard's
    LayerSlot& L = g.layers[layer];
    release_layer(L);
    auto& w = L.w;
    int rc = 0;
    if ((rc = upload(L, ffn_norm, D, &w.ffn_norm)) || (rc = upload(L, gate_inp, E * D, &w.router)) ||
        (rc = upload(L, exp_probs_b, E, &w.router_bias)) || (rc = upload(L, gate_sh_q, F * D, &w.gate_sh_q)) ||
        (rc = upload(L, gate_sh_s, F * gD, &w.gate_sh_s)) || (rc = upload(L, up_sh_q, F * D, &w.up_sh_q)) ||
        (rc = upload(L, up_sh_s, F * gD, &w.up_sh_s)) || (rc = upload(L, down_sh_q, D * F, &w.down_sh_q)) ||
        (rc = upload(L, down_sh_s, D * gF, &w.down_sh_s))) {
        release_layer(L);
        return rc;
    }
    if (routed) {
        if ((rc = upload(L, gate_q, Er * F * D, &w.gate_q)) || (rc = upload(L, gate_s, Er * F * gD, &w.gate_s)) ||
            (rc = upload(L, up_q, Er * F * D, &w.up_q)) || (rc = upload(L, up_s, Er * F * gD, &w.up_s)) ||
            (rc = upload(L, down_q, Er * D * F, &w.down_q)) || (rc = upload(L, down_s, Er * D * gF, &w.down_s))) {
            release_layer(L);
            return rc;
        }
    }
    CUDA_TRY(cudaStreamSynchronize(g.stream));
    L.ready = true;
    return publish_layer(layer);
}

int glm_cuda_bind_moe_layer_device(int layer, const float* ffn_norm, const float* gate_inp,
                                   const float* exp_probs_b, const int8_t* gate_sh_q, const float* gate_sh_s,
                                   const int8_t* up_sh_q, const float* up_sh_s, const int8_t* down_sh_q,
                                   const float* down_sh_s, const int8_t* gate_q, const float* gate_s,
                                   const int8_t* up_q, const float* up_s, const int8_t* down_q,
                                   const float* down_s) {
    std::lock_guard<std::mutex> lk(g_mu);
    if (!g.inited) return fail(GLM_CUDA_ERR_STATE, "glm_cuda_init has not been called");
    if (layer < 0 || layer >= (int)g.layers.size()) return fail(GLM_CUDA_ERR_ARG, "layer %d out of range", layer);
    if (!ffn_norm || !gate_inp || !exp_probs_b || !gate_sh_q || !gate_sh_s || !up_sh_q || !up_sh_s || !down_sh_q ||
        !down_sh_s)
        return fail(GLM_CUDA_ERR_ARG, "layer %d: shared-expert/router pointers must be non-NULL", layer);
    if (gate_q && (!gate_s || !up_q || !up_s || !down_q || !down_s))
        return fail(GLM_CUDA_ERR_ARG, "layer %d: routed block is incomplete", layer);
    const void* ptrs[] = {ffn_norm, gate_inp, exp_probs_b, gate_sh_q, gate_sh_s, up_sh_q, up_sh_s, down_sh_q,
                          down_sh_s, gate_q, gate_s, up_q, up_s, down_q, down_s};
    for (const void* p : ptrs)
        if (!aligned16(p)) return fail(GLM_CUDA_ERR_ARG, "layer %d: device weights must be 16-byte aligned", layer);
    LayerSlot& L = g.layers[layer];
    release_layer(L);
    L.w = glmq::MoeLayerDev{ffn_norm, gate_inp, exp_probs_b, gate_sh_q, gate_sh_s, up_sh_q, up_sh_s, down_sh_q,
                            down_sh_s, gate_q, gate_s, up_q, up_s, down_q, down_s};
    L.ready = true;
    return publish_layer(layer);
}

int glm_cuda_moe_layer(int layer, float* x, int n_tokens, int32_t* topk_idx, float* topk_w) {
    std::lock_guard<std::mutex> lk(g_mu);
    if (int rc = check_layer(layer)) return rc;
    if (!x || n_tokens < 0) return fail(GLM_CUDA_ERR_ARG, "x must be non-NULL and n_tokens >= 0");
    if (n_tokens == 0) return 0;
    if (int rc = ensure_stage(n_tokens)) return rc;
    const auto& d = g.dims;
    CUDA_TRY(cudaMemcpyAsync(g.x_dev, x, sizeof(float) * (size_t)n_tokens * d.D, cudaMemcpyHostToDevice, g.stream));
    if (int rc = moe_enqueue(layer, g.x_dev, n_tokens, topk_idx ? g.idx_dev : nullptr, topk_w ? g.w_dev : nullptr,
                             g.stream))
        return rc;
    CUDA_TRY(cudaMemcpyAsync(x, g.x_dev, sizeof(float) * (size_t)n_tokens * d.D, cudaMemcpyDeviceToHost, g.stream));
    if (topk_idx)
        CUDA_TRY(cudaMemcpyAsync(topk_idx, g.idx_dev, sizeof(int32_t) * (size_t)n_tokens * d.K,
                                 cudaMemcpyDeviceToHost, g.stream));
    if (topk_w)
        CUDA_TRY(cudaMemcpyAsync(topk_w, g.w_dev, sizeof(float) * (size_t)n_tokens * d.K, cudaMemcpyDeviceToHost,
                                 g.stream));
    CUDA_TRY(cudaMemcpyAsync(g.status_host, g.scratch.status, sizeof(unsigned int), cudaMemcpyDeviceToHost,
                             g.stream));
    CUDA_TRY(cudaStreamSynchronize(g.stream));
    return take_device_status();
}

int glm_cuda_moe_layer_async(int layer, float* x_dev, int n_tokens, int32_t* topk_idx_dev, float* topk_w_dev,
                             void* stream) {
    std::lock_guard<std::mutex> lk(g_mu);
    if (int rc = check_layer(layer)) return rc;
    if (!x_dev || n_tokens < 0) return fail(GLM_CUDA_ERR_ARG, "x_dev must be non-NULL and n_tokens >= 0");
    cudaStream_t st = stream ? static_cast<cudaStream_t>(stream) : g.stream;
    return moe_enqueue(layer, x_dev, n_tokens, topk_idx_dev, topk_w_dev, st);
}

int glm_cuda_moe_layers_async(int first_layer, int n_layers, float* x_dev, int32_t* topk_idx_dev,
                              float* topk_w_dev, void* stream) {
    std::lock_guard<std::mutex> lk(g_mu);
    if (!g.inited) return fail(GLM_CUDA_ERR_STATE, "glm_cuda_init has not been called");
    if (n_layers <= 0 || first_layer < 0 || first_layer + n_layers > (int)g.layers.size())
        return fail(GLM_CUDA_ERR_ARG, "layers [%d,%d) out of range [0,%zu)", first_layer, first_layer + n_layers,
                    g.layers.size());
    for (int l = first_layer; l < first_layer + n_layers; ++l)
        if (int rc = check_layer(l)) return rc;
    if (!x_dev) return fail(GLM_CUDA_ERR_ARG, "x_dev must be non-NULL");
    if (!g.persistent_ok)
        return fail(GLM_CUDA_ERR_ARG, "these model sizes do not fit the multi-layer decode kernel on this device");
    cudaStream_t st = stream ? static_cast<cudaStream_t>(stream) : g.stream;
    const int routed = routed_disabled_by_env() ? 0 : 1;
    cudaError_t e = glmq::launch_moe_persistent(g.layers_dev, first_layer, n_layers, g.dims, g.scratch, x_dev,
                                                topk_idx_dev, topk_w_dev, routed, g.num_sms, st,
                                                next_moe_layer(first_layer + n_layers - 1));
    g.launches += 1;
    if (e != cudaSuccess) return fail(GLM_CUDA_ERR_CUDA, "moe persistent launch: %s", cudaGetErrorString(e));
    return 0;
}

int glm_cuda_set_decode_path(int path) {
    std::lock_guard<std::mutex> lk(g_mu);
    if (!g.inited) return fail(GLM_CUDA_ERR_STATE, "glm_cuda_init has not been called");
    if (path != GLM_CUDA_PATH_AUTO && path != GLM_CUDA_PATH_PERSISTENT && path != GLM_CUDA_PATH_CHAIN)
        return fail(GLM_CUDA_ERR_ARG, "unknown decode path %d", path);
    if (path == GLM_CUDA_PATH_PERSISTENT && !g.persistent_ok)
        return fail(GLM_CUDA_ERR_ARG, "these model sizes do not fit the persistent decode kernel on this device");
    if (path == GLM_CUDA_PATH_CHAIN && !chain_ok())
        return fail(GLM_CUDA_ERR_ARG, "the three-kernel decode chain takes gs = 32 only");
    g.decode_path = path;
    return 0;
}

int glm_cuda_set_prefill_tokens(int min_tokens) {
    std::lock_guard<std::mutex> lk(g_mu);
    if (!g.inited) return fail(GLM_CUDA_ERR_STATE, "glm_cuda_init has not been called");
    if (min_tokens < 0) return fail(GLM_CUDA_ERR_ARG, "min_tokens must be >= 0");
    if (min_tokens > 0 && !g.prefill_ok)
        return fail(GLM_CUDA_ERR_ARG, "these model sizes do not fit the prefill kernels");
    const int old = g.prefill_ok ? g.prefill_min_tokens : 0;
    g.prefill_min_tokens = min_tokens;
    return old;
}

int glm_cuda_ep_setup(int n_shards, int shard, int max_tokens) {
    std::lock_guard<std::mutex> lk(g_mu);
    if (!g.inited) return fail(GLM_CUDA_ERR_STATE, "glm_cuda_init has not been called");
    for (const auto& L : g.layers)
        if (L.ready) return fail(GLM_CUDA_ERR_STATE, "glm_cuda_ep_setup must come before any layer is uploaded");
    if (glmq::ep_check(g.dims, n_shards) != cudaSuccess)
        return fail(GLM_CUDA_ERR_ARG, "n_shards %d must divide n_routed_experts %d (at most 8 shards) with the "
                    "prefill kernels' sizes", n_shards, g.dims.E);
    if (shard < 0 || shard >= n_shards || max_tokens < 1)
        return fail(GLM_CUDA_ERR_ARG, "shard %d of %d, max_tokens %d", shard, n_shards, max_tokens);
    glmq::EpShape e{};
    e.D = g.dims.D;
    e.F = g.dims.F;
    e.K = g.dims.K;
    e.E = g.dims.E;
    e.n_shards = n_shards;
    e.e_local = g.dims.E / n_shards;
    e.T_max = max_tokens;
    e.n_recv_cap = n_shards * max_tokens * (g.dims.K < e.e_local ? g.dims.K : e.e_local);
    if (g.ep_ws) cudaFree(g.ep_ws);
    g.ep_ws = nullptr;
    release_ep_peers();
    const size_t ws_bytes = glmq::ep_workspace_bytes(e);
    if (int rc = dev_alloc(&g.ep_ws, ws_bytes)) return rc;
    CUDA_TRY(cudaMemset(g.ep_ws, 0, ws_bytes));  // the push / scatter-back kernels' last-CTA counters start at 0
    g.ep = e;
    g.ep_shards = n_shards;
    g.ep_shard = shard;
    g.ep_layer = -1;
    return 0;
}

int glm_cuda_ep_dispatch(int layer, const float* x_dev, int n_tokens, float* send_rows_dev,
                         int32_t* send_expert_dev, int32_t* send_counts_dev, void* stream) {
    std::lock_guard<std::mutex> lk(g_mu);
    if (int rc = check_layer(layer, true)) return rc;
    if (!g.ep_ws) return fail(GLM_CUDA_ERR_STATE, "glm_cuda_ep_setup has not been called");
    if (!x_dev || !send_rows_dev || !send_expert_dev || !send_counts_dev || n_tokens < 1 || n_tokens > g.ep.T_max)
        return fail(GLM_CUDA_ERR_ARG, "ep_dispatch: buffers must be non-NULL and 1 <= n_tokens <= %d", g.ep.T_max);
    cudaStream_t st = stream ? static_cast<cudaStream_t>(stream) : g.stream;
    cudaError_t e = glmq::launch_ep_dispatch(g.layers[layer].w, g.dims, g.ep, g.ep_ws, x_dev, n_tokens, send_rows_dev,
                                             send_expert_dev, send_counts_dev, routed_disabled_by_env() ? 0 : 1,
                                             g.num_sms, g.scratch.stats, st);
    g.launches += 5;
    if (e != cudaSuccess) return fail(GLM_CUDA_ERR_CUDA, "ep dispatch launch: %s", cudaGetErrorString(e));
    g.ep_layer = layer;
    g.ep_T = n_tokens;
    g.ep_nrecv = -1;
    return 0;
}

int glm_cuda_ep_experts(int layer, const float* recv_rows_dev, const int32_t* recv_expert_dev, int n_recv,
                        float* out_rows_dev, void* stream) {
    std::lock_guard<std::mutex> lk(g_mu);
    if (int rc = check_layer(layer, true)) return rc;
    if (g.ep_layer != layer) return fail(GLM_CUDA_ERR_STATE, "ep_experts: layer %d was not dispatched last", layer);
    if (n_recv < 0 || n_recv > g.ep.n_recv_cap || (n_recv > 0 && (!recv_rows_dev || !recv_expert_dev || !out_rows_dev)))
        return fail(GLM_CUDA_ERR_ARG, "ep_experts: n_recv %d (cap %d) or NULL buffers", n_recv, g.ep.n_recv_cap);
    cudaStream_t st = stream ? static_cast<cudaStream_t>(stream) : g.stream;
    glmq::MoeDims dl = g.dims;
    dl.E = g.ep.e_local;
    cudaError_t e = glmq::launch_ep_experts(g.layers[layer].w, dl, g.ep, g.ep_ws, g.ep_T, recv_rows_dev,
                                            recv_expert_dev, n_recv, out_rows_dev,
                                            routed_disabled_by_env() ? 0 : 1, g.num_sms, g.scratch.status, st);
    g.launches += n_recv > 0 ? 5 : 4;
    if (e != cudaSuccess) return fail(GLM_CUDA_ERR_CUDA, "ep experts launch: %s", cudaGetErrorString(e));
    g.ep_nrecv = n_recv;
    return 0;
}

int glm_cuda_ep_combine(int layer, float* x_dev, const float* back_rows_dev, int32_t* topk_idx_dev,
                        float* topk_w_dev, void* stream) {
    std::lock_guard<std::mutex> lk(g_mu);
    if (int rc = check_layer(layer, true)) return rc;
    if (g.ep_layer != layer || g.ep_nrecv < 0)
        return fail(GLM_CUDA_ERR_STATE, "ep_combine: layer %d has not been through ep_dispatch and ep_experts", layer);
    if (!x_dev) return fail(GLM_CUDA_ERR_ARG, "ep_combine: x_dev must be non-NULL");
    cudaStream_t st = stream ? static_cast<cudaStream_t>(stream) : g.stream;
    cudaError_t e = glmq::launch_ep_combine(g.dims, g.ep, g.ep_ws, x_dev, g.ep_T, g.ep_nrecv, back_rows_dev,
                                            g.num_sms, st);
    if (e == cudaSuccess) e = glmq::ep_copy_routing(g.ep, g.ep_ws, g.ep_T, topk_idx_dev, topk_w_dev, st);
    g.launches += 1;
    if (e != cudaSuccess) return fail(GLM_CUDA_ERR_CUDA, "ep combine launch: %s", cudaGetErrorString(e));
    g.ep_layer = -1;
    return 0;
}

// The shape this rank's peer region is laid out for; every rank's must match.
// (static: a second copy of this library loaded in the same process must
// not bind to the first copy's function, which reads the first copy's state)
static glmq::EpRegionHeader own_region_header() {
    const glmq::EpRegion R = glmq::ep_region_layout(g.ep);
    glmq::EpRegionHeader h{};
    h.magic = glmq::kEpRegionMagic;
    h.n_shards = g.ep.n_shards;
    h.cap = R.cap;
    h.D = g.ep.D;
    h.K = g.ep.K;
    h.e_local = g.ep.e_local;
    h.T_max = g.ep.T_max;
    h.bytes = R.bytes;
    return h;
}

int glm_cuda_ep_peer_region(void** region_dev_out, void* ipc_handle_out) {
    std::lock_guard<std::mutex> lk(g_mu);
    if (!g.ep_ws) return fail(GLM_CUDA_ERR_STATE, "glm_cuda_ep_setup has not been called");
    if (!g.ep_region) {
        const glmq::EpRegion R = glmq::ep_region_layout(g.ep);
        if (int rc = dev_alloc(&g.ep_region, R.bytes)) return rc;
        CUDA_TRY(cudaMemset(g.ep_region, 0, R.bytes));  // counts 0, flags at epoch 0
        const glmq::EpRegionHeader h = own_region_header();
        CUDA_TRY(cudaMemcpy(g.ep_region + R.header, &h, sizeof h, cudaMemcpyHostToDevice));
    }
    if (region_dev_out) *region_dev_out = g.ep_region;
    if (ipc_handle_out) {
        cudaIpcMemHandle_t h;
        CUDA_TRY(cudaIpcGetMemHandle(&h, g.ep_region));
        static_assert(sizeof(h) == GLM_CUDA_IPC_HANDLE_BYTES, "IPC handle size");
        memcpy(ipc_handle_out, &h, sizeof h);
    }
    return 0;
}

int glm_cuda_ep_peer_open(const void* ipc_handle, void** region_dev_out) {
    std::lock_guard<std::mutex> lk(g_mu);
    if (!g.inited) return fail(GLM_CUDA_ERR_STATE, "glm_cuda_init has not been called");
    if (!ipc_handle || !region_dev_out) return fail(GLM_CUDA_ERR_ARG, "ep_peer_open: NULL argument");
    cudaIpcMemHandle_t h;
    memcpy(&h, ipc_handle, sizeof h);
    void* p = nullptr;
    CUDA_TRY(cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess));
    g.ep_opened.push_back(p);
    *region_dev_out = p;
    return 0;
}

int glm_cuda_ep_peer_connect(void* const* regions) {
    std::lock_guard<std::mutex> lk(g_mu);
    if (!g.ep_ws || !g.ep_region)
        return fail(GLM_CUDA_ERR_STATE, "glm_cuda_ep_setup and glm_cuda_ep_peer_region come first");
    if (!regions) return fail(GLM_CUDA_ERR_ARG, "ep_peer_connect: regions must be non-NULL");
    if (regions[g.ep_shard] != g.ep_region)
        return fail(GLM_CUDA_ERR_ARG, "ep_peer_connect: entry %d must be this rank's own region", g.ep_shard);
    glmq::EpPeers p{};
    const glmq::EpRegionHeader mine = own_region_header();
    const size_t hdr_off = glmq::ep_region_layout(g.ep).header;
    for (int d = 0; d < g.ep_shards; ++d) {
        if (!regions[d] || (reinterpret_cast<uintptr_t>(regions[d]) & 255u))
            return fail(GLM_CUDA_ERR_ARG, "ep_peer_connect: region %d is NULL or not 256-byte aligned", d);
        // every rank's region must have this rank's layout, or the kernels'
        // stores into it would land outside it
        glmq::EpRegionHeader h{};
        CUDA_TRY(cudaMemcpy(&h, static_cast<unsigned char*>(regions[d]) + hdr_off, sizeof h, cudaMemcpyDefault));
        if (memcmp(&h, &mine, sizeof h) != 0)
            return fail(GLM_CUDA_ERR_ARG,
                        "ep_peer_connect: region %d was laid out for another shape (n_shards %d, max_tokens %d, "
                        "dim %d; this rank: %d, %d, %d)", d, h.n_shards, h.T_max, h.D, mine.n_shards, mine.T_max,
                        mine.D);
        p.base[d] = static_cast<unsigned char*>(regions[d]);
    }
    g.ep_peers = p;
    g.ep_connected = true;
    g.ep_p2p_stage = 0;
    return 0;
}

int glm_cuda_ep_p2p_dispatch(int layer, const float* x_dev, int n_tokens, void* stream) {
    std::lock_guard<std::mutex> lk(g_mu);
    if (int rc = check_layer(layer, true)) return rc;
    if (!g.ep_connected) return fail(GLM_CUDA_ERR_STATE, "glm_cuda_ep_peer_connect has not been called");
    if (g.ep_p2p_stage != 0) return fail(GLM_CUDA_ERR_STATE, "ep_p2p_dispatch: the previous layer was not combined");
    if (!x_dev || n_tokens < 1 || n_tokens > g.ep.T_max)
        return fail(GLM_CUDA_ERR_ARG, "ep_p2p_dispatch: x_dev must be non-NULL and 1 <= n_tokens <= %d", g.ep.T_max);
    cudaStream_t st = stream ? static_cast<cudaStream_t>(stream) : g.stream;
    const unsigned epoch = g.ep_epoch + 1;
    cudaError_t e = glmq::launch_ep_p2p_dispatch(g.layers[layer].w, g.dims, g.ep, g.ep_ws, x_dev, n_tokens,
                                                 routed_disabled_by_env() ? 0 : 1, g.num_sms, g.scratch.stats,
                                                 g.ep_peers, g.ep_shard, epoch, st);
    g.launches += 6;
    if (e != cudaSuccess) return fail(GLM_CUDA_ERR_CUDA, "ep p2p dispatch launch: %s", cudaGetErrorString(e));
    g.ep_epoch = epoch;
    g.ep_layer = layer;
    g.ep_T = n_tokens;
    g.ep_p2p_stage = 1;
    return 0;
}

int glm_cuda_ep_p2p_experts(int layer, void* stream) {
    std::lock_guard<std::mutex> lk(g_mu);
    if (int rc = check_layer(layer, true)) return rc;
    if (g.ep_p2p_stage != 1 || g.ep_layer != layer)
        return fail(GLM_CUDA_ERR_STATE, "ep_p2p_experts: layer %d was not dispatched last", layer);
    cudaStream_t st = stream ? static_cast<cudaStream_t>(stream) : g.stream;
    glmq::MoeDims dl = g.dims;
    dl.E = g.ep.e_local;
    cudaError_t e = glmq::launch_ep_p2p_experts(g.layers[layer].w, dl, g.ep, g.ep_ws, g.ep_T,
                                                routed_disabled_by_env() ? 0 : 1, g.num_sms, g.scratch.status,
                                                g.ep_peers, g.ep_shard, g.ep_epoch, st);
    g.launches += 6;
    if (e != cudaSuccess) return fail(GLM_CUDA_ERR_CUDA, "ep p2p experts launch: %s", cudaGetErrorString(e));
    g.ep_p2p_stage = 2;
    return 0;
}

int glm_cuda_ep_p2p_combine(int layer, float* x_dev, int32_t* topk_idx_dev, float* topk_w_dev, void* stream) {
    std::lock_guard<std::mutex> lk(g_mu);
    if (int rc = check_layer(layer, true)) return rc;
    if (g.ep_p2p_stage != 2 || g.ep_layer != layer)
        return fail(GLM_CUDA_ERR_STATE, "ep_p2p_combine: layer %d has not been through ep_p2p_experts", layer);
    if (!x_dev) return fail(GLM_CUDA_ERR_ARG, "ep_p2p_combine: x_dev must be non-NULL");
    cudaStream_t st = stream ? static_cast<cudaStream_t>(stream) : g.stream;
    cudaError_t e = glmq::launch_ep_p2p_combine(g.dims, g.ep, g.ep_ws, x_dev, g.ep_T, g.num_sms, g.scratch.status,
                                                g.ep_peers, g.ep_shard, g.ep_epoch, st);
    if (e == cudaSuccess) e = glmq::ep_copy_routing(g.ep, g.ep_ws, g.ep_T, topk_idx_dev, topk_w_dev, st);
    g.launches += 2;
    if (e != cudaSuccess) return fail(GLM_CUDA_ERR_CUDA, "ep p2p combine launch: %s", cudaGetErrorString(e));
    g.ep_layer = -1;
    g.ep_p2p_stage = 0;
    return 0;
}

int glm_cuda_ep_p2p_counts(int32_t* send_counts, int32_t* recv_counts) {
    std::lock_guard<std::mutex> lk(g_mu);
    if (!g.ep_connected) return fail(GLM_CUDA_ERR_STATE, "glm_cuda_ep_peer_connect has not been called");
    if (!send_counts || !recv_counts) return fail(GLM_CUDA_ERR_ARG, "ep_p2p_counts: NULL argument");
    CUDA_TRY(cudaDeviceSynchronize());  // the layer may have run on the caller's stream
    cudaError_t e = glmq::ep_p2p_counts(g.ep, g.ep_ws, g.ep_region, send_counts, recv_counts, g.stream);
    if (e != cudaSuccess) return fail(GLM_CUDA_ERR_CUDA, "ep p2p counts: %s", cudaGetErrorString(e));
    return 0;
}

int glm_cuda_ep_status(void) {
    std::lock_guard<std::mutex> lk(g_mu);
    if (!g.inited) return fail(GLM_CUDA_ERR_STATE, "glm_cuda_init has not been called");
    CUDA_TRY(cudaMemcpyAsync(g.status_host, g.scratch.status, sizeof(unsigned int), cudaMemcpyDeviceToHost,
                             g.stream));
    CUDA_TRY(cudaStreamSynchronize(g.stream));
    return take_device_status();
}

int glm_cuda_decode_path(void) {
    std::lock_guard<std::mutex> lk(g_mu);
    if (!g.inited) return fail(GLM_CUDA_ERR_STATE, "glm_cuda_init has not been called");
    if (!decode_kernels_ok()) return GLM_CUDA_PATH_BATCHED;
    return use_persistent() ? GLM_CUDA_PATH_PERSISTENT : GLM_CUDA_PATH_CHAIN;
}

int glm_cuda_moe_layer_profile(int layer, float* x_dev, float ms_out[3]) {
    std::lock_guard<std::mutex> lk(g_mu);
    if (int rc = check_layer(layer)) return rc;
    if (!x_dev || !ms_out) return fail(GLM_CUDA_ERR_ARG, "x_dev and ms_out must be non-NULL");
    if (!chain_ok()) return fail(GLM_CUDA_ERR_ARG, "the three-kernel decode chain takes gs = 32 only");
    cudaEvent_t ev[4] = {nullptr, nullptr, nullptr, nullptr};
    for (auto& e : ev) CUDA_TRY(cudaEventCreate(&e));
    const int routed = routed_disabled_by_env() ? 0 : 1;
    cudaError_t err = glmq::launch_moe_decode(g.layers[layer].w, g.dims, g.scratch, x_dev, x_dev, routed,
                                              g.num_sms, g.stream, ev);
    g.launches += 3;
    if (err == cudaSuccess) err = cudaEventSynchronize(ev[3]);
    for (int i = 0; err == cudaSuccess && i < 3; ++i) err = cudaEventElapsedTime(&ms_out[i], ev[i], ev[i + 1]);
    for (auto& e : ev) cudaEventDestroy(e);
    if (err != cudaSuccess) return fail(GLM_CUDA_ERR_CUDA, "moe profile: %s", cudaGetErrorString(err));
    return 0;
}

int glm_cuda_matvec_q80(const int8_t* qmat, const float* smat, const float* x, float* y, int rows, int dim, int gs) {
    std::lock_guard<std::mutex> lk(g_mu);
    if (!g.inited) return fail(GLM_CUDA_ERR_STATE, "glm_cuda_init has not been called");
    if (!qmat || !smat || !x || !y || rows <= 0 || dim <= 0) return fail(GLM_CUDA_ERR_ARG, "bad matvec arguments");
    if ((gs != 32 && gs != 16) || dim % 64)
        return fail(GLM_CUDA_ERR_ARG, "matvec: unsupported gs=%d dim=%d", gs, dim);
    auto it = g.mv_cache.find(qmat);
    if (it != g.mv_cache.end() && (it->second.rows != rows || it->second.dim != dim || it->second.gs != gs)) {
        cudaFree(it->second.q);
        cudaFree(it->second.s);
        g.mv_cache.erase(it);
        it = g.mv_cache.end();
    }
    if (it == g.mv_cache.end()) {
        MatvecEntry m;
        m.rows = rows;
        m.dim = dim;
        m.gs = gs;
        if (int rc = dev_alloc(&m.q, (size_t)rows * dim)) return rc;
        if (int rc = dev_alloc(&m.s, (size_t)rows * (dim / gs))) {
            cudaFree(m.q);
            return rc;
        }
        CUDA_TRY(cudaMemcpyAsync(m.q, qmat, (size_t)rows * dim, cudaMemcpyHostToDevice, g.stream));
        CUDA_TRY(cudaMemcpyAsync(m.s, smat, sizeof(float) * (size_t)rows * (dim / gs), cudaMemcpyHostToDevice,
                                 g.stream));
        it = g.mv_cache.emplace(qmat, m).first;
    }
    if ((size_t)dim > g.mv_x_cap) {
        if (g.mv_x) cudaFree(g.mv_x);
        g.mv_x = nullptr;
        g.mv_x_cap = 0;
        if (int rc = dev_alloc(&g.mv_x, (size_t)dim)) return rc;
        g.mv_x_cap = dim;
    }
    if ((size_t)rows > g.mv_y_cap) {
        if (g.mv_y) cudaFree(g.mv_y);
        g.mv_y = nullptr;
        g.mv_y_cap = 0;
        if (int rc = dev_alloc(&g.mv_y, (size_t)rows)) return rc;
        g.mv_y_cap = rows;
    }
    CUDA_TRY(cudaMemcpyAsync(g.mv_x, x, sizeof(float) * dim, cudaMemcpyHostToDevice, g.stream));
    cudaError_t e = glmq::launch_q80_matvec(it->second.q, it->second.s, g.mv_x, g.mv_y, rows, dim, gs, g.num_sms,
                                            g.stream);
    g.launches += 1;
    if (e != cudaSuccess) return fail(GLM_CUDA_ERR_CUDA, "matvec launch: %s", cudaGetErrorString(e));
    CUDA_TRY(cudaMemcpyAsync(y, g.mv_y, sizeof(float) * rows, cudaMemcpyDeviceToHost, g.stream));
    CUDA_TRY(cudaStreamSynchronize(g.stream));
    return 0;
}

int glm_cuda_matvec_q80_async(const int8_t* q_dev, const float* s_dev, const float* x_dev, float* y_dev, int rows,
                              int dim, int gs, void* stream) {
    std::lock_guard<std::mutex> lk(g_mu);
    if (!g.inited) return fail(GLM_CUDA_ERR_STATE, "glm_cuda_init has not been called");
    if (!q_dev || !s_dev || !x_dev || !y_dev || rows <= 0 || dim <= 0)
        return fail(GLM_CUDA_ERR_ARG, "bad matvec arguments");
    if ((gs != 32 && gs != 16) || dim % 64)
        return fail(GLM_CUDA_ERR_ARG, "matvec: unsupported gs=%d dim=%d", gs, dim);
    cudaStream_t st = stream ? static_cast<cudaStream_t>(stream) : g.stream;
    cudaError_t e = glmq::launch_q80_matvec(q_dev, s_dev, x_dev, y_dev, rows, dim, gs, g.num_sms, st);
    g.launches += 1;
    if (e != cudaSuccess) return fail(GLM_CUDA_ERR_CUDA, "matvec launch: %s", cudaGetErrorString(e));
    return 0;
}

int glm_cuda_synchronize(void) {
    std::lock_guard<std::mutex> lk(g_mu);
    if (!g.inited) return fail(GLM_CUDA_ERR_STATE, "glm_cuda_init has not been called");
    CUDA_TRY(cudaDeviceSynchronize());
    CUDA_TRY(cudaGetLastError());
    CUDA_TRY(cudaMemcpy(g.status_host, g.scratch.status, sizeof(unsigned int), cudaMemcpyDeviceToHost));
    return take_device_status();
}

int glm_cuda_route_stats(uint64_t out[4]) {
    std::lock_guard<std::mutex> lk(g_mu);
    if (!g.inited) return fail(GLM_CUDA_ERR_STATE, "glm_cuda_init has not been called");
    if (!out) return fail(GLM_CUDA_ERR_ARG, "out must be non-NULL");
    unsigned long long h[4] = {0, 0, 0, 0};
    CUDA_TRY(cudaDeviceSynchronize());
    CUDA_TRY(cudaMemcpy(h, g.scratch.stats, sizeof h, cudaMemcpyDeviceToHost));
    for (int i = 0; i < 4; ++i) out[i] = h[i];
    return 0;
}

uint64_t glm_cuda_launch_count(void) {
    std::lock_guard<std::mutex> lk(g_mu);
    return g.launches;
}

const char* glm_cuda_last_error(void) { return g_err.c_str(); }

void glm_cuda_free(void) {
    std::lock_guard<std::mutex> lk(g_mu);
    if (g.inited) {
        cudaStreamSynchronize(g.stream);
        release_all();
    }
}

}  // extern "C"

// ------------------------------------------------------------ full decoder

namespace {

template <typename T>
int put(std::vector<void*>& owned, bool copy, const T* src, size_t count, const T** out) {
    *out = nullptr;
    if (!src) return 0;
    if (!copy) {
        if (reinterpret_cast<uintptr_t>(src) & 15u) return fail(GLM_CUDA_ERR_ARG, "device weights must be 16-byte aligned");
        *out = src;
        return 0;
    }
    T* d = nullptr;
    if (int rc = dev_alloc(&d, count)) return rc;
    owned.push_back(d);
    CUDA_TRY(cudaMemcpyAsync(d, src, count * sizeof(T), cudaMemcpyHostToDevice, g.stream));
    *out = d;
    return 0;
}

int check_model() {
    if (!g.inited || !g.m.inited) return fail(GLM_CUDA_ERR_STATE, "glm_cuda_model_init has not been called");
    if (!g.m.globals_ready) return fail(GLM_CUDA_ERR_STATE, "model globals (embedding, LM head, layer-0 FFN) missing");
    for (int l = 0; l < g.m.d.n_layers; ++l) {
        if (!g.m.attn[l].ready) return fail(GLM_CUDA_ERR_STATE, "attention layer %d has no weights", l);
        if (l > 0 && !g.layers[l].ready) return fail(GLM_CUDA_ERR_STATE, "MoE layer %d has no weights", l);
    }
    return 0;
}

// The decoder's matvecs stage their weight rows in shared memory before the
// launch wait (launch_q80_matvec's `stage`): measured 1.5 % faster per token
// on the config-2 decode than streaming them after it.
constexpr bool kStage = true;

#define LAUNCH_TRY(call)                                                                              \
    do {                                                                                              \
        cudaError_t e_ = (call);                                                                      \
        if (e_ != cudaSuccess) return fail(GLM_CUDA_ERR_CUDA, "%s: %s", #call, cudaGetErrorString(e_)); \
    } while (0)

// One decode step at the device-resident (token, pos): glm_cpu_forward_token
// (infer.c:1767-1901) with every linear layer on the GPU; logits and the
// argmax land in device memory.
int enqueue_step(cudaStream_t st) {
    Model& m = g.m;
    const GlmCudaModelDims& d = m.d;
    const int D = d.dim, gs = d.group_size, ns = g.num_sms;
    const int routed = routed_disabled_by_env() ? 0 : 1;
    const float kq_scale = 1.0f / sqrtf((float)d.head_k_dim);
    LAUNCH_TRY(glmq::launch_embed(m.tok_q, m.tok_s, m.token, m.x, D, gs, st));
    for (int l = 0; l < d.n_layers; ++l) {
        const AttnLayer& A = m.attn[l];
        // MLA attention (infer.c:978-1065)
        // (the rmsnorms of x and q_a run fused into the matvecs that read them)
        // q_a and kv_a both read rmsnorm(x) * attn_norm: one launch
        // (their weight rows staged in shared memory while the kernel before
        // them drains: kStage)
        LAUNCH_TRY(glmq::launch_q80_matvec2(A.q_a_q, A.q_a_s, m.q_a, d.q_lora_rank, A.kv_a_q, A.kv_a_s, m.kv_a,
                                            d.kv_lora_rank + d.rope_dim, m.x, D, gs, ns, st, A.attn_norm, kStage));
        LAUNCH_TRY(glmq::launch_q80_matvec(A.q_b_q, A.q_b_s, m.q_a, m.q_full, d.n_heads * d.head_k_dim, d.q_lora_rank,
                                           gs, ns, st, false, A.q_a_norm, kStage));
        float* comp = m.cache_comp + (size_t)l * d.cache_cap * d.kv_lora_rank;
        float* pe = m.cache_pe + (size_t)l * d.cache_cap * d.rope_dim;
        glmq::MlaArgs ma{m.q_full,       m.kv_a,        A.kv_a_norm,  comp,          pe,
                         A.k_b_q,        A.k_b_s,       A.v_b_q,      A.v_b_s,       m.att,
                         m.pos,          d.qk_nope_dim, d.rope_dim,   d.head_k_dim,  d.kv_lora_rank,
                         d.v_head_dim,   gs,            d.cache_cap,  kq_scale};
        LAUNCH_TRY(glmq::launch_mla(ma, d.n_heads, st));
        LAUNCH_TRY(glmq::launch_q80_matvec(A.attn_out_q, A.attn_out_s, m.att, m.x, D, d.n_heads * d.v_head_dim, gs,
                                           ns, st, true, nullptr, kStage));
        if (l == 0) {
            // dense SwiGLU FFN (infer.c:1067-1085)
            LAUNCH_TRY(glmq::launch_q80_matvec(m.l0_gate_q, m.l0_gate_s, m.x, m.ff_gate, d.hidden_dim, D, gs, ns, st,
                                               false, m.l0_norm, kStage));
            LAUNCH_TRY(glmq::launch_q80_matvec(m.l0_up_q, m.l0_up_s, m.x, m.ff_up, d.hidden_dim, D, gs, ns, st, false,
                                               m.l0_norm, kStage));
            LAUNCH_TRY(glmq::launch_silu_mul(m.ff_gate, m.ff_up, d.hidden_dim, ns, st));
            LAUNCH_TRY(glmq::launch_q80_matvec(m.l0_down_q, m.l0_down_s, m.ff_gate, m.x, D, d.hidden_dim, gs, ns, st,
                                               true));
            g.launches += 4;
        } else if (!decode_kernels_ok()) {
            // gs = 16: the batched kernels with one token (workspace sized at model init)
            LAUNCH_TRY(glmq::launch_moe_prefill(g.layers[l].w, g.dims, g.pf_ws, m.x, 1, nullptr, nullptr, routed, ns,
                                                g.scratch.status, g.scratch.stats, st));
            g.launches += 9;
        } else if (use_persistent()) {
            LAUNCH_TRY(glmq::launch_moe_persistent(g.layers_dev, l, 1, g.dims, g.scratch, m.x, nullptr, nullptr,
                                                   routed, ns, st, l + 1 < d.n_layers ? l + 1 : -1));
            g.launches += 1;
        } else {
            LAUNCH_TRY(glmq::launch_moe_decode(g.layers[l].w, g.dims, g.scratch, m.x, m.x, routed, ns, st));
            g.launches += 3;
        }
        g.launches += 4;  // q_a + kv_a, q_b, MLA, attention output
    }
    // final norm (fused), LM head, argmax (infer.c:1888-1893, 1218-1228)
    LAUNCH_TRY(glmq::launch_q80_matvec(m.out_q, m.out_s, m.x, m.logits, d.vocab_size, D, gs, ns, st, false,
                                       m.output_norm));
    LAUNCH_TRY(glmq::launch_argmax(m.logits, d.vocab_size, m.amax_part, m.amax_count, ns, m.argmax, st));
    g.launches += 3;  // embedding, LM head, argmax
    return 0;
}

// Positions pf_pos[0 .. T) (consecutive, ids in pf_tok) through every layer
// as one batch, layer by layer: per layer each token's attention in position
// order -- the causal order of infer.c's token loop (infer.c:2190-2233), so
// token t reads the cache rows that this pass wrote for the tokens before it
// -- then the FFN of all T tokens at once: the batched MoE kernels read each
// touched expert's weights once per layer instead of once per token. The
// attention kernels are the decode step's, so the cache rows are the ones
// token-by-token decoding writes. Leaves the batch's residual rows in pf_x.
int enqueue_prefill(int T, cudaStream_t st) {
    Model& m = g.m;
    const GlmCudaModelDims& d = m.d;
    const int D = d.dim, gs = d.group_size, ns = g.num_sms;
    const int routed = routed_disabled_by_env() ? 0 : 1;
    const float kq_scale = 1.0f / sqrtf((float)d.head_k_dim);
    for (int t = 0; t < T; ++t)
        LAUNCH_TRY(glmq::launch_embed(m.tok_q, m.tok_s, m.pf_tok + t, m.pf_x + (size_t)t * D, D, gs, st));
    g.launches += (unsigned long long)T;
    for (int l = 0; l < d.n_layers; ++l) {
        const AttnLayer& A = m.attn[l];
        float* comp = m.cache_comp + (size_t)l * d.cache_cap * d.kv_lora_rank;
        float* pe = m.cache_pe + (size_t)l * d.cache_cap * d.rope_dim;
        for (int t = 0; t < T; ++t) {
            float* xt = m.pf_x + (size_t)t * D;
            LAUNCH_TRY(glmq::launch_q80_matvec2(A.q_a_q, A.q_a_s, m.q_a, d.q_lora_rank, A.kv_a_q, A.kv_a_s, m.kv_a,
                                                d.kv_lora_rank + d.rope_dim, xt, D, gs, ns, st, A.attn_norm, kStage));
            LAUNCH_TRY(glmq::launch_q80_matvec(A.q_b_q, A.q_b_s, m.q_a, m.q_full, d.n_heads * d.head_k_dim,
                                               d.q_lora_rank, gs, ns, st, false, A.q_a_norm, kStage));
            glmq::MlaArgs ma{m.q_full,       m.kv_a,        A.kv_a_norm,  comp,          pe,
                             A.k_b_q,        A.k_b_s,       A.v_b_q,      A.v_b_s,       m.att,
                             m.pf_pos + t,   d.qk_nope_dim, d.rope_dim,   d.head_k_dim,  d.kv_lora_rank,
                             d.v_head_dim,   gs,            d.cache_cap,  kq_scale};
            LAUNCH_TRY(glmq::launch_mla(ma, d.n_heads, st));
            LAUNCH_TRY(glmq::launch_q80_matvec(A.attn_out_q, A.attn_out_s, m.att, xt, D, d.n_heads * d.v_head_dim,
                                               gs, ns, st, true, nullptr, kStage));
            if (l == 0) {  // dense SwiGLU FFN (infer.c:1067-1085), token by token
                LAUNCH_TRY(glmq::launch_q80_matvec(m.l0_gate_q, m.l0_gate_s, xt, m.ff_gate, d.hidden_dim, D, gs, ns,
                                                   st, false, m.l0_norm, kStage));
                LAUNCH_TRY(glmq::launch_q80_matvec(m.l0_up_q, m.l0_up_s, xt, m.ff_up, d.hidden_dim, D, gs, ns, st,
                                                   false, m.l0_norm, kStage));
                LAUNCH_TRY(glmq::launch_silu_mul(m.ff_gate, m.ff_up, d.hidden_dim, ns, st));
                LAUNCH_TRY(glmq::launch_q80_matvec(m.l0_down_q, m.l0_down_s, m.ff_gate, xt, D, d.hidden_dim, gs, ns,
                                                   st, true));
                g.launches += 4;
            }
        }
        g.launches += 4ull * (unsigned long long)T;  // q_a + kv_a, q_b, MLA, attention output
        if (l > 0) {
            LAUNCH_TRY(glmq::launch_moe_prefill(g.layers[l].w, g.dims, g.pf_ws, m.pf_x, T, nullptr, nullptr, routed,
                                                ns, g.scratch.status, g.scratch.stats, st));
            g.launches += 9;
        }
    }
    return 0;
}

// Room for a batch of T prompt tokens and its positions / ids.
int ensure_model_prefill(int T) {
    Model& m = g.m;
    if (!g.prefill_ok) return fail(GLM_CUDA_ERR_STATE, "the batched prompt pass needs the prefill kernels (unsupported dims)");
    if (int rc = ensure_prefill_ws(T)) return rc;
    if (T <= m.pf_cap) return 0;
    if (m.pf_x) cudaFree(m.pf_x);
    if (m.pf_pos) cudaFree(m.pf_pos);
    if (m.pf_tok) cudaFree(m.pf_tok);
    if (m.pf_host) cudaFreeHost(m.pf_host);
    m.pf_x = nullptr;
    m.pf_pos = m.pf_tok = m.pf_host = nullptr;
    m.pf_cap = 0;
    if (int rc = dev_alloc(&m.pf_x, (size_t)T * m.d.dim)) return rc;
    if (int rc = dev_alloc(&m.pf_pos, T)) return rc;
    if (int rc = dev_alloc(&m.pf_tok, T)) return rc;
    CUDA_TRY(cudaHostAlloc(reinterpret_cast<void**>(&m.pf_host), 2 * sizeof(int) * (size_t)T, cudaHostAllocDefault));
    m.pf_cap = T;
    return 0;
}

// Stage the ids (clamped to the vocabulary as infer.c:2219) and positions
// start_pos .. start_pos + T - 1 of a batch.
int stage_prefill_batch(const int32_t* tokens, int T, int start_pos, cudaStream_t st) {
    Model& m = g.m;
    for (int t = 0; t < T; ++t) {
        const int id = tokens[t];
        m.pf_host[t] = (id < 0 || id >= m.d.vocab_size) ? 0 : id;
        m.pf_host[m.pf_cap + t] = start_pos + t;
    }
    CUDA_TRY(cudaMemcpyAsync(m.pf_tok, m.pf_host, sizeof(int) * (size_t)T, cudaMemcpyHostToDevice, st));
    CUDA_TRY(cudaMemcpyAsync(m.pf_pos, m.pf_host + m.pf_cap, sizeof(int) * (size_t)T, cudaMemcpyHostToDevice, st));
    return 0;
}

int status_check_sync() {
    CUDA_TRY(cudaMemcpyAsync(g.status_host, g.scratch.status, sizeof(unsigned int), cudaMemcpyDeviceToHost, g.stream));
    CUDA_TRY(cudaStreamSynchronize(g.stream));
    return take_device_status();
}

}  // namespace

extern "C" {

int glm_cuda_model_init(int device, const GlmCudaModelDims* dims) {
    std::lock_guard<std::mutex> lk(g_mu);
    if (!dims) return fail(GLM_CUDA_ERR_ARG, "dims must be non-NULL");
    const GlmCudaModelDims d = *dims;
    if (d.n_layers < 2 || d.n_heads <= 0 || d.vocab_size <= 0 || d.cache_cap <= 0 || d.hidden_dim <= 0)
        return fail(GLM_CUDA_ERR_ARG, "bad model dims");
    if (d.head_k_dim != d.qk_nope_dim + d.rope_dim || d.rope_dim % 2 || d.qk_nope_dim % 32 || d.kv_lora_rank % 64 ||
        d.q_lora_rank % 64 || (d.n_heads * d.v_head_dim) % 64 || d.hidden_dim % 64 ||
        (d.group_size != 32 && d.group_size != 16))
        return fail(GLM_CUDA_ERR_ARG, "unsupported attention/FFN dims");
    if (int rc = init_locked(device, d.dim, d.moe_ffn_dim, d.n_routed_experts, d.n_experts_used, d.group_size,
                             d.n_layers))
        return rc;
    Model& m = g.m;
    m.d = d;
    m.attn.assign(d.n_layers, AttnLayer{});
    const size_t cache = (size_t)d.n_layers * d.cache_cap;
    int rc = 0;
    if ((rc = dev_alloc(&m.x, d.dim)) || (rc = dev_alloc(&m.xn, d.dim)) || (rc = dev_alloc(&m.q_a, d.q_lora_rank)) ||
        (rc = dev_alloc(&m.q_full, (size_t)d.n_heads * d.head_k_dim)) ||
        (rc = dev_alloc(&m.kv_a, d.kv_lora_rank + d.rope_dim)) ||
        (rc = dev_alloc(&m.att, (size_t)d.n_heads * d.v_head_dim)) || (rc = dev_alloc(&m.ff_gate, d.hidden_dim)) ||
        (rc = dev_alloc(&m.ff_up, d.hidden_dim)) || (rc = dev_alloc(&m.logits, d.vocab_size)) ||
        (rc = dev_alloc(&m.cache_comp, cache * d.kv_lora_rank)) || (rc = dev_alloc(&m.cache_pe, cache * d.rope_dim)) ||
        (rc = dev_alloc(&m.pos, 1)) || (rc = dev_alloc(&m.token, 1)) || (rc = dev_alloc(&m.argmax, 1)) ||
        (rc = dev_alloc(&m.amax_part, g.num_sms)) || (rc = dev_alloc(&m.amax_count, 1))) {
        release_all();
        return rc;
    }
    CUDA_TRY(cudaMemset(m.amax_count, 0, sizeof(unsigned)));
    CUDA_TRY(cudaMemset(m.cache_comp, 0, sizeof(float) * cache * d.kv_lora_rank));
    CUDA_TRY(cudaMemset(m.cache_pe, 0, sizeof(float) * cache * d.rope_dim));
    CUDA_TRY(cudaHostAlloc(reinterpret_cast<void**>(&m.io_host), 2 * sizeof(int), cudaHostAllocDefault));
    if (!decode_kernels_ok())
        if (int rc2 = ensure_prefill_ws(1)) return rc2;  // the MoE layers of a captured step run batched
    m.inited = true;
    return 0;
}

static int model_globals(bool copy, const float* output_norm, const int8_t* tok_q, const float* tok_s,
                         const int8_t* out_q, const float* out_s, const float* l0_norm, const int8_t* gq,
                         const float* gsc, const int8_t* uq, const float* usc, const int8_t* dq, const float* dsc) {
    std::lock_guard<std::mutex> lk(g_mu);
    if (!g.inited || !g.m.inited) return fail(GLM_CUDA_ERR_STATE, "glm_cuda_model_init has not been called");
    const void* ptrs[] = {output_norm, tok_q, tok_s, out_q, out_s, l0_norm, gq, gsc, uq, usc, dq, dsc};
    for (const void* p : ptrs)
        if (!p) return fail(GLM_CUDA_ERR_ARG, "model globals must be non-NULL");
    Model& m = g.m;
    for (void* p : m.owned_globals) cudaFree(p);
    m.owned_globals.clear();
    m.globals_ready = false;
    const GlmCudaModelDims& d = m.d;
    const size_t D = d.dim, V = d.vocab_size, H = d.hidden_dim, gsz = d.group_size;
    auto& o = m.owned_globals;
    int rc = 0;
    if ((rc = put(o, copy, output_norm, D, &m.output_norm)) || (rc = put(o, copy, tok_q, V * D, &m.tok_q)) ||
        (rc = put(o, copy, tok_s, V * D / gsz, &m.tok_s)) || (rc = put(o, copy, out_q, V * D, &m.out_q)) ||
        (rc = put(o, copy, out_s, V * D / gsz, &m.out_s)) || (rc = put(o, copy, l0_norm, D, &m.l0_norm)) ||
        (rc = put(o, copy, gq, H * D, &m.l0_gate_q)) || (rc = put(o, copy, gsc, H * D / gsz, &m.l0_gate_s)) ||
        (rc = put(o, copy, uq, H * D, &m.l0_up_q)) || (rc = put(o, copy, usc, H * D / gsz, &m.l0_up_s)) ||
        (rc = put(o, copy, dq, D * H, &m.l0_down_q)) || (rc = put(o, copy, dsc, D * H / gsz, &m.l0_down_s)))
        return rc;
    CUDA_TRY(cudaStreamSynchronize(g.stream));
    m.globals_ready = true;
    return 0;
}

int glm_cuda_upload_model_globals(const float* output_norm, const int8_t* tok_q, const float* tok_s,
                                  const int8_t* out_q, const float* out_s, const float* l0_ffn_norm,
                                  const int8_t* l0_gate_q, const float* l0_gate_s, const int8_t* l0_up_q,
                                  const float* l0_up_s, const int8_t* l0_down_q, const float* l0_down_s) {
    return model_globals(true, output_norm, tok_q, tok_s, out_q, out_s, l0_ffn_norm, l0_gate_q, l0_gate_s, l0_up_q,
                         l0_up_s, l0_down_q, l0_down_s);
}

int glm_cuda_bind_model_globals_device(const float* output_norm, const int8_t* tok_q, const float* tok_s,
                                       const int8_t* out_q, const float* out_s, const float* l0_ffn_norm,
                                       const int8_t* l0_gate_q, const float* l0_gate_s, const int8_t* l0_up_q,
                                       const float* l0_up_s, const int8_t* l0_down_q, const float* l0_down_s) {
    return model_globals(false, output_norm, tok_q, tok_s, out_q, out_s, l0_ffn_norm, l0_gate_q, l0_gate_s, l0_up_q,
                         l0_up_s, l0_down_q, l0_down_s);
}

static int attn_layer(bool copy, int layer, const void* const* p) {
    std::lock_guard<std::mutex> lk(g_mu);
    if (!g.inited || !g.m.inited) return fail(GLM_CUDA_ERR_STATE, "glm_cuda_model_init has not been called");
    Model& m = g.m;
    if (layer < 0 || layer >= m.d.n_layers) return fail(GLM_CUDA_ERR_ARG, "attention layer %d out of range", layer);
    for (int i = 0; i < 15; ++i)
        if (!p[i]) return fail(GLM_CUDA_ERR_ARG, "attention layer %d: pointer %d is NULL", layer, i);
    AttnLayer& A = m.attn[layer];
    for (void* q : A.owned) cudaFree(q);
    A = AttnLayer{};
    const GlmCudaModelDims& d = m.d;
    const size_t D = d.dim, ql = d.q_lora_rank, kvl = d.kv_lora_rank, H = d.n_heads, gsz = d.group_size;
    const size_t qb_rows = H * d.head_k_dim, kva_rows = kvl + d.rope_dim, out_cols = H * d.v_head_dim;
    auto& o = A.owned;
    int rc = 0;
    if ((rc = put(o, copy, (const float*)p[0], D, &A.attn_norm)) ||
        (rc = put(o, copy, (const float*)p[1], ql, &A.q_a_norm)) ||
        (rc = put(o, copy, (const float*)p[2], kvl, &A.kv_a_norm)) ||
        (rc = put(o, copy, (const int8_t*)p[3], ql * D, &A.q_a_q)) ||
        (rc = put(o, copy, (const float*)p[4], ql * D / gsz, &A.q_a_s)) ||
        (rc = put(o, copy, (const int8_t*)p[5], qb_rows * ql, &A.q_b_q)) ||
        (rc = put(o, copy, (const float*)p[6], qb_rows * ql / gsz, &A.q_b_s)) ||
        (rc = put(o, copy, (const int8_t*)p[7], kva_rows * D, &A.kv_a_q)) ||
        (rc = put(o, copy, (const float*)p[8], kva_rows * D / gsz, &A.kv_a_s)) ||
        (rc = put(o, copy, (const int8_t*)p[9], H * kvl * d.qk_nope_dim, &A.k_b_q)) ||
        (rc = put(o, copy, (const float*)p[10], H * kvl * d.qk_nope_dim / gsz, &A.k_b_s)) ||
        (rc = put(o, copy, (const int8_t*)p[11], H * d.v_head_dim * kvl, &A.v_b_q)) ||
        (rc = put(o, copy, (const float*)p[12], H * d.v_head_dim * kvl / gsz, &A.v_b_s)) ||
        (rc = put(o, copy, (const int8_t*)p[13], D * out_cols, &A.attn_out_q)) ||
        (rc = put(o, copy, (const float*)p[14], D * out_cols / gsz, &A.attn_out_s)))
        return rc;
    CUDA_TRY(cudaStreamSynchronize(g.stream));
    A.ready = true;
    return 0;
}

int glm_cuda_upload_attn_layer(int layer, const float* attn_norm, const float* q_a_norm, const float* kv_a_norm,
                               const int8_t* q_a_q, const float* q_a_s, const int8_t* q_b_q, const float* q_b_s,
                               const int8_t* kv_a_q, const float* kv_a_s, const int8_t* k_b_q, const float* k_b_s,
                               const int8_t* v_b_q, const float* v_b_s, const int8_t* attn_out_q,
                               const float* attn_out_s) {
    const void* p[15] = {attn_norm, q_a_norm, kv_a_norm, q_a_q, q_a_s, q_b_q, q_b_s, kv_a_q,
                         kv_a_s,    k_b_q,    k_b_s,     v_b_q, v_b_s, attn_out_q, attn_out_s};
    return attn_layer(true, layer, p);
}

int glm_cuda_bind_attn_layer_device(int layer, const float* attn_norm, const float* q_a_norm, const float* kv_a_norm,
                                    const int8_t* q_a_q, const float* q_a_s, const int8_t* q_b_q, const float* q_b_s,
                                    const int8_t* kv_a_q, const float* kv_a_s, const int8_t* k_b_q,
                                    const float* k_b_s, const int8_t* v_b_q, const float* v_b_s,
                                    const int8_t* attn_out_q, const float* attn_out_s) {
    const void* p[15] = {attn_norm, q_a_norm, kv_a_norm, q_a_q, q_a_s, q_b_q, q_b_s, kv_a_q,
                         kv_a_s,    k_b_q,    k_b_s,     v_b_q, v_b_s, attn_out_q, attn_out_s};
    return attn_layer(false, layer, p);
}

int glm_cuda_forward_token(int token, int pos, float* logits) {
    std::lock_guard<std::mutex> lk(g_mu);
    if (int rc = check_model()) return rc;
    Model& m = g.m;
    if (pos < 0 || pos >= m.d.cache_cap) return fail(GLM_CUDA_ERR_ARG, "position %d outside the cache [0,%d)", pos,
                                                    m.d.cache_cap);
    if (token < 0 || token >= m.d.vocab_size) token = 0;  // as infer.c:1781
    m.io_host[0] = token;
    m.io_host[1] = pos;
    CUDA_TRY(cudaMemcpyAsync(m.token, &m.io_host[0], sizeof(int), cudaMemcpyHostToDevice, g.stream));
    CUDA_TRY(cudaMemcpyAsync(m.pos, &m.io_host[1], sizeof(int), cudaMemcpyHostToDevice, g.stream));
    if (int rc = enqueue_step(g.stream)) return rc;
    if (logits)
        CUDA_TRY(cudaMemcpyAsync(logits, m.logits, sizeof(float) * m.d.vocab_size, cudaMemcpyDeviceToHost, g.stream));
    return status_check_sync();
}

int glm_cuda_prefill(const int32_t* tokens, int n_tokens, int start_pos, float* logits) {
    std::lock_guard<std::mutex> lk(g_mu);
    if (int rc = check_model()) return rc;
    Model& m = g.m;
    if (!tokens || n_tokens < 1) return fail(GLM_CUDA_ERR_ARG, "prefill: tokens must be non-NULL and n_tokens >= 1");
    if (start_pos < 0 || start_pos + n_tokens > m.d.cache_cap)
        return fail(GLM_CUDA_ERR_ARG, "prefill: positions [%d,%d) outside the cache [0,%d)", start_pos,
                    start_pos + n_tokens, m.d.cache_cap);
    if (int rc = ensure_model_prefill(n_tokens)) return rc;
    cudaStream_t st = g.stream;
    if (int rc = stage_prefill_batch(tokens, n_tokens, start_pos, st)) return rc;
    if (int rc = enqueue_prefill(n_tokens, st)) return rc;
    if (logits) {
        // the last token's logits: final norm (fused) and LM head (infer.c:1888-1893)
        LAUNCH_TRY(glmq::launch_q80_matvec(m.out_q, m.out_s, m.pf_x + (size_t)(n_tokens - 1) * m.d.dim, m.logits,
                                           m.d.vocab_size, m.d.dim, m.d.group_size, g.num_sms, st, false,
                                           m.output_norm));
        g.launches += 1;
        CUDA_TRY(cudaMemcpyAsync(logits, m.logits, sizeof(float) * m.d.vocab_size, cudaMemcpyDeviceToHost, st));
    }
    return status_check_sync();
}

int glm_cuda_set_model_prefill(int min_tokens) {
    std::lock_guard<std::mutex> lk(g_mu);
    if (!g.inited) return fail(GLM_CUDA_ERR_STATE, "glm_cuda_init has not been called");
    if (min_tokens < 0) return fail(GLM_CUDA_ERR_ARG, "min_tokens must be >= 0");
    g.model_prefill_min = min_tokens;
    return 0;
}

int glm_cuda_generate(const int32_t* prompt, int n_prompt, int n_gen, int32_t* out_ids, float* device_ms) {
    std::lock_guard<std::mutex> lk(g_mu);
    if (int rc = check_model()) return rc;
    Model& m = g.m;
    if (!prompt || n_prompt <= 0 || n_gen <= 0 || !out_ids) return fail(GLM_CUDA_ERR_ARG, "bad generate arguments");
    if (n_prompt + n_gen - 1 > m.d.cache_cap)
        return fail(GLM_CUDA_ERR_ARG, "prompt + generation (%d) exceeds the cache (%d)", n_prompt + n_gen - 1,
                    m.d.cache_cap);
    if (n_prompt > m.prompt_cap) {
        if (m.prompt) cudaFree(m.prompt);
        m.prompt = nullptr;
        m.prompt_cap = 0;
        if (int rc = dev_alloc(&m.prompt, n_prompt)) return rc;
        m.prompt_cap = n_prompt;
    }
    if (n_gen > m.out_cap) {
        if (m.out_ids) cudaFree(m.out_ids);
        m.out_ids = nullptr;
        m.out_cap = 0;
        if (int rc = dev_alloc(&m.out_ids, n_gen)) return rc;
        m.out_cap = n_gen;
    }
    cudaStream_t st = g.stream;
    // positions [0, n_batch) as one batched pass, the rest step by step
    const int n_batch = (g.model_prefill_min > 0 && n_prompt - 1 >= g.model_prefill_min) ? n_prompt - 1 : 0;
    if (n_batch) {
        if (int rc = ensure_model_prefill(n_batch)) return rc;
        if (int rc = stage_prefill_batch(prompt, n_batch, 0, st)) return rc;
    }
    CUDA_TRY(cudaMemcpyAsync(m.prompt, prompt, sizeof(int32_t) * n_prompt, cudaMemcpyHostToDevice, st));
    int first = prompt[n_batch];
    if (first < 0 || first >= m.d.vocab_size) first = 0;
    m.io_host[0] = first;
    m.io_host[1] = n_batch;
    CUDA_TRY(cudaMemcpyAsync(m.token, &m.io_host[0], sizeof(int), cudaMemcpyHostToDevice, st));
    CUDA_TRY(cudaMemcpyAsync(m.pos, &m.io_host[1], sizeof(int), cudaMemcpyHostToDevice, st));
    // One decode step (+ picking the next token) captured once, replayed
    // for every position: the token and position live in device memory.
    cudaGraph_t graph = nullptr;
    cudaGraphExec_t exec = nullptr;
    CUDA_TRY(cudaStreamBeginCapture(st, cudaStreamCaptureModeThreadLocal));
    int rc = enqueue_step(st);
    if (!rc) {
        cudaError_t e = glmq::launch_decode_advance(m.pos, m.token, m.argmax, m.prompt, n_prompt, m.out_ids,
                                                    m.d.vocab_size, st);
        if (e != cudaSuccess) rc = fail(GLM_CUDA_ERR_CUDA, "decode advance: %s", cudaGetErrorString(e));
    }
    cudaError_t ec = cudaStreamEndCapture(st, &graph);
    if (rc) {
        if (graph) cudaGraphDestroy(graph);
        return rc;
    }
    if (ec != cudaSuccess) return fail(GLM_CUDA_ERR_CUDA, "graph capture: %s", cudaGetErrorString(ec));
    ec = cudaGraphInstantiate(&exec, graph, 0);
    cudaGraphDestroy(graph);
    if (ec != cudaSuccess) return fail(GLM_CUDA_ERR_CUDA, "graph instantiate: %s", cudaGetErrorString(ec));
    cudaEvent_t ev[2] = {nullptr, nullptr};
    if (device_ms) {
        cudaEventCreate(&ev[0]);
        cudaEventCreate(&ev[1]);
        cudaEventRecord(ev[0], st);
    }
    if (n_batch) {
        if (int prc = enqueue_prefill(n_batch, st)) {
            cudaStreamSynchronize(st);
            for (auto e : ev)
                if (e) cudaEventDestroy(e);
            cudaGraphExecDestroy(exec);
            return prc;
        }
    }
    const int steps = n_prompt - n_batch + n_gen - 1;
    for (int i = 0; i < steps && ec == cudaSuccess; ++i) ec = cudaGraphLaunch(exec, st);
    if (device_ms) cudaEventRecord(ev[1], st);
    g.launches += (unsigned long long)steps;
    if (ec == cudaSuccess) ec = cudaMemcpyAsync(out_ids, m.out_ids, sizeof(int32_t) * n_gen, cudaMemcpyDeviceToHost, st);
    if (ec == cudaSuccess) ec = cudaStreamSynchronize(st);
    if (device_ms && ec == cudaSuccess) cudaEventElapsedTime(device_ms, ev[0], ev[1]);
    for (auto e : ev)
        if (e) cudaEventDestroy(e);
    cudaGraphExecDestroy(exec);
    if (ec != cudaSuccess) return fail(GLM_CUDA_ERR_CUDA, "generate: %s", cudaGetErrorString(ec));
    return status_check_sync();
}

}  // extern "C"
