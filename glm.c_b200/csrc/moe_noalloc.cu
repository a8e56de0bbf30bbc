// glm_cuda_moe_layer_noalloc: the MoE decode layer for callers that must not
// allocate device memory.
//
// Who needs it: a host program that plans all of its GPU memory up front and
// may not allocate once it is serving -- for example an inference server that
// forbids allocation on the request path (a cudaMalloc there can block on the
// device, fragment a pool sized at start-up, or fail under memory pressure in
// the middle of a request), or an embedder that hands this library only
// pointers it already owns. Such a caller cannot call glm_cuda_init, which
// allocates the decode scratch and copies of the weights.
//
// What it does: the same three decode kernels as glm_cuda_moe_layer_async,
// but the scratch they need (normalised activations, SwiGLU activations,
// router intervals, top-k, the last-CTA counter) lives in the file-scope
// __device__ array below, of fixed size. The caller passes every input and
// output as device memory; nothing here calls cudaMalloc, cudaFree or any
// allocating routine.
//
// Limits: dim <= 4096, moe_ffn_dim <= 4096, n_routed_experts <= 256,
// n_experts_used <= 8 (larger sizes are rejected with GLM_CUDA_ERR_ARG), plus
// the shape rules of the other entry points (gs == 32, dim % 128 == 0,
// moe_ffn_dim % 64 == 0). Every GPU that loads the library holds this array
// (about 170 KB) until the process exits.
//
// Sharing: there is one array per device, shared by every call. Calls that
// overlap on the GPU (different streams, or host threads racing) race on it;
// callers must order them. Each call clears the counter and statistics words
// that must start at zero; everything else is fully written before it is read.
//
// Set-up: the first call on a device looks up the array's device address with
// cudaGetSymbolAddress (with that device current) and caches it. Make that
// first call before any stream capture begins.
#include <cstdio>
#include <cstdlib>
#include <mutex>

#include <cuda_runtime.h>

#include "glm_cuda.h"
#include "glm_internal.h"

namespace {

constexpr int kMaxDim = 4096;
constexpr int kMaxFfn = 4096;
constexpr int kMaxExperts = 256;
constexpr int kMaxTopK = 8;

constexpr size_t kOffXn = 0;                                                    // float [kMaxDim]
constexpr size_t kOffH = kOffXn + sizeof(float) * kMaxDim;                      // float [(K+1)][F]
constexpr size_t kOffCenter = kOffH + sizeof(float) * (kMaxTopK + 1) * kMaxFfn; // double [E]
constexpr size_t kOffBound = kOffCenter + sizeof(double) * kMaxExperts;          // double [E]
constexpr size_t kOffIdx = kOffBound + sizeof(double) * kMaxExperts;             // int32 [K]
constexpr size_t kOffW = kOffIdx + 64;                                           // float [K]
constexpr size_t kOffCounter = kOffW + 64;                                       // uint32 (zeroed per call)
constexpr size_t kOffStats = kOffCounter + 64;                                   // uint64 [4] (zeroed per call)
constexpr size_t kScratchBytes = kOffStats + 64;

static __device__ __align__(256) unsigned char g_noalloc_scratch[kScratchBytes];

constexpr int kMaxDevices = 64;
struct DeviceScratch {
    bool ready = false;
    unsigned char* base = nullptr;  // device address of g_noalloc_scratch on this device
    int num_sms = 0;
};
DeviceScratch g_dev[kMaxDevices];
std::mutex g_setup_mu;

thread_local char g_msg[256];

int reject(int code, const char* what) {
    snprintf(g_msg, sizeof g_msg, "glm_cuda_moe_layer_noalloc: %s", what);
    glmq::set_last_error(g_msg);
    fprintf(stderr, "[glm-cuda] %s\n", g_msg);
    return code;
}

// Once per device, with that device current: resolve the array's address.
int setup_device(int dev, DeviceScratch** out) {
    std::lock_guard<std::mutex> lk(g_setup_mu);
    DeviceScratch& d = g_dev[dev];
    if (!d.ready) {
        void* p = nullptr;
        cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
        if (e != cudaSuccess) return reject(GLM_CUDA_ERR_CUDA, cudaGetErrorString(e));
        int sms = 0;
        e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
        if (e != cudaSuccess) return reject(GLM_CUDA_ERR_CUDA, cudaGetErrorString(e));
        d.base = static_cast<unsigned char*>(p);
        d.num_sms = sms;
        d.ready = true;
    }
    *out = &d;
    return 0;
}

}  // namespace

extern "C" int glm_cuda_moe_layer_noalloc(
    const float* ffn_norm, const float* gate_inp, const float* exp_probs_b, const int8_t* gate_sh_q,
    const float* gate_sh_s, const int8_t* up_sh_q, const float* up_sh_s, const int8_t* down_sh_q,
    const float* down_sh_s, const int8_t* gate_q, const float* gate_s, const int8_t* up_q, const float* up_s,
    const int8_t* down_q, const float* down_s, int dim, int moe_ffn_dim, int n_routed_experts,
    int n_experts_used, int group_size, float* x_dev, int n_tokens, int32_t* topk_idx_dev, float* topk_w_dev,
    void* stream) {
    if (dim > kMaxDim || moe_ffn_dim > kMaxFfn || n_routed_experts > kMaxExperts || n_experts_used > kMaxTopK)
        return reject(GLM_CUDA_ERR_ARG, "size above the static scratch limit (dim<=4096, moe_ffn_dim<=4096, "
                                        "experts<=256, top-k<=8)");
    if (dim <= 0 || dim % 128 || moe_ffn_dim <= 0 || moe_ffn_dim % 64 || group_size != 32 ||
        n_experts_used < 1 || n_experts_used > n_routed_experts)
        return reject(GLM_CUDA_ERR_ARG, "unsupported shape (need gs==32, dim%128==0, moe_ffn_dim%64==0, "
                                        "1<=top-k<=experts)");
    if (!x_dev || n_tokens < 0 || !ffn_norm || !gate_inp || !exp_probs_b || !gate_sh_q || !gate_sh_s ||
        !up_sh_q || !up_sh_s || !down_sh_q || !down_sh_s)
        return reject(GLM_CUDA_ERR_ARG, "x, router and shared-expert pointers must be non-NULL");
    if (gate_q && (!gate_s || !up_q || !up_s || !down_q || !down_s))
        return reject(GLM_CUDA_ERR_ARG, "routed block is incomplete");
    if (n_tokens == 0) return 0;

    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return reject(GLM_CUDA_ERR_CUDA, cudaGetErrorString(e));
    if (dev < 0 || dev >= kMaxDevices) return reject(GLM_CUDA_ERR_ARG, "device ordinal above 63");
    DeviceScratch* d = nullptr;
    if (int rc = setup_device(dev, &d)) return rc;

    glmq::MoeScratch s;
    s.xn = reinterpret_cast<float*>(d->base + kOffXn);
    s.h = reinterpret_cast<float*>(d->base + kOffH);
    s.center = reinterpret_cast<double*>(d->base + kOffCenter);
    s.bound = reinterpret_cast<double*>(d->base + kOffBound);
    s.topk_idx = reinterpret_cast<int32_t*>(d->base + kOffIdx);
    s.topk_w = reinterpret_cast<float*>(d->base + kOffW);
    s.counter = reinterpret_cast<unsigned int*>(d->base + kOffCounter);
    s.stats = reinterpret_cast<unsigned long long*>(d->base + kOffStats);

    glmq::MoeLayerDev w{ffn_norm, gate_inp, exp_probs_b, gate_sh_q, gate_sh_s, up_sh_q, up_sh_s, down_sh_q,
                        down_sh_s, gate_q, gate_s, up_q, up_s, down_q, down_s};
    glmq::MoeDims dims{dim, moe_ffn_dim, n_routed_experts, n_experts_used, group_size};
    cudaStream_t st = static_cast<cudaStream_t>(stream);

    // The last-CTA counter must start at zero; the statistics start fresh.
    e = cudaMemsetAsync(d->base + kOffCounter, 0, kScratchBytes - kOffCounter, st);
    if (e != cudaSuccess) return reject(GLM_CUDA_ERR_CUDA, cudaGetErrorString(e));

    const char* env = getenv("GLM_DISABLE_MOE_ROUTED");  // as infer.c:1161-1165
    const int routed = (env && env[0] && env[0] != '0') ? 0 : 1;
    for (int t = 0; t < n_tokens; ++t) {
        float* xt = x_dev + (size_t)t * dim;
        e = glmq::launch_moe_decode(w, dims, s, xt, xt, routed, d->num_sms, st);
        if (e != cudaSuccess) return reject(GLM_CUDA_ERR_CUDA, cudaGetErrorString(e));
        if (topk_idx_dev) {
            e = cudaMemcpyAsync(topk_idx_dev + (size_t)t * n_experts_used, s.topk_idx,
                                sizeof(int32_t) * n_experts_used, cudaMemcpyDeviceToDevice, st);
            if (e != cudaSuccess) return reject(GLM_CUDA_ERR_CUDA, cudaGetErrorString(e));
        }
        if (topk_w_dev) {
            e = cudaMemcpyAsync(topk_w_dev + (size_t)t * n_experts_used, s.topk_w, sizeof(float) * n_experts_used,
                                cudaMemcpyDeviceToDevice, st);
            if (e != cudaSuccess) return reject(GLM_CUDA_ERR_CUDA, cudaGetErrorString(e));
        }
    }
    return 0;
}
