// Device kernels of the rest of GLM-4.7-Flash's batch-1 decode step around
// the MoE layers (glm_cpu_forward_token, infer.c:1767-1901): token
// embedding, rmsnorm, MLA attention with the compressed KV cache, the layer-0
// dense SwiGLU, and the greedy argmax (the rmsnorms that feed a linear layer
// run fused into the matvec, q80_matvec.cu). The Q8 linear layers run on the
// matvec kernel (q80_matvec.cu) and the MoE layers on the persistent kernel.
//
// Every kernel reads the token id and the position from device memory, so a
// whole decode step can be captured once in a CUDA graph and replayed for
// every position (the step ends with `decode_advance`, which picks the next
// token: the next prompt id, else the argmax, as glm_app_main's loop does,
// infer.c:2190-2228).
#include <cfloat>
#include <cmath>
#include <cstdint>

#include "glm_internal.h"
#include "q80_common.cuh"

namespace glmq {

namespace {

__device__ __forceinline__ float block_sum_f(float v, float* red) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
    __syncthreads();
    if (lane == 0) red[warp] = v;
    __syncthreads();
    float t = 0.f;
    for (int w = 0; w < nw; ++w) t += red[w];
    return t;
}

__device__ __forceinline__ double block_sum_d(double v, double* red) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
    __syncthreads();
    if (lane == 0) red[warp] = v;
    __syncthreads();
    double t = 0.0;
    for (int w = 0; w < nw; ++w) t += red[w];
    return t;
}

// 1/sqrtf(mean(x^2) + 1e-5) with the sum of squares in fp64 (infer.c:746-752).
__device__ __forceinline__ float rms_inv(const float* x, int n, double* red) {
    double ss = 0.0;
    for (int i = threadIdx.x; i < n; i += blockDim.x) ss += (double)x[i] * (double)x[i];
    ss = block_sum_d(ss, red);
    const float mean = (float)(ss / (double)n);
    return 1.0f / sqrtf(mean + 1e-5f);
}

// RoPE of infer.c:964-976 on pairs (2i, 2i+1), theta 1e6.
__device__ __forceinline__ void rope_pair(float& x0, float& x1, int i, int dim, int pos) {
    const float freq = powf(1000000.0f, -((float)i / (float)dim));
    const float ang = (float)pos * freq;
    const float c = cosf(ang), s = sinf(ang);
    const float a = x0 * c - x1 * s, b = x0 * s + x1 * c;
    x0 = a;
    x1 = b;
}

// x = dequant(tok_q[token]) (infer.c:1810-1812).
__global__ void embed_kernel(const int8_t* tok_q, const float* tok_s, const int* token, float* x, int D, int gs) {
    pdl_enter();
    const int t = *token;
    const int8_t* q = tok_q + (size_t)t * D;
    const float* s = tok_s + (size_t)t * (D / gs);
    for (int i = threadIdx.x; i < D; i += blockDim.x) x[i] = (float)q[i] * s[i / gs];
}

// kv_a[0:kv_lora] <- rmsnorm * kv_a_norm, stored as this position's
// compressed key; kv_a[kv_lora:] roped, stored as its rope key
// (infer.c:1003-1016).
__global__ void kv_cache_write_kernel(float* kv_a, const float* kv_norm, float* cache_comp, float* cache_pe,
                                      const int* pos_dev, int kv_lora, int rope) {
    pdl_enter();
    __shared__ double red[32];
    const int pos = *pos_dev;
    const float inv = rms_inv(kv_a, kv_lora, red);
    __syncthreads();
    float* comp = cache_comp + (size_t)pos * kv_lora;
    for (int i = threadIdx.x; i < kv_lora; i += blockDim.x) {
        const float v = kv_a[i] * inv * kv_norm[i];
        kv_a[i] = v;
        comp[i] = v;
    }
    float* pe = cache_pe + (size_t)pos * rope;
    for (int i = 2 * threadIdx.x; i + 1 < rope; i += 2 * blockDim.x) {
        float x0 = kv_a[kv_lora + i], x1 = kv_a[kv_lora + i + 1];
        rope_pair(x0, x1, i, rope, pos);
        pe[i] = x0;
        pe[i + 1] = x1;
    }
}

// kR rows of a planar Q8 matrix dotted with x (shared memory) by one warp,
// all rows' loads issued together: lane l covers the kBytes-wide pieces
// l, l + 32, ... of every row (cols a multiple of kBytes and of gs).
template <int kBytes, int kR>
__device__ __forceinline__ void q8_rows_dot(const int8_t* q, const float* s, const float* x, int cols, int gs,
                                            int r0, int nrows, float (&out)[kR]) {
    const int lane = threadIdx.x & 31;
    const int ng = cols / gs;
#pragma unroll
    for (int j = 0; j < kR; ++j) out[j] = 0.f;
    for (int c0 = lane * kBytes; c0 < cols; c0 += 32 * kBytes) {
        int w[kR][kBytes / 4];
        float sc[kR];
#pragma unroll
        for (int j = 0; j < kR; ++j) {
            const int r = r0 + j;
            if (r < nrows) {
                const int8_t* p = q + (size_t)r * cols + c0;
                if constexpr (kBytes == 16) {
                    const int4 v = *reinterpret_cast<const int4*>(p);
                    w[j][0] = v.x;
                    w[j][1] = v.y;
                    w[j][2] = v.z;
                    w[j][3] = v.w;
                } else {
                    const int2 v = *reinterpret_cast<const int2*>(p);
                    w[j][0] = v.x;
                    w[j][1] = v.y;
                }
                sc[j] = s[(size_t)r * ng + c0 / gs];
            } else {
#pragma unroll
                for (int k = 0; k < kBytes / 4; ++k) w[j][k] = 0;
                sc[j] = 0.f;
            }
        }
#pragma unroll
        for (int j = 0; j < kR; ++j) {
            float d = 0.f;
#pragma unroll
            for (int k = 0; k < kBytes; ++k) d += (float)(int8_t)(w[j][k >> 2] >> (8 * (k & 3))) * x[c0 + k];
            out[j] += sc[j] * d;
        }
    }
#pragma unroll
    for (int j = 0; j < kR; ++j)
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) out[j] += __shfl_xor_sync(0xffffffffu, out[j], off);
}

// MLA attention of one head per CTA (infer.c:1018-1058): q_pe roped,
// q_abs = k_b_h . q_nope, scores over the cache, softmax, context, and
// att_concat[h] = v_b_h . context. Every stage keeps many independent loads
// in flight (rows in groups of 8 per warp; cache rows split over the warps).
__global__ void __launch_bounds__(512) mla_heads_kernel(MlaArgs a) {
    pdl_enter();
    extern __shared__ __align__(16) float smf[];
    constexpr int kR = 8;
    const int h = blockIdx.x, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, nw = blockDim.x >> 5;
    const int pos = *a.pos;
    float* q_nope = smf;                   // [qk_nope]
    float* q_pe = q_nope + a.qk_nope;      // [rope]
    float* q_abs = q_pe + a.rope;          // [kv_lora]
    float* ctx = q_abs + a.kv_lora;        // [kv_lora]
    float* scores = ctx + a.kv_lora;       // [cache_cap]
    float* cpart = scores + a.cache_cap;   // [nw][kv_lora] per-warp context partials
    __shared__ float red[32];

    const float* qh = a.q_full + (size_t)h * a.head_k;
    for (int i = tid; i < a.qk_nope; i += blockDim.x) q_nope[i] = qh[i];
    for (int i = 2 * tid; i + 1 < a.rope; i += 2 * blockDim.x) {
        float x0 = qh[a.qk_nope + i], x1 = qh[a.qk_nope + i + 1];
        rope_pair(x0, x1, i, a.rope, pos);
        q_pe[i] = x0;
        q_pe[i + 1] = x1;
    }
    __syncthreads();

    // q_abs[r] = k_b_h[r] . q_nope  (k_b: [heads][kv_lora][qk_nope])
    const int8_t* kbq = a.k_b_q + (size_t)h * a.kv_lora * a.qk_nope;
    const float* kbs = a.k_b_s + (size_t)h * a.kv_lora * (a.qk_nope / a.gs);
    for (int r0 = warp * kR; r0 < a.kv_lora; r0 += nw * kR) {
        float v[kR];
        q8_rows_dot<8, kR>(kbq, kbs, q_nope, a.qk_nope, a.gs, r0, a.kv_lora, v);
        if (lane < kR && r0 + lane < a.kv_lora) {
            float mine = v[0];
#pragma unroll
            for (int j = 1; j < kR; ++j)
                if (lane == j) mine = v[j];
            q_abs[r0 + lane] = mine;
        }
    }
    __syncthreads();

    // scores[t] = (q_abs . kc[t] + q_pe . kp[t]) * kq_scale, two rows per warp step
    const float* cc = a.cache_comp;
    const float* cp = a.cache_pe;
    for (int t = warp; t <= pos; t += 2 * nw) {
        const int t2 = t + nw;
        const float* kc = cc + (size_t)t * a.kv_lora;
        const float* kc2 = cc + (size_t)(t2 <= pos ? t2 : t) * a.kv_lora;
        float d = 0.f, d2 = 0.f;
        for (int i = lane; i < a.kv_lora; i += 32) {
            d += q_abs[i] * kc[i];
            d2 += q_abs[i] * kc2[i];
        }
        for (int i = lane; i < a.rope; i += 32) {
            d += q_pe[i] * cp[(size_t)t * a.rope + i];
            d2 += q_pe[i] * cp[(size_t)(t2 <= pos ? t2 : t) * a.rope + i];
        }
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) {
            d += __shfl_xor_sync(0xffffffffu, d, off);
            d2 += __shfl_xor_sync(0xffffffffu, d2, off);
        }
        if (lane == 0) {
            scores[t] = d * a.kq_scale;
            if (t2 <= pos) scores[t2] = d2 * a.kq_scale;
        }
    }
    __syncthreads();

    // softmax (infer.c:951-962)
    float mx = -FLT_MAX;
    for (int t = tid; t <= pos; t += blockDim.x) mx = fmaxf(mx, scores[t]);
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
    if (lane == 0) red[warp] = mx;
    __syncthreads();
    mx = red[0];
    for (int w = 1; w < nw; ++w) mx = fmaxf(mx, red[w]);
    __syncthreads();
    float sum = 0.f;
    for (int t = tid; t <= pos; t += blockDim.x) {
        const float e = expf(scores[t] - mx);
        scores[t] = e;
        sum += e;
    }
    sum = block_sum_f(sum, red);
    const float inv = sum > 0.f ? 1.0f / sum : 1.0f;
    __syncthreads();

    // ctx = sum_t p[t] kc[t]: warp w takes positions w, w + nw, ... (lanes
    // over the row), then the warps' partials are added in warp order.
    for (int i = lane; i < a.kv_lora; i += 32) {
        float acc = 0.f;
        for (int t = warp; t <= pos; t += nw) acc += scores[t] * inv * cc[(size_t)t * a.kv_lora + i];
        cpart[warp * a.kv_lora + i] = acc;
    }
    __syncthreads();
    for (int i = tid; i < a.kv_lora; i += blockDim.x) {
        float acc = 0.f;
        for (int w = 0; w < nw; ++w) acc += cpart[w * a.kv_lora + i];
        ctx[i] = acc;
    }
    __syncthreads();

    // att_concat[h][r] = v_b_h[r] . ctx  (v_b: [heads][v_head][kv_lora])
    const int8_t* vbq = a.v_b_q + (size_t)h * a.v_head * a.kv_lora;
    const float* vbs = a.v_b_s + (size_t)h * a.v_head * (a.kv_lora / a.gs);
    float* out = a.att_concat + (size_t)h * a.v_head;
    for (int r0 = warp * kR; r0 < a.v_head; r0 += nw * kR) {
        float v[kR];
        q8_rows_dot<16, kR>(vbq, vbs, ctx, a.kv_lora, a.gs, r0, a.v_head, v);
        if (lane < kR && r0 + lane < a.v_head) {
            float mine = v[0];
#pragma unroll
            for (int j = 1; j < kR; ++j)
                if (lane == j) mine = v[j];
            out[r0 + lane] = mine;
        }
    }
}

// g = silu(g) * u (infer.c:1076-1078).
__global__ void silu_mul_kernel(float* g, const float* u, int n) {
    pdl_enter();
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
        const float v = g[i];
        g[i] = v / (1.0f + expf(-v)) * u[i];
    }
}

// First index of the maximum (argmax, infer.c:1218-1228: strict '>'): each
// CTA reduces a slice to (value, index) in `part`; the last CTA to finish
// (counter, reset by it) reduces the partials in CTA order.
__global__ void argmax_kernel(const float* x, int n, float2* part, unsigned* counter, int* out) {
    pdl_enter();
    __shared__ float bv[32];
    __shared__ int bi[32];
    __shared__ int last;
    const int per = (n + gridDim.x - 1) / gridDim.x;
    const int lo = blockIdx.x * per, hi = min(n, lo + per);
    float best = -INFINITY;
    int idx = n;
    for (int i = lo + threadIdx.x; i < hi; i += blockDim.x) {
        const float v = x[i];
        if (v > best) {  // i increases per thread: keeps the thread's first maximum
            best = v;
            idx = i;
        }
    }
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, best, off);
        const int oi = __shfl_xor_sync(0xffffffffu, idx, off);
        if (ov > best || (ov == best && oi < idx)) {
            best = ov;
            idx = oi;
        }
    }
    if (lane == 0) {
        bv[warp] = best;
        bi[warp] = idx;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        for (int w = 1; w < nw; ++w)
            if (bv[w] > best || (bv[w] == best && bi[w] < idx)) {
                best = bv[w];
                idx = bi[w];
            }
        part[blockIdx.x] = make_float2(best, __int_as_float(idx));
        __threadfence();
        last = atomicAdd(counter, 1u) == gridDim.x - 1;
    }
    __syncthreads();
    if (!last || threadIdx.x != 0) return;
    __threadfence();
    float b = -INFINITY;
    int bix = n;
    for (int c = 0; c < (int)gridDim.x; ++c) {
        const float2 p = __ldcg(part + c);
        const int pi = __float_as_int(p.y);
        if (p.x > b || (p.x == b && pi < bix)) {
            b = p.x;
            bix = pi;
        }
    }
    *counter = 0u;
    // glm.c's argmax starts from x[0]: a NaN there (or all-NaN logits) keeps
    // index 0, since no comparison with NaN succeeds
    *out = (bix < n && !isnan(__ldcg(x))) ? bix : 0;
}

// End of a decode step at position pos: the next token is the next prompt
// id while the prompt lasts, else the argmax (recorded as generated).
__global__ void decode_advance_kernel(int* pos, int* token, const int* argmax, const int* prompt, int n_prompt,
                                      int* out_ids, int vocab) {
    pdl_enter();
    const int p = *pos;
    int next;
    if (p + 1 < n_prompt) {
        next = prompt[p + 1];
        if (next < 0 || next >= vocab) next = 0;
    } else {
        next = *argmax;
        out_ids[p + 1 - n_prompt] = next;
    }
    *token = next;
    *pos = p + 1;
}

}  // namespace

cudaError_t launch_embed(const int8_t* tok_q, const float* tok_s, const int* token, float* x, int D, int gs,
                         cudaStream_t st) {
    return launch_pdl(embed_kernel, 1, 512, 0, st, tok_q, tok_s, token, x, D, gs);
}

cudaError_t launch_kv_cache_write(float* kv_a, const float* kv_norm, float* cache_comp, float* cache_pe,
                                  const int* pos, int kv_lora, int rope, cudaStream_t st) {
    return launch_pdl(kv_cache_write_kernel, 1, 512, 0, st, kv_a, kv_norm, cache_comp, cache_pe, pos, kv_lora, rope);
}

size_t mla_heads_smem(const MlaArgs& a, int cache_cap) {
    return sizeof(float) * ((size_t)a.qk_nope + a.rope + 2 * (size_t)a.kv_lora + cache_cap + 16 * (size_t)a.kv_lora);
}

cudaError_t launch_mla_heads(const MlaArgs& a, int n_heads, int cache_cap, cudaStream_t st) {
    const size_t smem = mla_heads_smem(a, cache_cap);
    if (smem > 200 * 1024) return cudaErrorInvalidValue;
    if (smem > 48 * 1024)
        if (cudaError_t e = ensure_smem_attr(reinterpret_cast<const void*>(mla_heads_kernel), (int)smem)) return e;
    return launch_pdl(mla_heads_kernel, n_heads, 512, smem, st, a);
}

cudaError_t launch_silu_mul(float* g, const float* u, int n, int num_sms, cudaStream_t st) {
    return launch_pdl(silu_mul_kernel, num_sms, 256, 0, st, g, u, n);
}

cudaError_t launch_argmax(const float* x, int n, float2* part, unsigned* counter, int nblocks, int* out,
                          cudaStream_t st) {
    return launch_pdl(argmax_kernel, nblocks, 512, 0, st, x, n, part, counter, out);
}

cudaError_t launch_decode_advance(int* pos, int* token, const int* argmax, const int* prompt, int n_prompt,
                                  int* out_ids, int vocab, cudaStream_t st) {
    return launch_pdl(decode_advance_kernel, 1, 1, 0, st, pos, token, argmax, prompt, n_prompt, out_ids, vocab);
}

}  // namespace glmq
