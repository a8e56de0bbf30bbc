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

#include <cooperative_groups.h>

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

// One lane's piece of kR rows of a planar Q8 matrix: kBytes weights of each
// row from column c0, and each row's scale of that piece (zero past nrows or
// past cols).
template <int kBytes, int kR>
struct Q8Frag {
    int w[kR][kBytes / 4];
    float sc[kR];
};

template <int kBytes, int kR>
__device__ __forceinline__ void q8_frag_load(const int8_t* q, const float* s, int cols, int gs, int r0, int nrows,
                                             int c0, Q8Frag<kBytes, kR>& f) {
    const int ng = cols / gs;
#pragma unroll
    for (int j = 0; j < kR; ++j) {
        const int r = r0 + j;
        if (r < nrows && c0 < cols) {
            const int8_t* p = q + (size_t)r * cols + c0;
            if constexpr (kBytes == 16) {
                const int4 v = *reinterpret_cast<const int4*>(p);
                f.w[j][0] = v.x;
                f.w[j][1] = v.y;
                f.w[j][2] = v.z;
                f.w[j][3] = v.w;
            } else {
                const int2 v = *reinterpret_cast<const int2*>(p);
                f.w[j][0] = v.x;
                f.w[j][1] = v.y;
            }
            f.sc[j] = s[(size_t)r * ng + c0 / gs];
        } else {
#pragma unroll
            for (int k = 0; k < kBytes / 4; ++k) f.w[j][k] = 0;
            f.sc[j] = 0.f;
        }
    }
}

// out[j] += scale * (piece of row j) . x[c0 : c0 + kBytes] (x in shared memory)
template <int kBytes, int kR>
__device__ __forceinline__ void q8_frag_fma(const Q8Frag<kBytes, kR>& f, const float* x, int c0, int cols,
                                            float (&out)[kR]) {
    if (c0 >= cols) return;
#pragma unroll
    for (int j = 0; j < kR; ++j) {
        float d = 0.f;
#pragma unroll
        for (int k = 0; k < kBytes; ++k) d += (float)(int8_t)(f.w[j][k >> 2] >> (8 * (k & 3))) * x[c0 + k];
        out[j] += f.sc[j] * d;
    }
}

template <int kR>
__device__ __forceinline__ void warp_sum_rows(float (&out)[kR]) {
#pragma unroll
    for (int j = 0; j < kR; ++j)
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) out[j] += __shfl_xor_sync(0xffffffffu, out[j], off);
}

// kR rows of a planar Q8 matrix dotted with x (shared memory) by one warp,
// all rows' loads issued together: lane l covers the kBytes-wide pieces
// l, l + 32, ... of every row (cols a multiple of kBytes and of gs). When
// `first` holds the lane's first piece (loaded earlier), it is used instead
// of loading it.
template <int kBytes, int kR>
__device__ __forceinline__ void q8_rows_dot(const int8_t* q, const float* s, const float* x, int cols, int gs,
                                            int r0, int nrows, float (&out)[kR],
                                            const Q8Frag<kBytes, kR>* first = nullptr) {
    const int lane = threadIdx.x & 31;
#pragma unroll
    for (int j = 0; j < kR; ++j) out[j] = 0.f;
    for (int c0 = lane * kBytes; c0 < cols; c0 += 32 * kBytes) {
        Q8Frag<kBytes, kR> f;
        if (first && c0 == lane * kBytes)
            f = *first;
        else
            q8_frag_load(q, s, cols, gs, r0, nrows, c0, f);
        q8_frag_fma(f, x, c0, cols, out);
    }
    warp_sum_rows(out);
}

// Row r0 + lane's sum from q8_rows_dot's kR row sums (which every lane
// holds), for lanes [0, kR).
template <int kR>
__device__ __forceinline__ float pick_row(const float (&v)[kR], int lane) {
    float mine = v[0];
#pragma unroll
    for (int j = 1; j < kR; ++j)
        if (lane == j) mine = v[j];
    return mine;
}

// MLA attention (infer.c:1003-1058) for every head, one thread-block cluster
// of kMlaCluster CTAs per head; the CTAs of a head split every stage and
// exchange through distributed shared memory:
//   0. every CTA forms this position's key from kv_a: the latent part
//      rmsnorm * kv_a_norm, the rope part roped (infer.c:1003-1016); rank 0
//      of head 0 stores it in the cache, every CTA uses its own copy for
//      position pos;
//   1. q_abs = k_b_h . q_nope: each CTA computes 1/S of the rows and stores
//      them into every CTA of the cluster;
//   2. scores over 1/S of the positions, with the CTA's own max m and sum l
//      of exp(score - m), and its context partial sum_t exp(score_t - m) kc[t];
//   3. each CTA combines 1/S of the context columns over the cluster
//      (ctx = sum_r e^(m_r - M) part_r / sum_r e^(m_r - M) l_r, M the
//      largest m_r) and stores them into every CTA;
//   4. att_concat[h] = v_b_h . ctx: each CTA computes 1/S of the rows.
__global__ void __cluster_dims__(kMlaCluster, 1, 1) __launch_bounds__(kMlaThreads)
    mla_cluster_kernel(MlaArgs a) {
    namespace cg = cooperative_groups;
    cg::cluster_group cl = cg::this_cluster();
    constexpr int S = kMlaCluster, nw = kMlaThreads / 32;
    extern __shared__ __align__(16) float smf[];
    const int rank = (int)cl.block_rank(), h = blockIdx.x / S;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int r_lo = rank * a.kv_lora / S, r_hi = (rank + 1) * a.kv_lora / S;  // q_abs rows
    const int o_lo = rank * a.v_head / S, o_hi = (rank + 1) * a.v_head / S;    // output rows
    const int8_t* kbq = a.k_b_q + (size_t)h * a.kv_lora * a.qk_nope;
    const float* kbs = a.k_b_s + (size_t)h * a.kv_lora * (a.qk_nope / a.gs);
    const int8_t* vbq = a.v_b_q + (size_t)h * a.v_head * a.kv_lora;
    const float* vbs = a.v_b_s + (size_t)h * a.v_head * (a.kv_lora / a.gs);
    // Weights no kernel writes, loaded before waiting for the previous
    // kernel: each warp's first k_b and v_b pieces (for GLM-4.7-Flash's
    // shapes, all of this CTA's slices) and the kv_a_norm weights.
    constexpr int kRq = 8, kRo = 4;  // rows per warp step: q_abs, output
    Q8Frag<8, kRq> kf;
    Q8Frag<16, kRo> vf;
    q8_frag_load(kbq, kbs, a.qk_nope, a.gs, r_lo + warp * kRq, r_hi, lane * 8, kf);
    q8_frag_load(vbq, vbs, a.kv_lora, a.gs, o_lo + warp * kRo, o_hi, lane * 16, vf);
    float kn[kMlaStage];
#pragma unroll
    for (int u = 0; u < kMlaStage; ++u) {
        const int i = tid + u * kMlaThreads;
        kn[u] = i < a.kv_lora ? __ldg(a.kv_norm + i) : 0.f;
    }
    float* q_nope = smf;                      // [qk_nope]
    float* q_pe = q_nope + a.qk_nope;         // [rope]
    float* key = q_pe + a.rope;               // [kv_lora + rope] this position's cache entry
    float* q_abs = key + a.kv_lora + a.rope;  // [kv_lora]
    float* ctx = q_abs + a.kv_lora;           // [kv_lora]
    float* part = ctx + a.kv_lora;            // [kv_lora] this CTA's context partial
    float* stat = part + a.kv_lora;           // [2] m, l  (+2 pad)
    float* scores = stat + 4;                 // [ceil(cap / S)]
    __shared__ double red_d[32];
    __shared__ float red[32];

    pdl_enter();
    const int pos = *a.pos;
    // this head's query and the kv_a projection, every load in flight at once
    {
        const float* qh = a.q_full + (size_t)h * a.head_k;
        const int nkv = a.kv_lora + a.rope;
        float vq[kMlaStage], vk[kMlaStage];
#pragma unroll
        for (int u = 0; u < kMlaStage; ++u) {
            const int i = tid + u * kMlaThreads;
            vq[u] = i < a.head_k ? qh[i] : 0.f;
            vk[u] = i < nkv ? a.kv_a[i] : 0.f;
        }
#pragma unroll
        for (int u = 0; u < kMlaStage; ++u) {
            const int i = tid + u * kMlaThreads;
            if (i < a.head_k) q_nope[i] = vq[u];  // q_nope then q_pe: contiguous like q_full
            if (i < nkv) key[i] = vk[u];
        }
    }
    __syncthreads();
    // q_pe roped; this position's key: the latent part rmsnorm * kv_a_norm,
    // the rope part roped (infer.c:1003-1016)
    for (int i = 2 * tid; i + 1 < a.rope; i += 2 * kMlaThreads) {
        rope_pair(q_pe[i], q_pe[i + 1], i, a.rope, pos);
        rope_pair(key[a.kv_lora + i], key[a.kv_lora + i + 1], i, a.rope, pos);
    }
    const float inv = rms_inv(key, a.kv_lora, red_d);  // every read of key precedes its barriers
#pragma unroll
    for (int u = 0; u < kMlaStage; ++u) {
        const int i = tid + u * kMlaThreads;
        if (i < a.kv_lora) key[i] = key[i] * inv * kn[u];
    }
    __syncthreads();
    if (h == 0 && rank == 0) {
        for (int i = tid; i < a.kv_lora; i += kMlaThreads) a.cache_comp[(size_t)pos * a.kv_lora + i] = key[i];
        for (int i = tid; i < a.rope; i += kMlaThreads) a.cache_pe[(size_t)pos * a.rope + i] = key[a.kv_lora + i];
    }

    // 1. q_abs[r] = k_b_h[r] . q_nope (k_b: [heads][kv_lora][qk_nope]), rows [r_lo, r_hi)
    {
        constexpr int kR = kRq;
        for (int r0 = r_lo + warp * kR; r0 < r_hi; r0 += nw * kR) {
            float v[kR];
            q8_rows_dot<8, kR>(kbq, kbs, q_nope, a.qk_nope, a.gs, r0, r_hi, v, r0 == r_lo + warp * kR ? &kf : nullptr);
            const float mine = pick_row(v, lane);
            if (lane < kR && r0 + lane < r_hi)
#pragma unroll
                for (int d = 0; d < S; ++d) *cl.map_shared_rank(q_abs + r0 + lane, d) = mine;
        }
    }
    cl.sync();

    // 2. scores[t] = (q_abs . kc[t] + q_pe . kp[t]) * kq_scale over positions
    // [t_lo, t_hi): a warp per position, each lane 4 consecutive floats per
    // 128-float block, every load of the row in flight at once
    const int np = pos + 1, t_lo = rank * np / S, t_hi = (rank + 1) * np / S, nloc = t_hi - t_lo;
    for (int t = t_lo + warp; t < t_hi; t += nw) {
        const float* kc = t == pos ? key : a.cache_comp + (size_t)t * a.kv_lora;
        const float* kp = t == pos ? key + a.kv_lora : a.cache_pe + (size_t)t * a.rope;
        float4 c4[kMlaRowBlocks], p4;
#pragma unroll
        for (int u = 0; u < kMlaRowBlocks; ++u) {
            const int i = 4 * lane + 128 * u;
            c4[u] = i < a.kv_lora ? *reinterpret_cast<const float4*>(kc + i) : make_float4(0.f, 0.f, 0.f, 0.f);
        }
        p4 = 4 * lane < a.rope ? *reinterpret_cast<const float4*>(kp + 4 * lane) : make_float4(0.f, 0.f, 0.f, 0.f);
        float d = 0.f;
#pragma unroll
        for (int u = 0; u < kMlaRowBlocks; ++u) {
            const int i = 4 * lane + 128 * u;
            if (i < a.kv_lora) {
                const float4 qa = *reinterpret_cast<const float4*>(q_abs + i);
                d += qa.x * c4[u].x + qa.y * c4[u].y + qa.z * c4[u].z + qa.w * c4[u].w;
            }
        }
        if (4 * lane < a.rope) {
            const float4 qp = *reinterpret_cast<const float4*>(q_pe + 4 * lane);
            d += qp.x * p4.x + qp.y * p4.y + qp.z * p4.z + qp.w * p4.w;
        }
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) d += __shfl_xor_sync(0xffffffffu, d, off);
        if (lane == 0) scores[t - t_lo] = d * a.kq_scale;
    }
    __syncthreads();
    float mx = -FLT_MAX;  // a CTA without positions keeps -FLT_MAX and l = 0
    for (int t = tid; t < nloc; t += kMlaThreads) mx = fmaxf(mx, scores[t]);
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
    if (lane == 0) red[warp] = mx;
    __syncthreads();
    mx = red[0];
    for (int w = 1; w < nw; ++w) mx = fmaxf(mx, red[w]);
    __syncthreads();
    float sum = 0.f;
    for (int t = tid; t < nloc; t += kMlaThreads) {
        const float e = expf(scores[t] - mx);
        scores[t] = e;
        sum += e;
    }
    sum = block_sum_f(sum, red);  // ends with a block barrier: every exp is stored
    // context partial: thread pairs of columns, 8 positions' loads in flight
    for (int i = 2 * tid; i < a.kv_lora; i += 2 * kMlaThreads) {
        float2 acc = make_float2(0.f, 0.f);
        for (int t0 = t_lo; t0 < t_hi; t0 += 8) {
            float2 v[8];
#pragma unroll
            for (int u = 0; u < 8; ++u) {
                const int t = t0 + u;
                v[u] = t >= t_hi ? make_float2(0.f, 0.f)
                       : t == pos ? make_float2(key[i], key[i + 1])
                                  : *reinterpret_cast<const float2*>(a.cache_comp + (size_t)t * a.kv_lora + i);
            }
#pragma unroll
            for (int u = 0; u < 8; ++u) {
                const float e = t0 + u < t_hi ? scores[t0 + u - t_lo] : 0.f;
                acc.x += e * v[u].x;
                acc.y += e * v[u].y;
            }
        }
        part[i] = acc.x;
        part[i + 1] = acc.y;
    }
    if (tid == 0) {
        stat[0] = mx;
        stat[1] = sum;
    }
    cl.sync();

    // 3. ctx columns [c_lo, c_hi), combined over the cluster
    {
        float m_r[S], w_r[S];
        float M = -FLT_MAX;
#pragma unroll
        for (int r = 0; r < S; ++r) {
            m_r[r] = *cl.map_shared_rank(stat, r);
            M = fmaxf(M, m_r[r]);
        }
        float L = 0.f;
#pragma unroll
        for (int r = 0; r < S; ++r) {
            w_r[r] = expf(m_r[r] - M);
            L += *cl.map_shared_rank(stat + 1, r) * w_r[r];
        }
        const float invL = L > 0.f ? 1.0f / L : 1.0f;
        const int c_lo = rank * a.kv_lora / S, c_hi = (rank + 1) * a.kv_lora / S;
        for (int i = c_lo + tid; i < c_hi; i += kMlaThreads) {
            float pr[S];
#pragma unroll
            for (int r = 0; r < S; ++r) pr[r] = *cl.map_shared_rank(part + i, r);
            float acc = 0.f;
#pragma unroll
            for (int r = 0; r < S; ++r) acc += pr[r] * w_r[r];
            acc *= invL;
#pragma unroll
            for (int d = 0; d < S; ++d) *cl.map_shared_rank(ctx + i, d) = acc;
        }
    }
    cl.sync();  // last cluster-wide access: after it every CTA reads only its own memory

    // 4. att_concat[h][r] = v_b_h[r] . ctx (v_b: [heads][v_head][kv_lora]), rows [o_lo, o_hi)
    {
        constexpr int kR = kRo;
        float* out = a.att_concat + (size_t)h * a.v_head;
        for (int r0 = o_lo + warp * kR; r0 < o_hi; r0 += nw * kR) {
            float v[kR];
            q8_rows_dot<16, kR>(vbq, vbs, ctx, a.kv_lora, a.gs, r0, o_hi, v, r0 == o_lo + warp * kR ? &vf : nullptr);
            const float mine = pick_row(v, lane);
            if (lane < kR && r0 + lane < o_hi) out[r0 + lane] = mine;
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

size_t mla_smem(const MlaArgs& a) {
    const size_t per = ((size_t)a.cache_cap + kMlaCluster - 1) / kMlaCluster;
    return sizeof(float) * ((size_t)a.qk_nope + 2 * (size_t)a.rope + 4 * (size_t)a.kv_lora + 4 + per);
}

cudaError_t launch_mla(const MlaArgs& a, int n_heads, cudaStream_t st) {
    // q8_rows_dot widths, float4 rows, register staging and row blocks
    if (a.qk_nope % 8 || a.kv_lora % 16 || a.qk_nope % a.gs || a.kv_lora % a.gs || a.rope % 4 || a.rope > 128 ||
        a.head_k != a.qk_nope + a.rope || a.head_k > kMlaStage * kMlaThreads ||
        a.kv_lora + a.rope > kMlaStage * kMlaThreads || a.kv_lora > 128 * kMlaRowBlocks)
        return cudaErrorInvalidValue;
    const size_t smem = mla_smem(a);
    if (smem > 200 * 1024) return cudaErrorInvalidValue;
    if (cudaError_t e = ensure_smem_attr(reinterpret_cast<const void*>(mla_cluster_kernel), (int)smem)) return e;
    return launch_pdl(mla_cluster_kernel, n_heads * kMlaCluster, kMlaThreads, smem, st, a);
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
