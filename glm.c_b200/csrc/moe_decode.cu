// Batch-1 decode of one GLM-4.7-Flash MoE FFN layer on sm_100a.
//
// Replaces apply_moe_shared_ffn_layer (infer.c:1087-1216) for one token:
//
//   K1 moe_route_kernel     rmsnorm (infer.c:746-752) + fp32 router
//                           (infer.c:1103, 916-938) + sigmoid (1104-1107) +
//                           biased top-k (1110-1135) + normalisation
//                           (1136-1145). Expert ids are bit-identical to the
//                           reference: see "Exact routing" below.
//   K2 moe_gate_up_kernel   gate.xn and up.xn for the K routed experts (rank
//                           order) and the shared expert, fused with SwiGLU
//                           (infer.c:1184-1188, 1197-1201). One persistent
//                           CTA per SM owns an equal slice of the
//                           (K+1)*F rows.
//   K3 moe_down_kernel      down.h for all K+1 slots of an equal slice of the
//                           D output rows, fused with the weighted combine in
//                           rank order and the residual add
//                           (infer.c:1190-1192, 1203, 1212-1214).
//
// Exact routing. The reference's logit is a left-to-right fp32 sum. K1
// computes the same fp32 products, their sum in fp64 (the "centre") and a
// rigorous bound on how far the reference's serially rounded sum can be from
// it: 2^-24 * sum_i |prefix_i| (each serial add errs by at most half an ulp of
// its running sum), with the prefixes from an fp64 warp scan. Logit intervals
// map monotonically to sel = sigmoid + bias intervals, widened by one ulp of
// exp to cover libm differences (glibc's expf is not correctly rounded in
// about 1 of 15,000 inputs). If the K winners' intervals are pairwise disjoint
// and clear of every loser's interval, the ranking is certified. Otherwise
// every expert that could still be in the top K gets its logit recomputed in
// exactly the reference's order (serial __fadd_rn/__fmul_rn chain, no FMA),
// and the ranking is re-certified with the exp-ulp intervals; a tie that only
// libm's last bit could decide is counted in stats[2].
#include <cmath>
#include <cstdint>

#include "glm_internal.h"
#include "q80_common.cuh"

namespace glmq {

constexpr int kRouteWarps = 4;
constexpr int kRouteThreads = kRouteWarps * 32;
constexpr int kMaxTopK = 8;  // K+1 slots must fit the 16 warps of K3
constexpr int kFfnWarps = 16;
constexpr int kFfnThreads = kFfnWarps * 32;
constexpr int kUnroll = 2;

// ---------------------------------------------------------------- K1 route

struct RouteArgs {
    const float* x;
    const float* ffn_norm;
    const float* router;
    const float* bias;
    float* xn_out;
    double* center;
    double* bound;
    int32_t* topk_idx;
    float* topk_w;
    unsigned int* counter;
    unsigned long long* stats;
    int D, E, K;
};

__host__ __device__ __forceinline__ int pad64(int i) { return i + (i >> 6); }

__device__ __forceinline__ double warp_sum_d(double v) {
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
    return v;
}

// exp rounded once from a double-precision exp (<= 1 double ulp before
// rounding), i.e. correctly rounded except at vanishingly rare midpoints.
__device__ __forceinline__ float exp_cr(float v) { return (float)exp((double)v); }
__device__ __forceinline__ float sigmoid_of_exp(float e) { return __fdiv_rn(1.0f, __fadd_rn(1.0f, e)); }

// The reference's exact router logit: s = 0; s = s + w[i]*x[i], left to right.
__device__ float serial_logit(const float* __restrict__ wrow, const float* xs, int D) {
    float s = 0.0f;
    for (int i = 0; i < D; i += 4) {
        const float4 w4 = *reinterpret_cast<const float4*>(wrow + i);
        s = __fadd_rn(s, __fmul_rn(w4.x, xs[pad64(i)]));
        s = __fadd_rn(s, __fmul_rn(w4.y, xs[pad64(i + 1)]));
        s = __fadd_rn(s, __fmul_rn(w4.z, xs[pad64(i + 2)]));
        s = __fadd_rn(s, __fmul_rn(w4.w, xs[pad64(i + 3)]));
    }
    return s;
}

// rank[0..R) = experts by (sel desc, id asc) among those with sel > -inf
// (NaN never ranks), -1 when exhausted. Called by one full warp.
__device__ void warp_rank(const float* sel, int* taken, int E, int R, int* rank) {
    const int lane = threadIdx.x & 31;
    for (int e = lane; e < E; e += 32) taken[e] = 0;
    __syncwarp();
    for (int r = 0; r < R; ++r) {
        float best = -INFINITY;
        int bid = -1;
        for (int e = lane; e < E; e += 32) {
            const float v = sel[e];
            if (!taken[e] && v > best) {
                best = v;
                bid = e;
            }
        }
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) {
            const float ov = __shfl_xor_sync(0xffffffffu, best, off);
            const int oid = __shfl_xor_sync(0xffffffffu, bid, off);
            if (oid >= 0 && (bid < 0 || ov > best || (ov == best && oid < bid))) {
                best = ov;
                bid = oid;
            }
        }
        if (lane == 0) {
            rank[r] = bid;
            if (bid >= 0) taken[bid] = 2 + r;  // 2+rank marks "taken at rank"
        }
        __syncwarp();
    }
}

// True when the first K ranks are present and provably ordered: every
// adjacent pair of winners and the last winner vs every loser have disjoint
// [lo, hi] sel intervals. Called by one full warp; `taken` holds 2+rank.
__device__ bool warp_certify(const int* rank, const int* taken, const float* lo, const float* hi, int E, int K) {
    const int lane = threadIdx.x & 31;
    bool ok = true;
    for (int k = 0; k < K; ++k) ok = ok && rank[k] >= 0;
    for (int k = 0; ok && k + 1 < K; ++k) ok = lo[rank[k]] > hi[rank[k + 1]];
    float rest = -INFINITY;
    for (int e = lane; e < E; e += 32)
        if (taken[e] < 2 || taken[e] >= 2 + K) rest = fmaxf(rest, hi[e]);
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) rest = fmaxf(rest, __shfl_xor_sync(0xffffffffu, rest, off));
    if (ok) ok = lo[rank[K - 1]] > rest;
    return ok;
}

__global__ void __launch_bounds__(kRouteThreads) moe_route_kernel(RouteArgs a) {
    extern __shared__ __align__(16) unsigned char sm[];
    const int D = a.D, E = a.E, K = a.K;
    float* xs = reinterpret_cast<float*>(sm);                  // pad64(D)
    float* sel_c = xs + ((pad64(D) + 3) & ~3);                  // [E] each
    float* sel_lo = sel_c + E;
    float* sel_hi = sel_lo + E;
    float* p_c = sel_hi + E;
    int* taken = reinterpret_cast<int*>(p_c + E);
    __shared__ double red[kRouteWarps];
    __shared__ float s_inv;
    __shared__ int s_last, s_cert;
    __shared__ int s_rank[kMaxTopK + 1];

    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;

    // rmsnorm: sum of squares in fp64 (products of floats are exact in fp64).
    double ss = 0.0;
    for (int i = tid; i < D; i += kRouteThreads) {
        const double v = (double)a.x[i];
        ss = __dadd_rn(ss, __dmul_rn(v, v));
    }
    ss = warp_sum_d(ss);
    if (lane == 0) red[warp] = ss;
    __syncthreads();
    if (tid == 0) {
        double S = 0.0;
        for (int w = 0; w < kRouteWarps; ++w) S += red[w];
        // Both this sum and the reference's serial one are within
        // 2047*2^-53*S of the exact sum; certify the rounded float mean.
        const double b = S * 0x1p-40;
        const float lo = (float)((S - b) / (double)D), hi = (float)((S + b) / (double)D);
        float mean;
        if (lo == hi) {
            mean = lo;
        } else {
            double seq = 0.0;
            for (int i = 0; i < D; ++i) {
                const double v = (double)a.x[i];
                seq = __dadd_rn(seq, __dmul_rn(v, v));
            }
            mean = (float)(seq / (double)D);
            if (blockIdx.x == 0) atomicAdd(&a.stats[3], 1ull);
        }
        s_inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(mean, 1e-5f)));
    }
    __syncthreads();
    const float inv = s_inv;
    for (int i = tid; i < D; i += kRouteThreads) {
        const float v = __fmul_rn(__fmul_rn(a.x[i], inv), a.ffn_norm[i]);
        xs[pad64(i)] = v;
        if (blockIdx.x == 0) a.xn_out[i] = v;
    }
    __syncthreads();

    // Router logit centre + bound, one warp per expert, lane-contiguous blocks.
    const int per = D >> 5;
    for (int e = blockIdx.x * kRouteWarps + warp; e < E; e += gridDim.x * kRouteWarps) {
        const float* wr = a.router + (size_t)e * D + (size_t)lane * per;
        const int base = lane * per;
        double L = 0.0, sum_abs_p = 0.0;
        for (int j = 0; j < per; j += 4) {
            const float4 w4 = *reinterpret_cast<const float4*>(wr + j);
            const float p0 = __fmul_rn(w4.x, xs[pad64(base + j)]);
            const float p1 = __fmul_rn(w4.y, xs[pad64(base + j + 1)]);
            const float p2 = __fmul_rn(w4.z, xs[pad64(base + j + 2)]);
            const float p3 = __fmul_rn(w4.w, xs[pad64(base + j + 3)]);
            L += (double)p0 + (double)p1 + (double)p2 + (double)p3;
            sum_abs_p += fabs((double)p0) + fabs((double)p1) + fabs((double)p2) + fabs((double)p3);
        }
        double inc = L;
#pragma unroll
        for (int off = 1; off < 32; off <<= 1) {
            const double y = __shfl_up_sync(0xffffffffu, inc, off);
            if (lane >= off) inc += y;
        }
        const double C = __shfl_sync(0xffffffffu, inc, 31);
        double run = inc - L, sabs = 0.0;
        for (int j = 0; j < per; ++j) {
            run += (double)__fmul_rn(wr[j], xs[pad64(base + j)]);
            sabs += fabs(run);
        }
        sabs = warp_sum_d(sabs);
        sum_abs_p = warp_sum_d(sum_abs_p);
        if (lane == 0) {
            a.center[e] = C;
            a.bound[e] = 1.01 * 0x1p-24 * sabs + 0x1p-40 * sum_abs_p;
        }
    }

    // The last CTA to finish selects.
    __threadfence();
    __syncthreads();
    if (tid == 0) s_last = (atomicAdd(a.counter, 1u) == gridDim.x - 1);
    __syncthreads();
    if (!s_last) return;
    __threadfence();

    for (int e = tid; e < E; e += kRouteThreads) {
        const double C = __ldcg(a.center + e), B = __ldcg(a.bound + e);
        const float b = a.bias[e];
        const float lc = __double2float_rn(C);
        const float llo = __double2float_rd(C - B), lhi = __double2float_ru(C + B);
        const float pc = sigmoid_of_exp(exp_cr(-lc));
        p_c[e] = pc;
        sel_c[e] = __fadd_rn(pc, b);
        sel_lo[e] = __fadd_rn(sigmoid_of_exp(nextafterf(exp_cr(-llo), INFINITY)), b);
        sel_hi[e] = __fadd_rn(sigmoid_of_exp(nextafterf(exp_cr(-lhi), 0.0f)), b);
    }
    __syncthreads();
    const int R = (K + 1 < E) ? K + 1 : E;
    if (warp == 0) {
        warp_rank(sel_c, taken, E, R, s_rank);
        const bool ok = warp_certify(s_rank, taken, sel_lo, sel_hi, E, K);
        if (lane == 0) s_cert = ok ? 1 : 0;
    }
    __syncthreads();

    if (!s_cert) {
        // Every expert whose interval reaches the weakest winner's lower end
        // may be in the top K: recompute those logits exactly.
        float tau = INFINITY;
        int nvalid = 0;
        for (int k = 0; k < K; ++k)
            if (s_rank[k] >= 0) {
                tau = fminf(tau, sel_lo[s_rank[k]]);
                ++nvalid;
            }
        if (nvalid < K) tau = -INFINITY;
        __syncthreads();
        for (int e = tid; e < E; e += kRouteThreads) {
            const float hi = sel_hi[e];
            if (hi >= tau) {
                const float b = a.bias[e];
                const float l = serial_logit(a.router + (size_t)e * D, xs, D);
                const float ec = exp_cr(-l);
                const float p = sigmoid_of_exp(ec);
                p_c[e] = p;
                sel_c[e] = __fadd_rn(p, b);
                sel_lo[e] = __fadd_rn(sigmoid_of_exp(nextafterf(ec, INFINITY)), b);
                sel_hi[e] = __fadd_rn(sigmoid_of_exp(nextafterf(ec, 0.0f)), b);
            } else {
                sel_c[e] = __int_as_float(0x7fc00000);  // provably out of the top K
                sel_lo[e] = sel_c[e];
                sel_hi[e] = sel_c[e];
            }
        }
        __syncthreads();
        if (warp == 0) {
            warp_rank(sel_c, taken, E, R, s_rank);
            const bool ok = warp_certify(s_rank, taken, sel_lo, sel_hi, E, K);
            if (lane == 0) {
                atomicAdd(&a.stats[1], 1ull);
                if (!ok && nvalid == K) atomicAdd(&a.stats[2], 1ull);
            }
        }
        __syncthreads();
    }

    if (tid == 0) {
        float sum = 0.0f;
        for (int k = 0; k < K; ++k)
            if (s_rank[k] >= 0) sum = __fadd_rn(sum, p_c[s_rank[k]]);
        const bool norm = sum > 0.0f;
        const float inv_sum = norm ? __fdiv_rn(1.0f, sum < 6.103515625e-5f ? 6.103515625e-5f : sum) : 1.0f;
        for (int k = 0; k < K; ++k) {
            const int id = s_rank[k];
            float w = id >= 0 ? p_c[id] : -1e30f;
            if (norm) w = __fmul_rn(w, inv_sum);
            a.topk_idx[k] = id;
            a.topk_w[k] = w;
        }
        *a.counter = 0u;
        atomicAdd(&a.stats[0], 1ull);
    }
}

// ------------------------------------------------------------ K2 gate/up

struct GateUpArgs {
    const float* xn;
    const int32_t* topk_idx;
    const int8_t* gate_q;
    const float* gate_s;
    const int8_t* up_q;
    const float* up_s;
    const int8_t* gate_sh_q;
    const float* gate_sh_s;
    const int8_t* up_sh_q;
    const float* up_sh_s;
    float* h;
    int D, F, K, routed_enabled;
};

struct RowQ8x2 {
    const int8_t* q0 = nullptr;
    const float* s0 = nullptr;
    const int8_t* q1 = nullptr;
    const float* s1 = nullptr;
};

// Flattened row r of the (K+1)*F gate/up space -> gate row (q0,s0) and up
// row (q1,s1); null when the row is out of range or its slot is inactive.
__device__ __forceinline__ RowQ8x2 gate_up_row(const GateUpArgs& a, int r, int re) {
    RowQ8x2 p;
    if (r >= re) return p;
    const int slot = r / a.F, rr = r - slot * a.F;
    const size_t sgrp = (size_t)(a.D >> 5);
    if (slot < a.K) {
        if (!a.routed_enabled) return p;
        const int e = a.topk_idx[slot];
        if (e < 0) return p;
        const size_t row = (size_t)e * a.F + rr;
        p.q0 = a.gate_q + row * a.D;
        p.s0 = a.gate_s + row * sgrp;
        p.q1 = a.up_q + row * a.D;
        p.s1 = a.up_s + row * sgrp;
    } else {
        p.q0 = a.gate_sh_q + (size_t)rr * a.D;
        p.s0 = a.gate_sh_s + (size_t)rr * sgrp;
        p.q1 = a.up_sh_q + (size_t)rr * a.D;
        p.s1 = a.up_sh_s + (size_t)rr * sgrp;
    }
    return p;
}

__device__ __forceinline__ float silu_f(float v) { return v / (1.0f + expf(-v)); }

__global__ void __launch_bounds__(kFfnThreads, 1) moe_gate_up_kernel(GateUpArgs a) {
    extern __shared__ __align__(16) unsigned char sm[];
    const int nch = a.D >> 6;
    int8_t* planes = reinterpret_cast<int8_t*>(sm);
    float* sxg = reinterpret_cast<float*>(sm + nch * kChunkBytes);
    float* sxtab = sxg + (a.D >> 5);
    float* part = sxtab + nch * kChunkTab;  // [kFfnWarps][16][2]

    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, gid = lane >> 2, t = lane & 3;
    const int total = (a.K + 1) * a.F;
    const int rb = (int)((long long)blockIdx.x * total / gridDim.x);
    const int re = (int)((long long)(blockIdx.x + 1) * total / gridDim.x);
    const int ntiles = (re - rb + 15) >> 4;
    int ks = kFfnWarps / (ntiles > 0 ? ntiles : 1);
    ks = ks < 1 ? 1 : (ks > nch ? nch : ks);
    const int tiles_per_pass = kFfnWarps / ks;

    quantize_to_planes(a.xn, a.D, planes, sxg, sxtab);

    const int boff = b_frag_offset(lane);
    const int kq = warp % ks, tw = warp / ks;
    const int jb = kq * nch / ks, je = (kq + 1) * nch / ks;

    for (int tile0 = 0; tile0 < ntiles; tile0 += tiles_per_pass) {
        const int tile = tile0 + tw;
        float ag0 = 0.f, ag1 = 0.f, au0 = 0.f, au1 = 0.f;
        if (tw < tiles_per_pass && tile < ntiles) {
            const RowQ8x2 r0 = gate_up_row(a, rb + tile * 16 + gid, re);
            const RowQ8x2 r1 = gate_up_row(a, rb + tile * 16 + gid + 8, re);
            for (int j = jb; j < je; j += kUnroll) {
                int4 qg0[kUnroll], qg1[kUnroll], qu0[kUnroll], qu1[kUnroll];
                float2 sg0[kUnroll], sg1[kUnroll], su0[kUnroll], su1[kUnroll];
#pragma unroll
                for (int u = 0; u < kUnroll; ++u) {
                    const int jj = j + u;
                    const bool in = jj < je;
                    const int off = jj * kChunkCols + 16 * t;
                    const int4 z4 = make_int4(0, 0, 0, 0);
                    const float2 z2 = make_float2(0.f, 0.f);
                    qg0[u] = (in && r0.q0) ? ld_weights16(r0.q0 + off) : z4;
                    qg1[u] = (in && r1.q0) ? ld_weights16(r1.q0 + off) : z4;
                    qu0[u] = (in && r0.q1) ? ld_weights16(r0.q1 + off) : z4;
                    qu1[u] = (in && r1.q1) ? ld_weights16(r1.q1 + off) : z4;
                    sg0[u] = (in && r0.s0) ? ld_scales2(r0.s0 + 2 * jj) : z2;
                    sg1[u] = (in && r1.s0) ? ld_scales2(r1.s0 + 2 * jj) : z2;
                    su0[u] = (in && r0.s1) ? ld_scales2(r0.s1 + 2 * jj) : z2;
                    su1[u] = (in && r1.s1) ? ld_scales2(r1.s1 + 2 * jj) : z2;
                }
#pragma unroll
                for (int u = 0; u < kUnroll; ++u) {
                    const int jj = j + u;
                    if (jj < je) {
                        const int4 b = boff >= 0 ? *reinterpret_cast<const int4*>(planes + jj * kChunkBytes + boff)
                                                 : make_int4(0, 0, 0, 0);
                        const float2 tab = *reinterpret_cast<const float2*>(sxtab + jj * kChunkTab + 2 * t);
                        chunk_mma_accumulate(qg0[u], qg1[u], sg0[u], sg1[u], b, tab, t, ag0, ag1);
                        chunk_mma_accumulate(qu0[u], qu1[u], su0[u], su1[u], b, tab, t, au0, au1);
                    }
                }
            }
        }
        ag0 = quad_sum(ag0);
        ag1 = quad_sum(ag1);
        au0 = quad_sum(au0);
        au1 = quad_sum(au1);
        if (t == 0 && tw < tiles_per_pass) {
            float* p = part + (tw * ks + kq) * 32;
            p[gid * 2] = ag0;
            p[gid * 2 + 1] = au0;
            p[(gid + 8) * 2] = ag1;
            p[(gid + 8) * 2 + 1] = au1;
        }
        __syncthreads();
        for (int i = threadIdx.x; i < tiles_per_pass * 16; i += kFfnThreads) {
            const int tl = i >> 4, rr = i & 15;
            const int r = rb + (tile0 + tl) * 16 + rr;
            if (tile0 + tl < ntiles && r < re) {
                float gsum = 0.f, usum = 0.f;
                for (int k = 0; k < ks; ++k) {
                    gsum += part[(tl * ks + k) * 32 + rr * 2];
                    usum += part[(tl * ks + k) * 32 + rr * 2 + 1];
                }
                a.h[r] = silu_f(gsum) * usum;
            }
        }
        __syncthreads();
    }
}

// -------------------------------------------------------------- K3 down

struct DownArgs {
    const float* h;
    const int32_t* topk_idx;
    const float* topk_w;
    const int8_t* down_q;
    const float* down_s;
    const int8_t* down_sh_q;
    const float* down_sh_s;
    const float* x_in;
    float* x_out;
    int D, F, K, routed_enabled;
};

__global__ void __launch_bounds__(kFfnThreads, 1) moe_down_kernel(DownArgs a) {
    extern __shared__ __align__(16) unsigned char sm[];
    const int NS = a.K + 1, nch = a.F >> 6;
    int8_t* planes = reinterpret_cast<int8_t*>(sm);
    float* sxg = reinterpret_cast<float*>(sm + NS * nch * kChunkBytes);
    float* sxtab = sxg + NS * (a.F >> 5);
    float* part = sxtab + NS * nch * kChunkTab;  // [kFfnWarps][16]

    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, gid = lane >> 2, t = lane & 3;
    const int rb = (int)((long long)blockIdx.x * a.D / gridDim.x);
    const int re = (int)((long long)(blockIdx.x + 1) * a.D / gridDim.x);
    const int ntiles = (re - rb + 15) >> 4;
    int ks = kFfnWarps / NS;
    ks = ks < 1 ? 1 : (ks > nch ? nch : ks);

    // All K+1 activation vectors are contiguous ([slot][F], F % 64 == 0), so
    // one quantisation pass covers them; slot s starts at chunk s*nch.
    quantize_to_planes(a.h, NS * a.F, planes, sxg, sxtab);

    const int boff = b_frag_offset(lane);
    const bool active = warp < NS * ks;
    const int slot = warp / ks, kq = warp % ks;
    const int jb = kq * nch / ks, je = (kq + 1) * nch / ks;
    int expert = -1;
    if (active && slot < a.K) expert = a.routed_enabled ? a.topk_idx[slot] : -1;
    const bool slot_live = active && (slot == a.K || expert >= 0);
    const size_t fgrp = (size_t)(a.F >> 5);

    for (int tile = 0; tile < ntiles; ++tile) {
        float acc0 = 0.f, acc1 = 0.f;
        if (slot_live) {
            const int r0 = rb + tile * 16 + gid, r1 = r0 + 8;
            const int8_t *q0 = nullptr, *q1 = nullptr;
            const float *s0 = nullptr, *s1 = nullptr;
            if (slot < a.K) {
                if (r0 < re) { q0 = a.down_q + ((size_t)expert * a.D + r0) * a.F; s0 = a.down_s + ((size_t)expert * a.D + r0) * fgrp; }
                if (r1 < re) { q1 = a.down_q + ((size_t)expert * a.D + r1) * a.F; s1 = a.down_s + ((size_t)expert * a.D + r1) * fgrp; }
            } else {
                if (r0 < re) { q0 = a.down_sh_q + (size_t)r0 * a.F; s0 = a.down_sh_s + (size_t)r0 * fgrp; }
                if (r1 < re) { q1 = a.down_sh_q + (size_t)r1 * a.F; s1 = a.down_sh_s + (size_t)r1 * fgrp; }
            }
            const int8_t* pl = planes + slot * nch * kChunkBytes;
            const float* tb = sxtab + slot * nch * kChunkTab;
            for (int j = jb; j < je; j += kUnroll) {
                int4 qa[kUnroll], qb[kUnroll];
                float2 sa[kUnroll], sb[kUnroll];
#pragma unroll
                for (int u = 0; u < kUnroll; ++u) {
                    const int jj = j + u;
                    const bool in = jj < je;
                    const int off = jj * kChunkCols + 16 * t;
                    qa[u] = (in && q0) ? ld_weights16(q0 + off) : make_int4(0, 0, 0, 0);
                    qb[u] = (in && q1) ? ld_weights16(q1 + off) : make_int4(0, 0, 0, 0);
                    sa[u] = (in && s0) ? ld_scales2(s0 + 2 * jj) : make_float2(0.f, 0.f);
                    sb[u] = (in && s1) ? ld_scales2(s1 + 2 * jj) : make_float2(0.f, 0.f);
                }
#pragma unroll
                for (int u = 0; u < kUnroll; ++u) {
                    const int jj = j + u;
                    if (jj < je) {
                        const int4 b = boff >= 0 ? *reinterpret_cast<const int4*>(pl + jj * kChunkBytes + boff)
                                                 : make_int4(0, 0, 0, 0);
                        const float2 tab = *reinterpret_cast<const float2*>(tb + jj * kChunkTab + 2 * t);
                        chunk_mma_accumulate(qa[u], qb[u], sa[u], sb[u], b, tab, t, acc0, acc1);
                    }
                }
            }
        }
        acc0 = quad_sum(acc0);
        acc1 = quad_sum(acc1);
        if (t == 0) {
            part[warp * 16 + gid] = acc0;
            part[warp * 16 + gid + 8] = acc1;
        }
        __syncthreads();
        if (threadIdx.x < 16) {
            const int rr = threadIdx.x, r = rb + tile * 16 + rr;
            if (r < re) {
                // infer.c:1175,1192 then 1212-1214: acc += (1.8 w_k) y_k in rank
                // order, then x += y_shared + acc.
                float acc = 0.0f;
                for (int k = 0; k < a.K; ++k) {
                    const int e = a.topk_idx[k];
                    if (e < 0 || !a.routed_enabled) continue;
                    float y = 0.f;
                    for (int q = 0; q < ks; ++q) y += part[(k * ks + q) * 16 + rr];
                    acc = __fadd_rn(acc, __fmul_rn(__fmul_rn(a.topk_w[k], 1.8f), y));
                }
                float ysh = 0.f;
                for (int q = 0; q < ks; ++q) ysh += part[(a.K * ks + q) * 16 + rr];
                a.x_out[r] = __fadd_rn(a.x_in[r], __fadd_rn(ysh, acc));
            }
        }
        __syncthreads();
    }
}

// ------------------------------------------------------------- launcher

static size_t route_smem(int D, int E) {
    return (size_t)((pad64(D) + 3) & ~3) * 4 + (size_t)E * 4 * 4 + (size_t)E * 4;
}
static size_t gate_up_smem(int D) {
    const int nch = D >> 6;
    return (size_t)nch * kChunkBytes + (size_t)(D >> 5) * 4 + (size_t)nch * kChunkTab * 4 + kFfnWarps * 32 * 4;
}
static size_t down_smem(int F, int NS) {
    const int nch = F >> 6;
    return (size_t)NS * nch * kChunkBytes + (size_t)NS * (F >> 5) * 4 + (size_t)NS * nch * kChunkTab * 4 +
           kFfnWarps * 16 * 4;
}

cudaError_t launch_moe_decode(const MoeLayerDev& w, const MoeDims& d, const MoeScratch& s, const float* x_in,
                              float* x_out, int routed_enabled, int num_sms, cudaStream_t stream,
                              cudaEvent_t* events) {
    if (d.K < 1 || d.K > kMaxTopK || d.K > d.E || d.gs != 32 || d.D % 128 || d.F % 64) return cudaErrorInvalidValue;
    const size_t sm1 = route_smem(d.D, d.E), sm2 = gate_up_smem(d.D), sm3 = down_smem(d.F, d.K + 1);
    if (sm1 > 200 * 1024 || sm2 > 200 * 1024 || sm3 > 200 * 1024) return cudaErrorInvalidValue;
    cudaError_t err;
    if ((err = ensure_smem_attr(reinterpret_cast<const void*>(moe_route_kernel), (int)sm1)) ||
        (err = ensure_smem_attr(reinterpret_cast<const void*>(moe_gate_up_kernel), (int)sm2)) ||
        (err = ensure_smem_attr(reinterpret_cast<const void*>(moe_down_kernel), (int)sm3)))
        return err;

    RouteArgs ra{x_in, w.ffn_norm, w.router, w.router_bias, s.xn, s.center, s.bound, s.topk_idx, s.topk_w,
                 s.counter, s.stats, d.D, d.E, d.K};
    const int route_ctas = (d.E + kRouteWarps - 1) / kRouteWarps;
    if (events) cudaEventRecord(events[0], stream);
    moe_route_kernel<<<route_ctas, kRouteThreads, sm1, stream>>>(ra);
    if (events) cudaEventRecord(events[1], stream);

    GateUpArgs ga{s.xn, s.topk_idx, w.gate_q, w.gate_s, w.up_q, w.up_s, w.gate_sh_q, w.gate_sh_s,
                  w.up_sh_q, w.up_sh_s, s.h, d.D, d.F, d.K, routed_enabled && w.gate_q != nullptr};
    moe_gate_up_kernel<<<num_sms, kFfnThreads, sm2, stream>>>(ga);
    if (events) cudaEventRecord(events[2], stream);

    DownArgs da{s.h, s.topk_idx, s.topk_w, w.down_q, w.down_s, w.down_sh_q, w.down_sh_s, x_in, x_out,
                d.D, d.F, d.K, routed_enabled && w.down_q != nullptr};
    moe_down_kernel<<<num_sms, kFfnThreads, sm3, stream>>>(da);
    if (events) cudaEventRecord(events[3], stream);
    return cudaGetLastError();
}

}  // namespace glmq
