// Exact MoE routing on the GPU: the expert ids glm.c's CPU path would pick,
// bit for bit (apply_moe_shared_ffn_layer, infer.c:1098-1145).
//
// The reference's router logit is a left-to-right fp32 sum of fp32 products
// (dot_f32, infer.c:916-938); its probability is 1/(1+expf(-logit)) with
// glibc's expf; the selection sorts sel = p + bias with a strict '>' (ties go
// to the lower id) and never picks NaN or -inf. On the GPU every logit is
// known as a centre C (compensated sum of the same fp32 products) and a
// rigorous bound B on |reference logit - C|: a serial fp32 sum errs by at
// most 2^-24 * sum_i |prefix_i|, and the prefixes are estimated with their
// own error added. Logit intervals map monotonically to sel intervals,
// widened by 3 ulp of exp (CUDA's expf is within 2 ulp and glibc's within
// 0.502 ulp of the true value). If every winner's interval lies strictly
// above the interval of every expert ranked after it, the ranking is
// certified. Otherwise every expert that could still be in the top K has its
// logit recomputed in exactly the reference's order (serial __fadd_rn /
// __fmul_rn chain, no FMA) and a correctly rounded exp, and the ranking is
// re-certified; a tie that only libm's last bit could decide is counted.
#pragma once

#include <cmath>
#include <cstdint>

#include <cuda_runtime.h>

namespace glmq {

constexpr int kMaxTopK = 8;

__host__ __device__ __forceinline__ int pad64(int i) { return i + (i >> 6); }

__device__ __forceinline__ double warp_sum_d(double v) {
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
    return v;
}

__device__ __forceinline__ float warp_sum_f(float v) {
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, off));
    return v;
}

// exp rounded once from a double-precision exp, i.e. correctly rounded except
// at vanishingly rare midpoints.
__device__ __forceinline__ float exp_cr(float v) { return (float)exp((double)v); }

// n representable floats above / below a non-negative v (inf stays inf, 0
// stays 0 going down).
__device__ __forceinline__ float ulp_up(float v, int n) {
    return isinf(v) ? v : __int_as_float(__float_as_int(v) + n);
}
__device__ __forceinline__ float ulp_down(float v, int n) {
    const int b = __float_as_int(v);
    return isinf(v) ? v : (b > n ? __int_as_float(b - n) : 0.0f);
}

// Error-free transformation: s + c accumulates p with the rounding error of
// every step carried in c.
__device__ __forceinline__ void two_sum_acc(float& s, float& c, float p) {
    const float t = __fadd_rn(s, p);
    const float z = __fsub_rn(t, s);
    c = __fadd_rn(c, __fadd_rn(__fsub_rn(s, __fsub_rn(t, z)), __fsub_rn(p, z)));
    s = t;
}

// (hi, lo) += (ohi, olo), keeping the rounding error of hi + ohi.
__device__ __forceinline__ void two_sum_merge(float& hi, float& lo, float ohi, float olo) {
    const float t = __fadd_rn(hi, ohi);
    const float z = __fsub_rn(t, hi);
    const float err = __fadd_rn(__fsub_rn(hi, __fsub_rn(t, z)), __fsub_rn(ohi, z));
    lo = __fadd_rn(__fadd_rn(lo, olo), err);
    hi = t;
}

__device__ __forceinline__ float sigmoid_of_exp(float e) { return __fdiv_rn(1.0f, __fadd_rn(1.0f, e)); }

// The reference's exact router logit: s = 0; s = s + w[i]*x[i], left to right
// (infer.c:916-938), with xn in plain shared-memory layout. wrow may be in
// global or shared memory (generic loads).
__device__ __forceinline__ float serial_logit(const float* wrow, const float* xs, int D) {
    float s = 0.0f;
#pragma unroll 8
    for (int i = 0; i < D; i += 4) {
        const float4 w4 = *reinterpret_cast<const float4*>(wrow + i);
        s = __fadd_rn(s, __fmul_rn(w4.x, xs[i]));
        s = __fadd_rn(s, __fmul_rn(w4.y, xs[i + 1]));
        s = __fadd_rn(s, __fmul_rn(w4.z, xs[i + 2]));
        s = __fadd_rn(s, __fmul_rn(w4.w, xs[i + 3]));
    }
    return s;
}

// Centre and bound of one router logit, computed by the whole warps
// [0, nthreads) of a block (synchronising with `sync()`) from the router row
// `wr` and xn `xs`, both in shared memory. Row-interleaved form: element
// 32k + lane belongs to row k (k < D/32 <= 64), so every access is
// bank-conflict free and the rows are spread over the warps. The reference's
// prefixes are P_{32k+l} = R_k + Q_{k,l}: Q_{k,l} the inclusive fp32 warp scan
// of row k (tree depth 5, error <= 5u * sum|p| over the row), R_k the
// exclusive prefix of the row totals T_k from a warp scan over row pairs
// (depth <= 7, error <= 8u * sum|T| on top of the T errors), so
//   |computed prefix - exact| <= 10u * sum|p| + 8u * sum|T| + u * |computed|.
// The reference's serial sum is within u * sum_i |its prefix_i| of the exact
// sum; the returned bound B covers that plus the centre's own error.
// `scratch` holds 64 + 5 * (nthreads/32) floats. C, B are returned in thread 0.
template <int kR, typename Sync>
__device__ __forceinline__ void block_logit_bound_rows(const float* wr, const float* xs, int D, int tid, int nthreads,
                                                       float* scratch, Sync sync, double& C, double& B) {
    const int lane = tid & 31, warp = tid >> 5, nwarps = nthreads >> 5;
    const int rows = D >> 5;  // at most kR * nwarps
    float* rowtot = scratch;  // [64]
    float* w_hi = scratch + 64;
    float* w_lo = w_hi + nwarps;
    float* w_sabs = w_lo + nwarps;
    float* w_abs = w_sabs + nwarps;
    float* w_absT = w_abs + nwarps;
    // This warp's rows k = warp + j * nwarps (j < kR) stay in registers: their
    // products p and inclusive fp32 warp scans Q_{k,l}, the scans' shuffle
    // steps interleaved across the rows (each row's own sums are unchanged).
    float p[kR], v[kR];
#pragma unroll
    for (int j = 0; j < kR; ++j) {
        const int k = warp + j * nwarps;
        p[j] = k < rows ? __fmul_rn(wr[32 * k + lane], xs[32 * k + lane]) : 0.0f;
        v[j] = p[j];
    }
#pragma unroll
    for (int off = 1; off < 32; off <<= 1) {
#pragma unroll
        for (int j = 0; j < kR; ++j) {
            const float y = __shfl_up_sync(0xffffffffu, v[j], off);
            if (lane >= off) v[j] = __fadd_rn(v[j], y);
        }
    }
    float s = 0.0f, cmp = 0.0f, abs_p = 0.0f;
#pragma unroll
    for (int j = 0; j < kR; ++j) {  // rows ascending, as the serial order
        if (warp + j * nwarps < rows) {
            two_sum_acc(s, cmp, p[j]);
            abs_p += fabsf(p[j]);
            if (lane == 31) rowtot[warp + j * nwarps] = v[j];
        }
    }
    sync();
    // Every warp scans the row totals itself: lane l holds rows 2l and 2l+1.
    const float t0 = 2 * lane < rows ? rowtot[2 * lane] : 0.0f;
    const float t1 = 2 * lane + 1 < rows ? rowtot[2 * lane + 1] : 0.0f;
    float incl = __fadd_rn(t0, t1);
#pragma unroll
    for (int off = 1; off < 32; off <<= 1) {
        const float y = __shfl_up_sync(0xffffffffu, incl, off);
        if (lane >= off) incl = __fadd_rn(incl, y);
    }
    float r_even = __shfl_up_sync(0xffffffffu, incl, 1);
    if (lane == 0) r_even = 0.0f;
    const float r_odd = __fadd_rn(r_even, t0);
    float sabs = 0.0f;
#pragma unroll
    for (int j = 0; j < kR; ++j) {
        const int k = warp + j * nwarps;
        if (k < rows) {  // warp-uniform
            const float R = __shfl_sync(0xffffffffu, (k & 1) ? r_odd : r_even, k >> 1);
            sabs = __fadd_rn(sabs, fabsf(__fadd_rn(R, v[j])));
        }
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) {
        const float ohi = __shfl_xor_sync(0xffffffffu, s, off);
        const float olo = __shfl_xor_sync(0xffffffffu, cmp, off);
        two_sum_merge(s, cmp, ohi, olo);
    }
    sabs = warp_sum_f(sabs);
    abs_p = warp_sum_f(abs_p);
    const float absT = warp_sum_f(fabsf(t0) + fabsf(t1));
    if (lane == 0) {
        w_hi[warp] = s;
        w_lo[warp] = cmp;
        w_sabs[warp] = sabs;
        w_abs[warp] = abs_p;
        w_absT[warp] = absT;
    }
    sync();
    if (warp == 0) {
        float thi = lane < nwarps ? w_hi[lane] : 0.0f, tlo = lane < nwarps ? w_lo[lane] : 0.0f;
        float sa = lane < nwarps ? w_sabs[lane] : 0.0f, ab = lane < nwarps ? w_abs[lane] : 0.0f;
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) {
            const float ohi = __shfl_xor_sync(0xffffffffu, thi, off);
            const float olo = __shfl_xor_sync(0xffffffffu, tlo, off);
            two_sum_merge(thi, tlo, ohi, olo);
            sa = __fadd_rn(sa, __shfl_xor_sync(0xffffffffu, sa, off));
            ab = __fadd_rn(ab, __shfl_xor_sync(0xffffffffu, ab, off));
        }
        if (lane == 0) {
            const double u = 0x1p-24, n = (double)D;
            const double drift = 10.0 * u * (double)ab + 8.0 * u * (double)w_absT[0];
            // sa is an fp32 sum of <= 2048 non-negative terms (relative error
            // < 2e-4); 1.01 covers the reference prefixes' own deviation.
            const double sum_abs_prefix = (double)sa * 1.0002 + n * drift * 1.0001;
            C = (double)thi + (double)tlo;
            B = 1.01 * u * sum_abs_prefix + 0x1p-38 * (double)ab;
        }
    }
}

// Shared-memory scratch of block_select.
struct SelectScratch {
    float* sel_c;
    float* sel_lo;
    float* sel_hi;
    float* p_c;
    int* taken;  // rank of each expert (E = unranked)
    int* rank;   // [kMaxTopK + 1] expert at each rank, -1 past the last
    int* cert;   // [1]
};

// Ranks every expert into S.taken and the first R into S.rank (preset to -1
// and *S.cert to 1 by the caller), then clears *S.cert unless the top K are
// present and provably ordered: each winner's [lo, hi] sel interval lies
// strictly above the interval of every expert ranked after it. Two sync()s;
// nthreads a multiple of 32.
template <typename Sync>
__device__ __forceinline__ void rank_and_certify(const SelectScratch& S, int E, int K, int R, int tid, int nthreads,
                                                 Sync sync) {
    // rank_of with P threads per expert (a power of two <= 8 that fits the
    // block): thread sub of expert i counts the experts j = sub, sub + P, ...
    // that beat it, the P counts are added by shuffles within aligned lanes
    int P = 1;
    while (P < 8 && 2 * P * E <= nthreads) P <<= 1;
    for (int t = tid; t - (tid & 31) < P * E; t += nthreads) {  // warp-uniform: the warp's first t
        const int i = t / P, sub = t % P;
        int r = 0;
        bool ranks = false;
        if (i < E) {
            const float v = S.sel_c[i];
            ranks = v > -INFINITY;  // NaN and -inf never rank (infer.c:1118-1124)
            if (ranks)
                for (int j = sub; j < E; j += P) {
                    const float u = S.sel_c[j];
                    r += (u > v || (u == v && j < i)) ? 1 : 0;
                }
        }
        for (int off = 1; off < P; off <<= 1) r += __shfl_xor_sync(0xffffffffu, r, off);
        if (i < E && sub == 0) {
            if (!ranks) r = E;
            S.taken[i] = r;
            if (r < R) S.rank[r] = i;
        }
    }
    sync();
    if (tid < 32) {
        // the largest upper end among the experts ranked K or later (NaN and
        // -inf ends take no part in fmaxf), then the winners from the last
        // up, each against that and the upper ends of the winners after it
        float hm = -INFINITY;
        for (int i = tid; i < E; i += 32)
            if (S.taken[i] >= K) hm = fmaxf(hm, S.sel_hi[i]);
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) hm = fmaxf(hm, __shfl_xor_sync(0xffffffffu, hm, off));
        if (tid == 0) {
            bool ok = S.rank[K - 1] >= 0;
            for (int k = K - 1; k >= 0 && ok; --k) {
                const int w = S.rank[k];
                ok = S.sel_lo[w] > hm;
                hm = fmaxf(hm, S.sel_hi[w]);
            }
            if (!ok) *S.cert = 0;
        }
    }
    sync();
}

// Top-k selection from per-expert logit centres/bounds (shared memory), run
// by the threads [0, nthreads >= 32) of a block that synchronise with
// `sync()`. Writes the ranked expert ids to idx[K] and their normalised
// weights to w[K] (shared memory) exactly as infer.c:1110-1145 would. `xs`
// (xn in shared memory) and the router rows in global memory serve the exact
// fallback. stats (may be null): [0] calls, [1] fallbacks, [2] ties only
// libm's last bit could decide. With exact_fallback false, a ranking that
// does not certify returns with *S.cert == 0 and idx / w untouched (and
// counts nothing): the caller routes that token again with the fallback.
template <typename Sync>
__device__ void block_select(const double* center, const double* bound, const float* bias, int E, int K,
                             const float* router, const float* xs, int D, int tid, int nthreads,
                             const SelectScratch& S, int* idx, float* w, unsigned long long* stats, Sync sync,
                             float* rowbuf = nullptr, int nbuf = 0, bool exact_fallback = true) {
    // the centre, lower and upper sel of every expert, each on its own thread
    for (int t = tid; t < 3 * E; t += nthreads) {
        const int i = t % E, which = t / E;
        const double C = center[i], B = bound[i];
        const float b = bias[i];
        if (which == 0) {
            const float pc = sigmoid_of_exp(expf(-__double2float_rn(C)));
            S.p_c[i] = pc;
            S.sel_c[i] = __fadd_rn(pc, b);
        } else if (which == 1) {
            S.sel_lo[i] = __fadd_rn(sigmoid_of_exp(ulp_up(expf(-__double2float_rd(C - B)), 3)), b);
        } else {
            S.sel_hi[i] = __fadd_rn(sigmoid_of_exp(ulp_down(expf(-__double2float_ru(C + B)), 3)), b);
        }
    }
    const int R = (K + 1 < E) ? K + 1 : E;
    if (tid < R) S.rank[tid] = -1;
    if (tid == 0) *S.cert = 1;
    sync();
    rank_and_certify(S, E, K, R, tid, nthreads, sync);
    // without the fallback an uncertified ranking leaves idx / w untouched
    // and *S.cert == 0 (identical in every thread: read after a barrier)
    if (!exact_fallback && !*S.cert) return;

    if (!*S.cert) {
        // Every expert whose interval reaches the weakest winner's lower end
        // may be in the top K: recompute those logits exactly.
        float tau = INFINITY;
        int nvalid = 0;
        for (int k = 0; k < K; ++k)
            if (S.rank[k] >= 0) {
                tau = fminf(tau, S.sel_lo[S.rank[k]]);
                ++nvalid;
            }
        if (nvalid < K) tau = -INFINITY;
        sync();
        auto exact = [&](int i, const float* wrow) {
            const float b = bias[i];
            const float l = serial_logit(wrow, xs, D);
            const float ec = exp_cr(-l);
            const float p = sigmoid_of_exp(ec);
            S.p_c[i] = p;
            S.sel_c[i] = __fadd_rn(p, b);
            S.sel_lo[i] = __fadd_rn(sigmoid_of_exp(nextafterf(ec, INFINITY)), b);
            S.sel_hi[i] = __fadd_rn(sigmoid_of_exp(nextafterf(ec, 0.0f)), b);
        };
        auto drop = [&](int i) {
            S.sel_c[i] = __int_as_float(0x7fc00000);  // provably out of the top K
            S.sel_lo[i] = S.sel_c[i];
            S.sel_hi[i] = S.sel_c[i];
        };
        if (rowbuf && nbuf > 0) {
            // Candidates in batches of nbuf: their router rows are copied to
            // shared memory first, so each serial chain reads on-chip data
            // instead of waiting on L2 for every element.
            if (tid == 0) {
                int n = 0;
                for (int i = 0; i < E; ++i)
                    if (S.sel_hi[i] >= tau) S.taken[n++] = i;
                *S.cert = n;
            }
            sync();
            const int ncand = *S.cert;
            for (int i = tid; i < E; i += nthreads)
                if (!(S.sel_hi[i] >= tau)) drop(i);
            for (int b0 = 0; b0 < ncand; b0 += nbuf) {
                const int nb = ncand - b0 < nbuf ? ncand - b0 : nbuf;
                for (int v = tid * 4; v < nb * D; v += nthreads * 4) {
                    const int r = v / D, c = v - r * D;
                    *reinterpret_cast<float4*>(rowbuf + (size_t)r * D + c) =
                        __ldg(reinterpret_cast<const float4*>(router + (size_t)S.taken[b0 + r] * D + c));
                }
                sync();
                if (tid < nb) exact(S.taken[b0 + tid], rowbuf + (size_t)tid * D);
                sync();
            }
        } else {
            for (int i = tid; i < E; i += nthreads) {
                if (S.sel_hi[i] >= tau) exact(i, router + (size_t)i * D);
                else drop(i);
            }
        }
        if (tid < R) S.rank[tid] = -1;
        if (tid == 0) *S.cert = 1;
        sync();
        rank_and_certify(S, E, K, R, tid, nthreads, sync);
        if (tid == 0 && stats) {
            atomicAdd(&stats[1], 1ull);
            if (!*S.cert && nvalid == K) atomicAdd(&stats[2], 1ull);
        }
    }

    if (tid < 32) {
        // infer.c:1136-1144: sum in rank order, then w_k *= 1/max(sum, 2^-14).
        const int lane = tid;
        const int id = lane < K ? S.rank[lane] : -1;
        const float pk = id >= 0 ? S.p_c[id] : -1e30f;
        float sum = 0.0f;
        for (int k = 0; k < K; ++k) {
            const float v = __shfl_sync(0xffffffffu, pk, k);
            if (__shfl_sync(0xffffffffu, id, k) >= 0) sum = __fadd_rn(sum, v);
        }
        const bool norm = sum > 0.0f;
        const float inv_sum = norm ? __fdiv_rn(1.0f, sum < 6.103515625e-5f ? 6.103515625e-5f : sum) : 1.0f;
        if (lane < K) {
            idx[lane] = id;
            w[lane] = norm ? __fmul_rn(pk, inv_sum) : pk;
        }
        if (lane == 0 && stats) atomicAdd(&stats[0], 1ull);
    }
    sync();
}

// rmsnorm scale of infer.c:746-752, certified bit-exact: S is an fp64 sum of
// x^2 in any order. Both it and the reference's serial fp64 sum are within
// 2047 * 2^-53 * S of the exact sum, so if every value in S +- 2^-40 S
// rounds to the same float mean, that is the reference's mean; otherwise x
// (global memory) is summed serially. Returns 1/sqrtf(mean + 1e-5).
__device__ __forceinline__ float rms_inv_certified(double S, const float* x, int D, unsigned long long* fallbacks) {
    const double b = S * 0x1p-40;
    const float lo = (float)((S - b) / (double)D), hi = (float)((S + b) / (double)D);
    float mean;
    if (lo == hi) {
        mean = lo;
    } else {
        double seq = 0.0;
        for (int i = 0; i < D; ++i) {
            const double v = (double)__ldcg(x + i);
            seq = __dadd_rn(seq, __dmul_rn(v, v));
        }
        mean = (float)(seq / (double)D);
        if (fallbacks) atomicAdd(fallbacks, 1ull);
    }
    return __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(mean, 1e-5f)));
}

// The certification of rms_inv_certified alone: true and the mean glm.c
// computes if every value in S +- 2^-40 S rounds to the same float mean.
__device__ __forceinline__ bool rms_mean_certify(double S, int D, float& mean) {
    const double b = S * 0x1p-40;
    const float lo = (float)((S - b) / (double)D), hi = (float)((S + b) / (double)D);
    mean = lo;
    return lo == hi;
}

__device__ __forceinline__ float rms_inv_of_mean(float mean) {
    return __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(mean, 1e-5f)));
}

// rms_inv_certified for x held in shared memory in the padded layout
// (element i at xsp[i + 4 * (i / 64)]): the serial fallback reads on-chip.
__device__ __forceinline__ float rms_inv_certified_padded(double S, const float* xsp, int D,
                                                          unsigned long long* fallbacks) {
    const double b = S * 0x1p-40;
    const float lo = (float)((S - b) / (double)D), hi = (float)((S + b) / (double)D);
    float mean;
    if (lo == hi) {
        mean = lo;
    } else {
        double seq = 0.0;
        for (int i = 0; i < D; ++i) {
            const double v = (double)xsp[i + 4 * (i >> 6)];
            seq = __dadd_rn(seq, __dmul_rn(v, v));
        }
        mean = (float)(seq / (double)D);
        if (fallbacks) atomicAdd(fallbacks, 1ull);
    }
    return __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(mean, 1e-5f)));
}

}  // namespace glmq
