// Batch-1 planar Q8 matvec on sm_100a: y[r] = sum_g s[r,g] * sum_k q[r,gs*g+k] x[gs*g+k]
// (gs = 32: integer tensor-core kernel; gs = 16: CUDA-core kernel below)
// Replaces matvec_q80_rows (infer.c:765-786) behind matvec_rows (infer.c:792-797).
//
// One persistent CTA per SM owns an equal contiguous slice of the rows; its
// 16 warps split the slice into 16-row tiles and, when the slice has fewer
// tiles than warps, also split the columns (k-split) and reduce through shared
// memory. The dot products run on the integer tensor core (see
// q80_common.cuh); the activation vector is quantised once per CTA into
// shared-memory digit planes.
#include <cstdint>

#include "glm_internal.h"
#include "q80_common.cuh"

namespace glmq {

constexpr int kMvWarps = 16;
constexpr int kMvThreads = kMvWarps * 32;
constexpr int kMvUnroll = 4;
constexpr size_t kMvPrefetch = 32768;  // weight bytes per CTA pulled into L2 before the launch wait

struct MatvecArgs {
    const int8_t* q;
    const float* s;
    const float* x;
    float* y;
    int rows, cols;
    int accumulate;      // y += result instead of y = result
    const float* norm;   // if set: x is first replaced by rmsnorm(x) * norm (infer.c:746-752)
};

__global__ void __launch_bounds__(kMvThreads, 1) q80_matvec_kernel(MatvecArgs a) {
    {
        // Before waiting for the previous kernel (which writes x, never the
        // weights' values this kernel reads afterwards): pull the first
        // kMvPrefetch bytes of this CTA's weight rows and their scales into
        // L2, so the stream starts while the previous kernel drains. A hint
        // only: the loads below come after the wait.
        const long long r0 = (long long)blockIdx.x * a.rows / gridDim.x;
        const long long r1 = (long long)(blockIdx.x + 1) * a.rows / gridDim.x;
        const size_t qb = (size_t)(r1 - r0) * a.cols, sb = qb / 8;  // gs = 32: 4 bytes of scale per 32 weights
        const char* qp = reinterpret_cast<const char*>(a.q) + (size_t)r0 * a.cols;
        const char* sp = reinterpret_cast<const char*>(a.s) + (size_t)r0 * (a.cols / 8);
        for (size_t o = (size_t)threadIdx.x * 128; o < qb && o < kMvPrefetch; o += (size_t)kMvThreads * 128)
            asm volatile("prefetch.global.L2 [%0];\n" ::"l"(qp + o));
        for (size_t o = (size_t)threadIdx.x * 128; o < sb && o < kMvPrefetch / 8; o += (size_t)kMvThreads * 128)
            asm volatile("prefetch.global.L2 [%0];\n" ::"l"(sp + o));
    }
    pdl_enter();
    extern __shared__ __align__(16) unsigned char sm[];
    const int nch = a.cols >> 6;
    int8_t* planes = reinterpret_cast<int8_t*>(sm);
    float* sxg = reinterpret_cast<float*>(sm + (size_t)nch * kChunkBytes);
    float* sxtab = sxg + (a.cols >> 5);
    float* part = sxtab + (size_t)nch * kChunkTab;  // [kMvWarps][16]
    float* xs = part + kMvWarps * 16;                 // [cols] normalised x (with a.norm)

    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, gid = lane >> 2, t = lane & 3;
    const int rb = (int)((long long)blockIdx.x * a.rows / gridDim.x);
    const int re = (int)((long long)(blockIdx.x + 1) * a.rows / gridDim.x);
    const int ntiles = (re - rb + 15) >> 4;
    int ks = kMvWarps / (ntiles > 0 ? ntiles : 1);
    ks = ks < 1 ? 1 : (ks > nch ? nch : ks);
    const int tiles_per_pass = kMvWarps / ks;

    if (a.norm) {
        // rmsnorm fused into the activation load: every CTA forms the same
        // xn = x * (1/sqrtf(mean(x^2) + 1e-5)) * w (sum of squares in fp64).
        __shared__ double red[kMvWarps];
        double ss = 0.0;
        for (int i = threadIdx.x; i < a.cols; i += kMvThreads) ss += (double)a.x[i] * (double)a.x[i];
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, off);
        if (lane == 0) red[warp] = ss;
        __syncthreads();
        double tot = 0.0;
        for (int w = 0; w < kMvWarps; ++w) tot += red[w];
        const float mean = (float)(tot / (double)a.cols);
        const float inv = 1.0f / sqrtf(mean + 1e-5f);
        for (int i = threadIdx.x; i < a.cols; i += kMvThreads) xs[i] = a.x[i] * inv * a.norm[i];
        __syncthreads();
        quantize_to_planes(xs, a.cols, planes, sxg, sxtab);
    } else {
        quantize_to_planes(a.x, a.cols, planes, sxg, sxtab);
    }

    const int boff = b_frag_offset(lane);
    const int kq = warp % ks, tw = warp / ks;
    const int jb = kq * nch / ks, je = (kq + 1) * nch / ks;
    const size_t sgrp = (size_t)(a.cols >> 5);

    for (int tile0 = 0; tile0 < ntiles; tile0 += tiles_per_pass) {
        const int tile = tile0 + tw;
        float acc0 = 0.f, acc1 = 0.f;
        if (tw < tiles_per_pass && tile < ntiles) {
            const int r0 = rb + tile * 16 + gid, r1 = r0 + 8;
            const int8_t* q0 = r0 < re ? a.q + (size_t)r0 * a.cols : nullptr;
            const int8_t* q1 = r1 < re ? a.q + (size_t)r1 * a.cols : nullptr;
            const float* s0 = r0 < re ? a.s + (size_t)r0 * sgrp : nullptr;
            const float* s1 = r1 < re ? a.s + (size_t)r1 * sgrp : nullptr;
            for (int j = jb; j < je; j += kMvUnroll) {
                int4 qa[kMvUnroll], qb[kMvUnroll];
                float2 sa[kMvUnroll], sb[kMvUnroll];
#pragma unroll
                for (int u = 0; u < kMvUnroll; ++u) {
                    const int jj = j + u;
                    const bool in = jj < je;
                    const int off = jj * kChunkCols + 16 * t;
                    qa[u] = (in && q0) ? ld_weights16(q0 + off) : make_int4(0, 0, 0, 0);
                    qb[u] = (in && q1) ? ld_weights16(q1 + off) : make_int4(0, 0, 0, 0);
                    sa[u] = (in && s0) ? ld_scales2(s0 + 2 * jj) : make_float2(0.f, 0.f);
                    sb[u] = (in && s1) ? ld_scales2(s1 + 2 * jj) : make_float2(0.f, 0.f);
                }
#pragma unroll
                for (int u = 0; u < kMvUnroll; ++u) {
                    const int jj = j + u;
                    if (jj < je) {
                        const int4 b = boff >= 0 ? *reinterpret_cast<const int4*>(planes + jj * kChunkBytes + boff)
                                                 : make_int4(0, 0, 0, 0);
                        const float2 tab = *reinterpret_cast<const float2*>(sxtab + jj * kChunkTab + 2 * t);
                        chunk_mma_accumulate(qa[u], qb[u], sa[u], sb[u], b, tab, t, acc0, acc1);
                    }
                }
            }
        }
        acc0 = quad_sum(acc0);
        acc1 = quad_sum(acc1);
        if (ks == 1) {
            if (t == 0 && tw < tiles_per_pass && tile < ntiles) {
                const int r0 = rb + tile * 16 + gid;
                if (r0 < re) a.y[r0] = a.accumulate ? a.y[r0] + acc0 : acc0;
                if (r0 + 8 < re) a.y[r0 + 8] = a.accumulate ? a.y[r0 + 8] + acc1 : acc1;
            }
            continue;  // uniform across the CTA: ks is
        }
        if (t == 0 && tw < tiles_per_pass) {
            part[warp * 16 + gid] = acc0;
            part[warp * 16 + gid + 8] = acc1;
        }
        __syncthreads();
        for (int i = threadIdx.x; i < tiles_per_pass * 16; i += kMvThreads) {
            const int tl = i >> 4, rr = i & 15;
            const int r = rb + (tile0 + tl) * 16 + rr;
            if (tile0 + tl < ntiles && r < re) {
                float sum = 0.f;
                for (int k = 0; k < ks; ++k) sum += part[(tl * ks + k) * 16 + rr];
                a.y[r] = a.accumulate ? a.y[r] + sum : sum;
            }
        }
        __syncthreads();
    }
}

// gs = 16 (glm.c's own export, glm47_flash_export.py:36): the int8 MMA of
// the kernel above sums 32 columns under one weight scale, so 16-column
// groups take this CUDA-core kernel instead. Lane = one 16-byte group per
// step (coalesced 512-byte warp loads), int8 -> fp32 by the exponent trick,
// per-group dot, then s[row][group] * dot accumulated as in glm.c's
// matvec_q80_rows (infer.c:765-786); one warp per row, rows strided over
// the persistent CTAs.
constexpr int kG16Warps = 16;

__global__ void __launch_bounds__(kG16Warps * 32) q80_matvec_g16_kernel(MatvecArgs a) {
    pdl_enter();
    extern __shared__ __align__(16) unsigned char sm16[];
    float* xs = reinterpret_cast<float*>(sm16);  // [cols]
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    if (a.norm) {
        __shared__ double red[kG16Warps];
        double ss = 0.0;
        for (int i = threadIdx.x; i < a.cols; i += blockDim.x) ss += (double)a.x[i] * (double)a.x[i];
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, off);
        if (lane == 0) red[warp] = ss;
        __syncthreads();
        double tot = 0.0;
        for (int w = 0; w < kG16Warps; ++w) tot += red[w];
        const float mean = (float)(tot / (double)a.cols);
        const float inv = 1.0f / sqrtf(mean + 1e-5f);
        for (int i = threadIdx.x; i < a.cols; i += blockDim.x) xs[i] = a.x[i] * inv * a.norm[i];
    } else {
        for (int i = threadIdx.x; i < a.cols; i += blockDim.x) xs[i] = a.x[i];
    }
    __syncthreads();
    const int ng = a.cols >> 4;
    for (int r = blockIdx.x * kG16Warps + warp; r < a.rows; r += gridDim.x * kG16Warps) {
        const int8_t* qr = a.q + (size_t)r * a.cols;
        const float* sr = a.s + (size_t)r * ng;
        float acc = 0.0f;
        for (int g = lane; g < ng; g += 32) {
            const int4 q = ld_weights16(qr + 16 * g);
            const float sc = __ldg(sr + g);
            const float4* xv = reinterpret_cast<const float4*>(xs + 16 * g);
            const uint32_t w4[4] = {(uint32_t)q.x, (uint32_t)q.y, (uint32_t)q.z, (uint32_t)q.w};
            float dot = 0.0f;
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const float4 x4 = xv[j];
                const uint32_t u = w4[j] ^ 0x80808080u;  // bytes q + 128
                const float q0 = __uint_as_float(__byte_perm(u, 0x4B000000u, 0x7650)) - 8388736.0f;
                const float q1 = __uint_as_float(__byte_perm(u, 0x4B000000u, 0x7651)) - 8388736.0f;
                const float q2 = __uint_as_float(__byte_perm(u, 0x4B000000u, 0x7652)) - 8388736.0f;
                const float q3 = __uint_as_float(__byte_perm(u, 0x4B000000u, 0x7653)) - 8388736.0f;
                dot = fmaf(q0, x4.x, dot);
                dot = fmaf(q1, x4.y, dot);
                dot = fmaf(q2, x4.z, dot);
                dot = fmaf(q3, x4.w, dot);
            }
            acc = fmaf(sc, dot, acc);
        }
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, off);
        if (lane == 0) a.y[r] = a.accumulate ? a.y[r] + acc : acc;
    }
}

size_t q80_matvec_smem_bytes(int cols, bool norm) {
    const int nch = cols >> 6;
    return (size_t)nch * kChunkBytes + (size_t)(cols >> 5) * 4 + (size_t)nch * kChunkTab * 4 + kMvWarps * 16 * 4 +
           (norm ? (size_t)cols * 4 : 0);
}

cudaError_t launch_q80_matvec(const int8_t* q, const float* s, const float* x, float* y, int rows, int cols,
                              int gs, int num_sms, cudaStream_t stream, bool accumulate, const float* norm) {
    if ((gs != 32 && gs != 16) || cols % 64 || rows <= 0) return cudaErrorInvalidValue;
    if (gs == 16) {
        const size_t smem16 = (size_t)cols * 4;
        if (smem16 > 200 * 1024) return cudaErrorInvalidValue;
        cudaError_t e = ensure_smem_attr(reinterpret_cast<const void*>(q80_matvec_g16_kernel), (int)smem16);
        if (e) return e;
        int grid = num_sms * 2;
        if (grid > (rows + kG16Warps - 1) / kG16Warps) grid = (rows + kG16Warps - 1) / kG16Warps;
        MatvecArgs a{q, s, x, y, rows, cols, accumulate ? 1 : 0, norm};
        return launch_pdl(q80_matvec_g16_kernel, grid, kG16Warps * 32, smem16, stream, a);
    }
    const size_t smem = q80_matvec_smem_bytes(cols, norm != nullptr);
    if (smem > 200 * 1024) return cudaErrorInvalidValue;
    if (cudaError_t e = ensure_smem_attr(reinterpret_cast<const void*>(q80_matvec_kernel), (int)smem)) return e;
    int grid = num_sms;
    if (grid > (rows + 15) / 16) grid = (rows + 15) / 16;
    MatvecArgs a{q, s, x, y, rows, cols, accumulate ? 1 : 0, norm};
    return launch_pdl(q80_matvec_kernel, grid, kMvThreads, smem, stream, a);
}

}  // namespace glmq
