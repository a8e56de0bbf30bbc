// Batch-1 planar Q8 matvec on sm_100a: y[r] = sum_g s[r,g] * sum_k q[r,gs*g+k] x[gs*g+k]
// (gs = 32 or 16, both on the integer tensor core; see q80_common.cuh)
// Replaces matvec_q80_rows (infer.c:765-786) behind matvec_rows (infer.c:792-797).
//
// One persistent CTA per SM owns an equal contiguous slice of the rows; its
// 16 warps split the slice into 16-row tiles and, when the slice has fewer
// tiles than warps, also split the columns (k-split) and reduce through shared
// memory. The dot products run on the integer tensor core (see
// q80_common.cuh); the activation vector is quantised once per CTA into
// shared-memory digit planes.
#include <cstdint>
#include <type_traits>

#include "glm_internal.h"
#include "q80_common.cuh"

namespace glmq {

constexpr int kMvWarps = 16;
constexpr int kMvThreads = kMvWarps * 32;
constexpr int kMvUnroll = 4;
constexpr size_t kMvPrefetch = 262144;  // weight bytes per CTA pulled into L2 before the launch wait
constexpr int kMvStage = 8;            // x / norm floats per thread loaded at once (all in flight)

struct MatvecArgs {
    const int8_t* q;
    const float* s;
    const float* x;
    float* y;
    int rows, cols;
    int accumulate;      // y += result instead of y = result
    const float* norm;   // if set: x is first replaced by rmsnorm(x) * norm (infer.c:746-752)
    // optional second matrix on the same x (rows2 = 0: none): its rows follow
    // the first matrix's in the row split and land in y2
    const int8_t* q2;
    const float* s2;
    float* y2;
    int rows2;
    // 1: this CTA's weight rows are copied into shared memory before the
    // launch wait (mv_stage_bytes of them past the activation buffers)
    int stage = 0;

    __device__ __forceinline__ const int8_t* qrow(int r) const {
        return r < rows ? q + (size_t)r * cols : q2 + (size_t)(r - rows) * cols;
    }
    __device__ __forceinline__ const float* srow(int r, int groups) const {
        return r < rows ? s + (size_t)r * groups : s2 + (size_t)(r - rows) * groups;
    }
    __device__ __forceinline__ float* yrow(int r) const { return r < rows ? y + r : y2 + (r - rows); }
};

// Group-scale floats of x, rounded up to a multiple of 4 so that the table
// after them starts on a 16-byte boundary.
__host__ __device__ constexpr int sxg_floats(int cols) { return ((cols >> 5) + 3) & ~3; }

// Shared memory before the staged weights: digit planes, x-group scales,
// epilogue table, k-split partials and (with a norm) the normalised x,
// rounded up to 128 bytes.
__host__ __device__ inline size_t mv_base_bytes(int cols, bool norm) {
    const size_t nch = (size_t)(cols >> 6);
    const size_t b = nch * kChunkBytes + (size_t)sxg_floats(cols) * 4 + nch * kChunkTab * 4 + kMvWarps * 16 * 4 +
                     (norm ? (size_t)cols * 4 : 0);
    return (b + 127) & ~(size_t)127;
}

// Staged weight rows: each row's weights, then each row's scales. A 16-byte
// load is served 8 lanes at a time, i.e. 4 lanes each of 2 rows at one
// column offset: weight rows padded by 64 bytes put those two rows on
// different halves of the banks; scale rows padded by 16 bytes spread the 4
// rows of a 16-lane phase of the 8-byte scale loads.
__host__ __device__ inline int mv_qpitch(int cols) { return cols + 64; }
__host__ __device__ inline int mv_spitch(int cols, int gs) { return cols * 4 / gs + 16; }
__host__ __device__ inline size_t mv_stage_bytes(int nrows, int cols, int gs) {
    return (size_t)nrows * (size_t)(mv_qpitch(cols) + mv_spitch(cols, gs));
}

// kStage (a.stage set): the weight rows staged in shared memory; a separate
// instantiation, so that the streaming kernel keeps its own register budget.
template <int kGS, bool kStage>
__global__ void __launch_bounds__(kMvThreads, 1) q80_matvec_kernel(MatvecArgs a) {
    constexpr int kTab = kChunkTab;  // the gs = 32 table (gs = 16 reads sxg directly)
    extern __shared__ __align__(16) unsigned char sm[];
    __shared__ __align__(8) uint64_t stage_bar;
    const int rb = (int)((long long)blockIdx.x * (a.rows + a.rows2) / gridDim.x);
    const int re = (int)((long long)(blockIdx.x + 1) * (a.rows + a.rows2) / gridDim.x);
    const int qpitch = mv_qpitch(a.cols), spitch = mv_spitch(a.cols, kGS), sbytes = a.cols * 4 / kGS;
    int8_t* wq = reinterpret_cast<int8_t*>(sm + mv_base_bytes(a.cols, a.norm != nullptr));
    unsigned char* ws = reinterpret_cast<unsigned char*>(wq) + (size_t)(re - rb) * qpitch;
    if constexpr (kStage) {
        // Before waiting for the previous kernel (which writes x, never the
        // weights): copy this CTA's weight rows and scales into shared
        // memory, one bulk copy per row and part, so that the dot loop after
        // the wait reads them on chip.
        if (threadIdx.x < 32) {
            if (threadIdx.x == 0) {
                mbar_init(&stage_bar, 1);
                mbar_init_fence();
                mbar_arrive_expect_tx(&stage_bar, (uint32_t)(re - rb) * (uint32_t)(a.cols + sbytes));
            }
            __syncwarp();
            for (int i = threadIdx.x; i < re - rb; i += 32) {
                bulk_copy_g2s(wq + (size_t)i * qpitch, a.qrow(rb + i), (uint32_t)a.cols, &stage_bar);
                bulk_copy_g2s(ws + (size_t)i * spitch, a.srow(rb + i, a.cols / kGS), (uint32_t)sbytes, &stage_bar);
            }
        }
    } else {
        // Before waiting for the previous kernel (which writes x, never the
        // weights' values this kernel reads afterwards): pull the first
        // kMvPrefetch bytes of this CTA's weight rows and their scales into
        // L2 (one bulk request per contiguous range), so the stream runs
        // while the previous kernel works. A hint only: the loads below come
        // after the wait.
        const int total = a.rows + a.rows2;
        const int r0 = (int)((long long)blockIdx.x * total / gridDim.x);
        const int r1 = (int)((long long)(blockIdx.x + 1) * total / gridDim.x);
        constexpr int kSDiv = kGS / 4;  // weight bytes per scale byte
        // the slice's rows of each matrix are contiguous: [r0, r1) split at a.rows
        const int ra[2] = {r0, r0 > a.rows ? r0 : a.rows}, rz[2] = {r1 < a.rows ? r1 : a.rows, r1};
        size_t budget = kMvPrefetch;
        for (int part = 0; part < 2 && threadIdx.x == 0; ++part) {
            if (rz[part] <= ra[part] || budget == 0) continue;
            size_t qb = (size_t)(rz[part] - ra[part]) * a.cols;
            qb = qb < budget ? qb : budget;
            bulk_prefetch_l2(a.qrow(ra[part]), qb);
            bulk_prefetch_l2(a.srow(ra[part], a.cols / kGS), qb / kSDiv);
            budget -= qb;
        }
    }
    // the first kMvStage * kMvThreads norm weights (no kernel writes them)
    float nv[kMvStage];
    if (a.norm) {
#pragma unroll
        for (int u = 0; u < kMvStage; ++u) {
            const int i = threadIdx.x + u * kMvThreads;
            nv[u] = i < a.cols ? __ldg(a.norm + i) : 0.f;
        }
    }
    pdl_enter();
    const int nch = a.cols >> 6;
    int8_t* planes = reinterpret_cast<int8_t*>(sm);
    float* sxg = reinterpret_cast<float*>(sm + (size_t)nch * kChunkBytes);
    float* sxtab = sxg + sxg_floats(a.cols);  // 16-byte aligned: the gs = 16 table is read as float4
    float* part = sxtab + (size_t)nch * kTab;       // [kMvWarps][16]
    float* xs = part + kMvWarps * 16;                 // [cols] normalised x (with a.norm)

    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, gid = lane >> 2, t = lane & 3;
    const int ntiles = (re - rb + 15) >> 4;
    int ks = kMvWarps / (ntiles > 0 ? ntiles : 1);
    ks = ks < 1 ? 1 : (ks > nch ? nch : ks);
    const int tiles_per_pass = kMvWarps / ks;

    if (a.norm) {
        // rmsnorm fused into the activation load: every CTA forms the same
        // xn = x * (1/sqrtf(mean(x^2) + 1e-5)) * w (sum of squares in fp64).
        __shared__ double red[kMvWarps];
        double ss = 0.0;
        for (int base = threadIdx.x; base < a.cols; base += kMvThreads * kMvStage) {
            float v[kMvStage];
#pragma unroll
            for (int u = 0; u < kMvStage; ++u) {
                const int i = base + u * kMvThreads;
                v[u] = i < a.cols ? a.x[i] : 0.f;
            }
#pragma unroll
            for (int u = 0; u < kMvStage; ++u) {
                const int i = base + u * kMvThreads;
                if (i < a.cols) {
                    ss += (double)v[u] * (double)v[u];
                    xs[i] = v[u];
                }
            }
        }
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, off);
        if (lane == 0) red[warp] = ss;
        __syncthreads();
        double tot = 0.0;
        for (int w = 0; w < kMvWarps; ++w) tot += red[w];
        const float mean = (float)(tot / (double)a.cols);
        const float inv = 1.0f / sqrtf(mean + 1e-5f);
        for (int base = threadIdx.x, c = 0; base < a.cols; base += kMvThreads * kMvStage, ++c) {
            float w[kMvStage];
#pragma unroll
            for (int u = 0; u < kMvStage; ++u) {
                const int i = base + u * kMvThreads;
                w[u] = c == 0 ? nv[u] : (i < a.cols ? a.norm[i] : 0.f);
            }
#pragma unroll
            for (int u = 0; u < kMvStage; ++u) {
                const int i = base + u * kMvThreads;
                if (i < a.cols) xs[i] = xs[i] * inv * w[u];  // each thread rescales the xs it stored
            }
        }
        __syncthreads();
        quantize_to_planes(xs, a.cols, planes, sxg, sxtab);
    } else {
        quantize_to_planes(a.x, a.cols, planes, sxg, sxtab);
    }

    const int boff = b_frag_offset(lane);
    const G16Lane gl = g16_lane(lane);
    const int kq = warp % ks, tw = warp / ks;
    const int jb = kq * nch / ks, je = (kq + 1) * nch / ks;
    const size_t sgrp = (size_t)(a.cols / kGS);

    // the staged rows (normally landed long before): a copy that never lands
    // leaves this CTA on the global loads instead
    bool staged = false;
    if constexpr (kStage) staged = mbar_wait_bounded(&stage_bar, 0);
    auto run_tiles = [&](auto staged_tag) {
        constexpr bool kSt = decltype(staged_tag)::value;
        for (int tile0 = 0; tile0 < ntiles; tile0 += tiles_per_pass) {
            const int tile = tile0 + tw;
            float acc0 = 0.f, acc1 = 0.f;
            if (tw < tiles_per_pass && tile < ntiles) {
                const int r0 = rb + tile * 16 + gid, r1 = r0 + 8;
                const int8_t *q0, *q1;
                const float *s0, *s1;
                if constexpr (kSt) {  // this CTA's rows in shared memory
                    q0 = r0 < re ? wq + (size_t)(r0 - rb) * qpitch : nullptr;
                    q1 = r1 < re ? wq + (size_t)(r1 - rb) * qpitch : nullptr;
                    s0 = r0 < re ? reinterpret_cast<const float*>(ws + (size_t)(r0 - rb) * spitch) : nullptr;
                    s1 = r1 < re ? reinterpret_cast<const float*>(ws + (size_t)(r1 - rb) * spitch) : nullptr;
                } else {
                    q0 = r0 < re ? a.qrow(r0) : nullptr;
                    q1 = r1 < re ? a.qrow(r1) : nullptr;
                    s0 = r0 < re ? a.srow(r0, (int)sgrp) : nullptr;
                    s1 = r1 < re ? a.srow(r1, (int)sgrp) : nullptr;
                }
                const int4 z4 = make_int4(0, 0, 0, 0);
                for (int j = jb; j < je; j += kMvUnroll) {
                    int4 qa[kMvUnroll], qb[kMvUnroll];
                    float2 sa[kMvUnroll], sb[kMvUnroll];  // gs 16: .x, the scale of the lane's group
    #pragma unroll
                    for (int u = 0; u < kMvUnroll; ++u) {
                        const int jj = j + u;
                        const bool in = jj < je;
                        const int off = jj * kChunkCols + 16 * t;
                        if constexpr (kSt) {
                            qa[u] = (in && q0) ? lds16(q0 + off) : z4;
                            qb[u] = (in && q1) ? lds16(q1 + off) : z4;
                        } else {
                            qa[u] = (in && q0) ? ld_weights16(q0 + off) : z4;
                            qb[u] = (in && q1) ? ld_weights16(q1 + off) : z4;
                        }
                        sa[u] = sb[u] = make_float2(0.f, 0.f);
                        if constexpr (kGS == 32) {
                            if (in && s0) sa[u] = kSt ? *reinterpret_cast<const float2*>(s0 + 2 * jj) : ld_scales2(s0 + 2 * jj);
                            if (in && s1) sb[u] = kSt ? *reinterpret_cast<const float2*>(s1 + 2 * jj) : ld_scales2(s1 + 2 * jj);
                        } else {
                            if (in && s0) sa[u].x = kSt ? s0[4 * jj + t] : ld_scale1(s0 + 4 * jj + t);
                            if (in && s1) sb[u].x = kSt ? s1[4 * jj + t] : ld_scale1(s1 + 4 * jj + t);
                        }
                    }
    #pragma unroll
                    for (int u = 0; u < kMvUnroll; ++u) {
                        const int jj = j + u;
                        if (jj < je) {
                            const int8_t* pl = planes + jj * kChunkBytes;
                            if constexpr (kGS == 32) {
                                const int4 b = boff >= 0 ? *reinterpret_cast<const int4*>(pl + boff) : z4;
                                const float2 tab = *reinterpret_cast<const float2*>(sxtab + jj * kChunkTab + 2 * t);
                                chunk_mma_accumulate(qa[u], qb[u], sa[u], sb[u], b, tab, t, acc0, acc1);
                            } else {
                                const int4 bx = gl.offX >= 0 ? *reinterpret_cast<const int4*>(pl + gl.offX) : z4;
                                const int4 by = gl.offY >= 0 ? *reinterpret_cast<const int4*>(pl + gl.offY) : z4;
                                chunk_mma_accumulate_g16(qa[u], qb[u], sa[u].x, sb[u].x, bx, by, sxg[2 * jj + (t >> 1)],
                                                         acc0, acc1);
                            }
                        }
                    }
                }
            }
            acc0 = quad_sum(acc0);
            acc1 = quad_sum(acc1);
            if (ks == 1) {
                if (t == 0 && tw < tiles_per_pass && tile < ntiles) {
                    const int r0 = rb + tile * 16 + gid;
                    if (r0 < re) {
                        float* y = a.yrow(r0);
                        *y = a.accumulate ? *y + acc0 : acc0;
                    }
                    if (r0 + 8 < re) {
                        float* y = a.yrow(r0 + 8);
                        *y = a.accumulate ? *y + acc1 : acc1;
                    }
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
                    float* y = a.yrow(r);
                    *y = a.accumulate ? *y + sum : sum;
                }
            }
            __syncthreads();
        }
    };
    if constexpr (kStage) {
        if (staged) {
            run_tiles(std::true_type{});
            return;
        }
    }
    run_tiles(std::false_type{});
}

size_t q80_matvec_smem_bytes(int cols, bool norm, int gs) {
    (void)gs;  // both group sizes share the layout
    return mv_base_bytes(cols, norm);
}

namespace {

bool matvec_aligned(const int8_t* q, const float* s, int gs) {
    // weight rows are read 16 bytes at a time, scales 2 floats (gs 32) or 1 (gs 16) at a time
    return !(reinterpret_cast<uintptr_t>(q) & 15u) && !(reinterpret_cast<uintptr_t>(s) & (gs == 16 ? 3u : 7u));
}

// Most shared memory a matvec CTA takes with its weight rows staged.
constexpr size_t kMvStagedSmemMax = 200 * 1024;

cudaError_t launch_matvec(MatvecArgs a, int gs, int num_sms, cudaStream_t stream, bool allow_stage) {
    if ((gs != 32 && gs != 16) || a.cols % 64 || a.rows <= 0 || a.rows2 < 0) return cudaErrorInvalidValue;
    if (!matvec_aligned(a.q, a.s, gs) || (a.rows2 > 0 && !matvec_aligned(a.q2, a.s2, gs)))
        return cudaErrorMisalignedAddress;
    size_t smem = q80_matvec_smem_bytes(a.cols, a.norm != nullptr, gs);
    if (smem > 200 * 1024) return cudaErrorInvalidValue;
    int grid = num_sms;
    if (grid > (a.rows + a.rows2 + 15) / 16) grid = (a.rows + a.rows2 + 15) / 16;
    // Stage each CTA's weight rows in shared memory when the caller allows it
    // and the slice fits (the decoder's attention matrices; not the LM head).
    // Bulk copies need 16-byte multiples: a row's scales are cols / 8 bytes
    // at gs 32.
    const int slice_rows = (a.rows + a.rows2 + grid - 1) / grid;
    const size_t staged = smem + mv_stage_bytes(slice_rows, a.cols, gs);
    const bool src16 = !(reinterpret_cast<uintptr_t>(a.s) & 15u) &&
                       (a.rows2 == 0 || !((reinterpret_cast<uintptr_t>(a.q2) | reinterpret_cast<uintptr_t>(a.s2)) & 15u));
    a.stage = allow_stage && src16 && (gs == 16 || a.cols % 128 == 0) && staged <= kMvStagedSmemMax ? 1 : 0;
    if (a.stage) smem = staged;
    auto kernel = gs == 16 ? (a.stage ? q80_matvec_kernel<16, true> : q80_matvec_kernel<16, false>)
                           : (a.stage ? q80_matvec_kernel<32, true> : q80_matvec_kernel<32, false>);
    if (cudaError_t e = ensure_smem_attr(reinterpret_cast<const void*>(kernel), (int)smem)) return e;
    return launch_pdl(kernel, grid, kMvThreads, smem, stream, a);
}

}  // namespace

cudaError_t launch_q80_matvec(const int8_t* q, const float* s, const float* x, float* y, int rows, int cols,
                              int gs, int num_sms, cudaStream_t stream, bool accumulate, const float* norm,
                              bool stage) {
    MatvecArgs a{q, s, x, y, rows, cols, accumulate ? 1 : 0, norm, nullptr, nullptr, nullptr, 0};
    return launch_matvec(a, gs, num_sms, stream, stage);
}

cudaError_t launch_q80_matvec2(const int8_t* q, const float* s, float* y, int rows, const int8_t* q2,
                               const float* s2, float* y2, int rows2, const float* x, int cols, int gs, int num_sms,
                               cudaStream_t stream, const float* norm, bool stage) {
    if (rows2 <= 0) return cudaErrorInvalidValue;
    MatvecArgs a{q, s, x, y, rows, cols, 0, norm, q2, s2, y2, rows2};
    return launch_matvec(a, gs, num_sms, stream, stage);
}

}  // namespace glmq
