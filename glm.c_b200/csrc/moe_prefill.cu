// Batched MoE prefill on sm_100a: T tokens through one MoE FFN layer
// (apply_moe_shared_ffn_layer, infer.c:1087-1216, applied to every token),
// with the expert products as grouped GEMMs on the 5th-generation tensor
// cores (tcgen05, accumulators in TMEM).
//
//   1 route_logits_kernel    certified rmsnorm; glm.c's router logits to
//                            the bit (serial fp32 chains, one per pair)
//   2 route_select_kernel    top-k (route_common.cuh) -> ids, weights
//   3 route_exact_kernel     the rare token whose ranking expf's last bits
//                            could decide, with the exact fallback
//   4 prefill_dispatch_kernel rows = (token, slot) pairs grouped by expert
//                            (+ the shared expert: every token), tile lists
//   5 gather_split_kernel    activation rows as bf16 hi + lo
//   6 q8_group_gemm_kernel   gate and up + SwiGLU: h = silu(xn . Wg) * (xn . Wu)
//   7 q8_group_gemm_kernel   down: Y[row][d] = h . Wd[d]
//   8 prefill_combine_kernel x += y_shared + sum_k (1.8 w_k) y_k, rank order
//
// Precision. The Q8 weights are dequantised in shared memory to bf16 pairs
// w = w_hi + w_lo (w_hi = bf16(q*s), w_lo = bf16(q*s - w_hi)) and the
// activations likewise; each tile runs the three MMAs hi*hi + hi*lo + lo*hi
// into one fp32 accumulator, so every product carries ~16 significant bits
// (relative error ~2^-16) instead of bf16's 8 -- the MoE output stays well
// inside the 1e-3 bar while the products run on the tensor cores.
//
// GEMM kernel. One persistent CTA per SM walks a list of tiles
// (expert, 64-row token tile, 128-row weight tile). Per 64-column K stage the
// 256 threads copy the int8 weight tile and its scales (cp.async) and the
// token tile's bf16 rows (straight into the 128-byte-swizzled K-major
// operand layout), two stages ahead of use; dequantise the weight tile into
// the A operands; and one thread issues the 12 tcgen05.mma (4 K-steps x 3
// products) with A = weights (M = 128) and B = tokens (N = 64), then commits
// to the stage buffer's mbarrier. The accumulator (128 x 64 fp32) lives in
// TMEM; four warps read it back with tcgen05.ld (thread = weight row).
#include <cstdint>
#include <utility>

#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include "glm_internal.h"
#include "q80_common.cuh"
#include "route_common.cuh"

namespace glmq {

namespace {

constexpr int kMaxGroups = 257;  // routed experts + the shared expert
constexpr int kTM = 128;     // weight rows per tile (MMA M)
constexpr int kTN = 128;     // token rows per tile (MMA N <= 128)
constexpr int kTK = 64;      // K per stage (bf16: 128 bytes per row = one swizzle atom)
constexpr uint64_t kGWaitNs = 2000000000ull;

// tcgen05 shared-memory descriptor: K-major, 128-byte swizzle, 8-row groups
// 1024 bytes apart (SBO), LBO 16 bytes, descriptor version 1.
__device__ __forceinline__ uint64_t umma_desc(uint32_t saddr) {
    return (uint64_t)((saddr >> 4) & 0x3FFFu) | ((uint64_t)1 << 16) | ((uint64_t)(1024 >> 4) << 32) |
           ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}

__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;\n" ::: "memory"); }
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;\n" ::: "memory"); }

__device__ __forceinline__ void tc_commit(uint64_t* bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];\n" ::"r"(smem_addr(bar))
                 : "memory");
}

__device__ __forceinline__ void tc_ld32(uint32_t taddr, float (&v)[32]) {
    uint32_t r[32];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
        "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];\n"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
          "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
          "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;\n" ::: "memory");
#pragma unroll
    for (int j = 0; j < 32; ++j) v[j] = __uint_as_float(r[j]);
}

__device__ __forceinline__ void split_bf16(float v, __nv_bfloat16& hi, __nv_bfloat16& lo) {
    hi = __float2bfloat16_rn(v);
    const float h = __bfloat162float(hi);
    lo = __float2bfloat16_rn(isinf(h) ? 0.0f : v - h);  // inf stays inf, not inf + NaN
}

// ------------------------------------------------------------------ routing

// Batched form, four kernels.
//
// route_norm_kernel: one warp per token. The row stays in registers between
// the fp64 sum of squares (certified rmsnorm scale, infer.c:746-752) and
// xn = (x * inv) * ffn_norm (infer.c:751), written to a.xn for the router and
// the GEMM gather.
//
// route_logits_kernel<NT, NE>: glm.c's router logits themselves, to the bit
// (dot_f32, infer.c:916-938: s = 0; s = s + w[i] * xn[i], each product and
// sum rounded to fp32, left to right). Every (token, expert) pair is one
// serial chain of two fp32 instructions per element -- fewer than any
// reassociated sum with a rigorous error bound needs -- and with T tokens
// there are T x E independent chains. A lane holds NT x NE chains (tokens
// ty + 4k, experts tx + 8j of its warp's tile; ty = lane / 8, tx = lane % 8),
// so one float4 of a token row and one of a router row feed NE and NT
// chains: shared-memory traffic per instruction falls as NT x NE grows. Two
// warps (stacked along the tokens) share the router rows. D streams through
// a ring of kLD-element chunks (as many as ~100 KB holds), xn rows and router
// rows both by cp.async. Rows are padded by 4 floats, so the 8 router rows a quarter-warp
// reads fall in distinct bank groups; a token row is a broadcast. Rows past
// the end are zero: s + 0 is s for every s the chain can hold (it starts at
// +0, so it is never -0). The select kernel receives each logit as a centre
// with bound 0.
//
// route_select_kernel: kRT tokens per CTA, 64 threads each on a named
// barrier: the same certified top-k as the decode path (route_common.cuh),
// without the exact fallback, so a CTA needs ~2.6 KB of shared memory and a
// whole batch of tokens is resident at once. With exact logits a ranking
// fails to certify only where expf's last bits could reorder two experts;
// such a token gets kRouteRedo as its first id and is routed again by
// route_exact_kernel.
constexpr int kRouteRedo = -2;         // never a routing result (ids are -1 .. E-1)
constexpr int kExactCtas = 296;        // route_exact_kernel CTAs (two per SM)
constexpr int kSelRows = 8;            // router rows staged at a time by the exact fallback
constexpr int kNormRegs = 16;          // float4 of a row a lane keeps (D <= 2048); longer rows are read twice
constexpr int kLWarps = 2;             // logit CTA: warps, stacked along the tokens
constexpr int kLThreads = 32 * kLWarps;
constexpr int kLD = 128;               // D elements per staged chunk
constexpr int kLPrefetch = 3;          // short tiles: steps between an operand load and its use
constexpr int kLRow = kLD + 4;         // padded row, floats
constexpr size_t kLRingBytes = 104 * 1024;  // logit CTA's chunk ring: two CTAs per SM
constexpr int kRT = 1;                 // tokens per select CTA
constexpr int kRThreads = 64 * kRT;

__device__ __forceinline__ void token_bar(int tb) {
    asm volatile("bar.sync %0, 64;\n" ::"r"(1 + tb) : "memory");
}

// 16-byte global -> shared copy; src_bytes 0 writes zeros (src not read).
__device__ __forceinline__ void cp_async16(void* dst, const void* src, int src_bytes) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(smem_addr(dst)), "l"(src), "r"(src_bytes)
                 : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
    asm volatile("cp.async.wait_group %0;\n" ::"n"(N) : "memory");
}

__global__ void __launch_bounds__(256) route_norm_kernel(PrefillRouteArgs a) {
    const int lane = threadIdx.x & 31, t = blockIdx.x * 8 + (threadIdx.x >> 5);
    if (t >= a.T) return;  // per-warp work only: no block barrier
    const int D = a.D, n4 = D / 4;
    const float4* xr = reinterpret_cast<const float4*>(a.x + (size_t)t * D);
    const float4* nr = reinterpret_cast<const float4*>(a.norm);
    float4* xo = reinterpret_cast<float4*>(a.xn + (size_t)t * D);
    const bool in_regs = n4 <= 32 * kNormRegs;
    float4 v[kNormRegs];
    double ss = 0.0;
    if (in_regs) {
#pragma unroll
        for (int k = 0; k < kNormRegs; ++k) {
            const int c = lane + 32 * k;
            v[k] = c < n4 ? xr[c] : make_float4(0.f, 0.f, 0.f, 0.f);
        }
#pragma unroll
        for (int k = 0; k < kNormRegs; ++k)
            ss += (double)v[k].x * v[k].x + (double)v[k].y * v[k].y + (double)v[k].z * v[k].z +
                  (double)v[k].w * v[k].w;
    } else {
        for (int c = lane; c < n4; c += 32) {
            const float4 u = xr[c];
            ss += (double)u.x * u.x + (double)u.y * u.y + (double)u.z * u.z + (double)u.w * u.w;
        }
    }
    ss = warp_sum_d(ss);
    float inv = 0.0f;
    if (lane == 0) inv = rms_inv_certified(ss, a.x + (size_t)t * D, D, a.stats ? &a.stats[3] : nullptr);
    inv = __shfl_sync(0xffffffffu, inv, 0);
    auto out = [&](int c, float4 u) {
        const float4 w = __ldg(nr + c);
        float4 o;  // infer.c:751: (x * inv) * w
        o.x = __fmul_rn(__fmul_rn(u.x, inv), w.x);
        o.y = __fmul_rn(__fmul_rn(u.y, inv), w.y);
        o.z = __fmul_rn(__fmul_rn(u.z, inv), w.z);
        o.w = __fmul_rn(__fmul_rn(u.w, inv), w.w);
        xo[c] = o;
    };
    if (in_regs) {
#pragma unroll
        for (int k = 0; k < kNormRegs; ++k)
            if (lane + 32 * k < n4) out(lane + 32 * k, v[k]);
    } else {
        for (int c = lane; c < n4; c += 32) out(c, xr[c]);
    }
}

// Chunks in flight: as many as kLRingBytes holds. A short tile computes a
// chunk in a fraction of the L2 latency, so it needs the deeper ring.
__host__ __device__ constexpr int route_logits_stages(int NT, int NE) {
    return (int)(kLRingBytes / (sizeof(float) * (size_t)(kLWarps * 4 * NT + 8 * NE) * kLRow));
}
__host__ __device__ constexpr size_t route_logits_smem(int NT, int NE) {
    return sizeof(float) * route_logits_stages(NT, NE) * (size_t)(kLWarps * 4 * NT + 8 * NE) * kLRow;
}

// Four elements of every chain of a lane: s = s + w * x, rounded per step
// (infer.c:920-926).
template <int NT, int NE>
__device__ __forceinline__ void logit_step(float (&acc)[NT][NE], const float4 (&xq)[NT], const float4 (&wq)[NE]) {
#pragma unroll
    for (int k = 0; k < NT; ++k)
#pragma unroll
        for (int j = 0; j < NE; ++j) {
            acc[k][j] = __fadd_rn(acc[k][j], __fmul_rn(wq[j].x, xq[k].x));
            acc[k][j] = __fadd_rn(acc[k][j], __fmul_rn(wq[j].y, xq[k].y));
            acc[k][j] = __fadd_rn(acc[k][j], __fmul_rn(wq[j].z, xq[k].z));
            acc[k][j] = __fadd_rn(acc[k][j], __fmul_rn(wq[j].w, xq[k].w));
        }
}

template <int NT, int NE>
__global__ void __launch_bounds__(kLThreads, 1) route_logits_kernel(PrefillRouteArgs a) {
    constexpr int TT = kLWarps * 4 * NT, TE = 8 * NE, ROWS = TT + TE;
    constexpr int CP = ROWS * (kLD / 4) / kLThreads;  // cp.async per thread per chunk
    constexpr int kLStages = route_logits_stages(NT, NE);
    static_assert(kLStages >= 3, "the ring holds at least three chunks");
    static_assert(ROWS * (kLD / 4) % kLThreads == 0, "chunk copies split evenly over the threads");
    extern __shared__ __align__(16) unsigned char smr[];
    float* ring = reinterpret_cast<float*>(smr);  // [kLStages][ROWS][kLRow]: TT xn rows, then TE router rows
    const int D = a.D, E = a.E, T = a.T;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int ty = lane >> 3, tx = lane & 7;
    const int t0 = blockIdx.x * TT, e0 = blockIdx.y * TE;
    const int nch = D / kLD;

    auto stage = [&](int c, int slot) {
        float* dst = ring + (size_t)slot * ROWS * kLRow;
#pragma unroll
        for (int k = 0; k < CP; ++k) {
            const int q = tid + k * kLThreads, r = q >> 5, c4 = q & 31;
            const float* src;
            bool ok;
            if (r < TT) {
                ok = t0 + r < T;
                src = a.xn + (size_t)(ok ? t0 + r : 0) * D;
            } else {
                ok = e0 + r - TT < E;
                src = a.router + (size_t)(ok ? e0 + r - TT : 0) * D;
            }
            cp_async16(dst + r * kLRow + 4 * c4, src + c * kLD + 4 * c4, ok ? 16 : 0);
        }
    };
#pragma unroll
    for (int s = 0; s < kLStages - 1; ++s) {
        if (s < nch) stage(s, s);
        cp_async_commit();  // one group per chunk, empty past the end
    }

    float acc[NT][NE];
#pragma unroll
    for (int k = 0; k < NT; ++k)
#pragma unroll
        for (int j = 0; j < NE; ++j) acc[k][j] = 0.0f;
    for (int c = 0; c < nch; ++c) {
        cp_async_wait<kLStages - 2>();  // this thread's copies of chunk c have landed
        __syncthreads();                // everyone's have; chunk c - 1's slot is free
        if (c + kLStages - 1 < nch) stage(c + kLStages - 1, (c + kLStages - 1) % kLStages);
        cp_async_commit();
        const float* base = ring + (size_t)(c % kLStages) * ROWS * kLRow;
        const float* xb = base + (warp * 4 * NT + ty) * kLRow;
        const float* wb = base + (TT + tx) * kLRow;
        if constexpr (NT * NE >= 16) {
            // enough independent chains per lane to cover the shared-memory latency
#pragma unroll 2
            for (int i = 0; i < kLD; i += 4) {
                float4 xq[NT], wq[NE];
#pragma unroll
                for (int k = 0; k < NT; ++k) xq[k] = *reinterpret_cast<const float4*>(xb + 4 * k * kLRow + i);
#pragma unroll
                for (int j = 0; j < NE; ++j) wq[j] = *reinterpret_cast<const float4*>(wb + 8 * j * kLRow + i);
                logit_step<NT, NE>(acc, xq, wq);
            }
        } else {
            // few chains: each step's operands are loaded kLPrefetch steps ahead (a
            // step's dependent adds take less time than a shared-memory load)
            float4 xq[kLPrefetch][NT], wq[kLPrefetch][NE];
#pragma unroll
            for (int st = 0; st < kLD / 4 + kLPrefetch; ++st) {
                if (st >= kLPrefetch) logit_step<NT, NE>(acc, xq[st % kLPrefetch], wq[st % kLPrefetch]);
                if (st < kLD / 4) {
#pragma unroll
                    for (int k = 0; k < NT; ++k)
                        xq[st % kLPrefetch][k] = *reinterpret_cast<const float4*>(xb + 4 * k * kLRow + 4 * st);
#pragma unroll
                    for (int j = 0; j < NE; ++j)
                        wq[st % kLPrefetch][j] = *reinterpret_cast<const float4*>(wb + 8 * j * kLRow + 4 * st);
                }
            }
        }
    }
    cp_async_wait<0>();  // no copy outlives the CTA (the trailing groups are empty)
#pragma unroll
    for (int k = 0; k < NT; ++k)
#pragma unroll
        for (int j = 0; j < NE; ++j) {
            const int t = t0 + warp * 4 * NT + ty + 4 * k, e = e0 + tx + 8 * j;
            if (t < T && e < E) {
                a.cen[(size_t)t * E + e] = (double)acc[k][j];
                a.bnd[(size_t)t * E + e] = 0.0;
            }
        }
}

__global__ void __launch_bounds__(kRThreads) route_select_kernel(PrefillRouteArgs a) {
    extern __shared__ __align__(16) unsigned char smr[];
    const int E = a.E, K = a.K, D = a.D;
    const int tid = threadIdx.x, warp = tid >> 5, tb = warp >> 1, ltid = tid & 63;
    const int t = blockIdx.x * kRT + tb;
    if (t >= a.T) return;  // both warps of the token leave together; barriers are per token
    double* cen = reinterpret_cast<double*>(smr) + (size_t)tb * 2 * E;
    double* bnd = cen + E;
    float* sel = reinterpret_cast<float*>(reinterpret_cast<double*>(smr) + (size_t)kRT * 2 * E) + (size_t)tb * 5 * E;
    int* misc = reinterpret_cast<int*>(reinterpret_cast<float*>(reinterpret_cast<double*>(smr) + (size_t)kRT * 2 * E) +
                                       (size_t)kRT * 5 * E) + tb * 64;
    // xn and the router rows stay in global memory (L2): only the rare exact
    // fallback reads them, so the CTA keeps ~2.6 KB of shared memory and a
    // whole batch of tokens is resident at once
    const float* xs = a.xn + (size_t)t * D;
    for (int i = ltid; i < E; i += 64) {
        cen[i] = a.cen[(size_t)t * E + i];
        bnd[i] = a.bnd[(size_t)t * E + i];
    }
    SelectScratch S;
    S.sel_c = sel;
    S.sel_lo = sel + E;
    S.sel_hi = sel + 2 * E;
    S.p_c = sel + 3 * E;
    S.taken = reinterpret_cast<int*>(sel + 4 * E);
    S.rank = misc;
    S.cert = misc + 16;
    int* s_idx = misc + 32;
    float* s_w = reinterpret_cast<float*>(misc + 48);
    token_bar(tb);
    block_select(cen, bnd, a.bias, E, K, a.router, xs, D, ltid, 64, S, s_idx, s_w,
                 (warp & 1) == 0 ? a.stats : nullptr, [tb]() { token_bar(tb); }, nullptr, 0, false);
    if (!*S.cert) {
        if (ltid == 0) a.topk_idx[(size_t)t * K] = kRouteRedo;  // route_exact_kernel takes it
    } else if (ltid < K) {
        a.topk_idx[(size_t)t * K + ltid] = s_idx[ltid];
        a.topk_w[(size_t)t * K + ltid] = s_w[ltid];
    }
}

// Byte offset of route_exact_kernel's staged xn: after the centres, bounds,
// sel arrays and 64 ints, rounded up to 16 bytes.
__host__ __device__ __forceinline__ size_t exact_xs_offset(int E) {
    return ((size_t)E * (2 * sizeof(double) + 5 * sizeof(float)) + 64 * sizeof(int) + 15) & ~(size_t)15;
}

// The tokens route_select_kernel marked kRouteRedo, each by a whole CTA of
// 64 threads in turn: block_select with the exact fallback, xn and the
// candidates' router rows staged in shared memory (serial chains on on-chip
// data). CTAs step over the unmarked tokens.
__global__ void __launch_bounds__(64) route_exact_kernel(PrefillRouteArgs a) {
    extern __shared__ __align__(16) unsigned char smr[];
    const int E = a.E, K = a.K, D = a.D, tid = threadIdx.x;
    double* cen = reinterpret_cast<double*>(smr);
    double* bnd = cen + E;
    float* sel = reinterpret_cast<float*>(bnd + E);
    int* misc = reinterpret_cast<int*>(sel + 5 * E);
    float* xs = reinterpret_cast<float*>(smr + exact_xs_offset(E));  // 16-byte aligned: float4 staging
    float* rowbuf = xs + D;
    SelectScratch S;
    S.sel_c = sel;
    S.sel_lo = sel + E;
    S.sel_hi = sel + 2 * E;
    S.p_c = sel + 3 * E;
    S.taken = reinterpret_cast<int*>(sel + 4 * E);
    S.rank = misc;
    S.cert = misc + 16;
    int* s_idx = misc + 32;
    float* s_w = reinterpret_cast<float*>(misc + 48);
    for (int t = blockIdx.x; t < a.T; t += gridDim.x) {
        if (a.topk_idx[(size_t)t * K] != kRouteRedo) continue;  // the same in every thread
        for (int i = tid; i < E; i += 64) {
            cen[i] = a.cen[(size_t)t * E + i];
            bnd[i] = a.bnd[(size_t)t * E + i];
        }
        for (int i = tid * 4; i < D; i += 256)
            *reinterpret_cast<float4*>(xs + i) = *reinterpret_cast<const float4*>(a.xn + (size_t)t * D + i);
        __syncthreads();
        block_select(cen, bnd, a.bias, E, K, a.router, xs, D, tid, 64, S, s_idx, s_w, a.stats,
                     []() { __syncthreads(); }, rowbuf, kSelRows);
        if (tid < K) {
            a.topk_idx[(size_t)t * K + tid] = s_idx[tid];
            a.topk_w[(size_t)t * K + tid] = s_w[tid];
        }
        __syncthreads();  // the shared arrays are refilled for the next token
    }
}

template <int NT, int NE>
cudaError_t launch_route_logits(const PrefillRouteArgs& ra, cudaStream_t st) {
    const size_t smem = route_logits_smem(NT, NE);
    cudaError_t err = ensure_smem_attr(reinterpret_cast<const void*>(route_logits_kernel<NT, NE>), (int)smem);
    if (err) return err;
    const int tt = kLWarps * 4 * NT, te = 8 * NE;
    route_logits_kernel<NT, NE><<<dim3((ra.T + tt - 1) / tt, (ra.E + te - 1) / te), kLThreads, smem, st>>>(ra);
    return cudaGetLastError();
}

// The largest per-lane chain tile (shared-memory traffic per instruction
// falls with it) that still gives every SM a CTA; a small batch takes short
// tiles, since a lane's chains run one after another.
cudaError_t launch_route_logit_tiles(const PrefillRouteArgs& ra, int num_sms, cudaStream_t st) {
    auto ctas = [&](int nt, int ne) {
        return (long)((ra.T + kLWarps * 4 * nt - 1) / (kLWarps * 4 * nt)) * ((ra.E + 8 * ne - 1) / (8 * ne));
    };
    if (ctas(4, 4) >= num_sms) return launch_route_logits<4, 4>(ra, st);
    if (ctas(2, 2) >= num_sms) return launch_route_logits<2, 2>(ra, st);
    return launch_route_logits<1, 2>(ra, st);
}

cudaError_t launch_route_batched(const PrefillRouteArgs& ra, int num_sms, cudaStream_t st) {
    if (ra.D % kLD) return cudaErrorInvalidValue;
    route_norm_kernel<<<(ra.T + 7) / 8, 256, 0, st>>>(ra);
    cudaError_t err = launch_route_logit_tiles(ra, num_sms, st);
    if (err) return err;
    const size_t smem2 = (size_t)kRT * (2 * ra.E * sizeof(double) + 5 * ra.E * sizeof(float) + 64 * sizeof(int));
    if ((err = ensure_smem_attr(reinterpret_cast<const void*>(route_select_kernel), (int)smem2))) return err;
    route_select_kernel<<<(ra.T + kRT - 1) / kRT, kRThreads, smem2, st>>>(ra);
    const size_t smem3 = exact_xs_offset(ra.E) + (1 + kSelRows) * (size_t)ra.D * sizeof(float);
    if ((err = ensure_smem_attr(reinterpret_cast<const void*>(route_exact_kernel), (int)smem3))) return err;
    route_exact_kernel<<<ra.T < kExactCtas ? ra.T : kExactCtas, 64, smem3, st>>>(ra);
    return cudaGetLastError();
}

// ----------------------------------------------------------------- dispatch

// One CTA. Groups 0..E-1 are the routed experts, group E the shared expert.
// Rows of a group are contiguous; a group's rows are cut into tiles of at
// most kTN rows; work item = (group, first row, rows, weight-row tile).
__global__ void __launch_bounds__(1024) prefill_dispatch_kernel(PrefillDispatchArgs a) {
    const int T = a.T, K = a.K, E = a.E, G = E + 1;
    __shared__ int cnt[kMaxGroups], off[kMaxGroups + 1], cur[kMaxGroups], toff[kMaxGroups + 1];
    for (int g = threadIdx.x; g < G; g += blockDim.x) {
        cnt[g] = g == E ? T : 0;
        cur[g] = 0;
    }
    for (int i = threadIdx.x; i < T * (K + 1); i += blockDim.x) a.tok_row[i] = -1;
    __syncthreads();
    if (a.routed)
        for (int i = threadIdx.x; i < T * K; i += blockDim.x) {
            const int e = a.topk_idx[i];
            if (e >= 0 && e < E) atomicAdd(&cnt[e], 1);
        }
    __syncthreads();
    if (threadIdx.x == 0) {
        int o = 0, to = 0;
        for (int g = 0; g < G; ++g) {
            off[g] = o;
            o += cnt[g];
            toff[g] = to;
            to += (cnt[g] + kTN - 1) / kTN;
        }
        off[G] = o;
        toff[G] = to;
        a.counts[0] = o;           // rows
        a.counts[1] = to * a.mt1;  // gate/up items
        a.counts[2] = to * a.mt2;  // down items
    }
    __syncthreads();
    // rows: (token, slot). Routed rows of a group in any order (rows are
    // independent); the shared expert's rows in token order.
    if (a.routed)
        for (int i = threadIdx.x; i < T * K; i += blockDim.x) {
            const int e = a.topk_idx[i];
            if (e < 0 || e >= E) continue;
            const int r = off[e] + atomicAdd(&cur[e], 1);
            const int t = i / K, k = i - t * K;
            a.row_tok[r] = t;
            a.tok_row[t * (K + 1) + k] = r;
        }
    for (int t = threadIdx.x; t < T; t += blockDim.x) {
        const int r = off[E] + t;
        a.row_tok[r] = t;
        a.tok_row[t * (K + 1) + K] = r;
    }
    // items, weight-row tile fastest: item = tile * mt + m-tile
    const int ntiles = toff[G];
    for (int tile = threadIdx.x; tile < ntiles; tile += blockDim.x) {
        int lo = 0, hi = G - 1;  // group with toff[g] <= tile < toff[g + 1]
        while (lo < hi) {
            const int mid = (lo + hi + 1) >> 1;
            if (toff[mid] <= tile) lo = mid;
            else hi = mid - 1;
        }
        const int g = lo;
        const int row0 = off[g] + (tile - toff[g]) * kTN;
        const int nrows = min(kTN, off[g] + cnt[g] - row0);
        for (int mt = 0; mt < a.mt1; ++mt) a.items1[tile * a.mt1 + mt] = make_int4(g, row0, nrows, mt);
        for (int mt = 0; mt < a.mt2; ++mt) a.items2[tile * a.mt2 + mt] = make_int4(g, row0, nrows, mt);
    }
}

// Activation rows (token xn) as bf16 hi + lo, 8 elements per thread.
__global__ void gather_split_kernel(const float* __restrict__ xn, const int* __restrict__ row_tok,
                                    const int* __restrict__ counts, int D, __nv_bfloat16* hi, __nv_bfloat16* lo) {
    const int per_row = D / 8;
    const size_t n = (size_t)counts[0] * per_row;
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
        const int r = (int)(i / per_row), c = (int)(i - (size_t)r * per_row) * 8;
        const float* src = xn + (size_t)row_tok[r] * D + c;
        const float4 v0 = *reinterpret_cast<const float4*>(src), v1 = *reinterpret_cast<const float4*>(src + 4);
        const float v[8] = {v0.x, v0.y, v0.z, v0.w, v1.x, v1.y, v1.z, v1.w};
        __align__(16) __nv_bfloat16 h[8], l[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) split_bf16(v[j], h[j], l[j]);
        *reinterpret_cast<int4*>(hi + (size_t)r * D + c) = *reinterpret_cast<const int4*>(h);
        *reinterpret_cast<int4*>(lo + (size_t)r * D + c) = *reinterpret_cast<const int4*>(l);
    }
}

// ------------------------------------------------------------- grouped GEMM
//
// Work item = (group, weight tile, up to kTN token rows). The weight tile is
// the MMA's A operand (M = 128 rows) and lives in TMEM; the token rows are the
// B operand (shared memory, 128-byte swizzle); the fp32 accumulator is in
// TMEM.
//   mode 0 (gate/up): the tile stacks 64 gate rows over the same 64 up rows,
//           so one accumulator holds both halves of SwiGLU for 64 features.
//   mode 1 (down): 128 rows of the down matrix.
// B holds the token rows' high parts followed by their low parts (n = rows
// rounded up to 32, loaded in 32-row boxes), so per
// K = 16 two MMAs compute the three products of the split:
//   D[:, 0:2n]  = A_hi . [B_hi; B_lo]      (first n columns: hi.hi, next n: hi.lo)
//   D[:, 0:n]  += A_lo . B_hi
// and the epilogue adds the two column halves.
//
// Warp roles (512 threads):
//   warps 0-3   epilogue: TMEM -> registers (thread = tile row), SwiGLU via a
//               shared-memory exchange of the gate and up halves (mode 0) or
//               plain store (mode 1)
//   warp 4      weight producer: TMA of raw int8 tiles (64-byte swizzle) and
//               their fp32 scales [rows][4 groups]
//   warp 5      MMA issuer (one thread) and TMEM owner
//   warp 6      activation producer: TMA of bf16 hi/lo rows (128-byte swizzle)
//   warp 7      idle
//   warps 8-15  dequantisers: raw tile -> A_hi / A_lo in TMEM with
//               tcgen05.st (thread = tile row r, half h of the 64 columns;
//               warp w may only reach TMEM lanes 32 (w % 4) .. + 31)
//
// TMEM columns: accumulator [0, 2 kTN); A stages [256, 512), kASlots x
// (A_hi 32 + A_lo 32 columns).

constexpr int kGemmThreads = 512;
constexpr int kRawSlots = 8, kASlots = 4, kBSlots = 4;
constexpr uint32_t kBBytes = 2 * kTN * 128; // bf16 rows [hi: n][lo: n], 128 bytes each
constexpr uint32_t kRawBytes = kTM * kTK;   // int8 [128][64]
constexpr uint32_t kScBytes = kTM * 16;     // fp32 scales [128][4]: 4 groups (gs 32: a k-slice pair; gs 16: one)
constexpr uint32_t kRawSlotBytes = kRawBytes + 2048;
constexpr uint32_t kTmemA = 256;            // first TMEM column of the A stages
constexpr int kStageLd = 33;                // epilogue exchange row stride (floats)

struct GemmLayout {
    static constexpr uint32_t b = 0;                                   // kBSlots
    static constexpr uint32_t raw = b + kBSlots * kBBytes;             // kRawSlots
    static constexpr uint32_t stage = raw + kRawSlots * kRawSlotBytes; // [2][64][kStageLd] fp32
    static constexpr uint32_t bars = stage + 2 * 64 * kStageLd * 4;
    static constexpr uint32_t total = bars + 512;
};
static_assert(GemmLayout::raw % 1024 == 0 && kRawSlotBytes % 1024 == 0, "tiles stay 1024-byte aligned");
static_assert(GemmLayout::total + 1024 <= 227 * 1024, "shared memory per CTA");
static_assert(kTmemA + kASlots * 64 <= 512 && 2 * kTN <= (int)kTmemA, "TMEM columns");

struct GemmBars {
    uint64_t raw_full[kRawSlots], raw_empty[kRawSlots];
    uint64_t a_full[kASlots], a_empty[kASlots];
    uint64_t b_full[kBSlots], b_empty[kBSlots];
    uint64_t acc_full, acc_empty;
    uint32_t tmem;
    int abort;
};
static_assert(sizeof(GemmBars) <= 512, "barrier block");

struct GemmMaps {
    CUtensorMap w[2];     // routed weights, matrix 0 / 1 ([E * Mtot rows][K] int8)
    CUtensorMap w_sh[2];  // shared expert weights ([Mtot rows][K] int8)
    CUtensorMap s[2];     // routed scales ([E * Mtot rows][K / 32] fp32)
    CUtensorMap s_sh[2];  // shared expert scales
    CUtensorMap bhi, blo; // activations [rows][K] bf16, 16-row boxes
};

__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap* map, int x, int y, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];\n" ::"r"(
            dst),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_addr(bar))
        : "memory");
}

// D (TMEM) (+)= A (TMEM) . B (shared memory descriptor)
__device__ __forceinline__ void tc_mma_ts(uint32_t d, uint32_t a, uint64_t bd, uint32_t idesc, uint32_t acc) {
    asm volatile(
        "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n}\n" ::"r"(
            d),
        "r"(a), "l"(bd), "r"(idesc), "r"(acc)
        : "memory");
}

__device__ __forceinline__ void tc_st16(uint32_t taddr, const uint32_t (&v)[16]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};\n" ::"r"(
            taddr),
        "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]), "r"(v[8]), "r"(v[9]),
        "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15])
        : "memory");
}

__device__ __forceinline__ void st_release_sys(unsigned* p, unsigned v) {
    asm volatile("st.release.sys.global.u32 [%0], %1;\n" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ unsigned ld_acquire_sys(const unsigned* p) {
    unsigned v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];\n" : "=r"(v) : "l"(p) : "memory");
    return v;
}

__device__ __forceinline__ void epi_bar() { asm volatile("bar.sync 1, 128;\n" ::: "memory"); }

// Wait for a phase; on a timeout flag the CTA (and the launch status) and
// return false so that every role leaves its loop.
__device__ __forceinline__ bool role_wait(GemmBars* B, uint64_t* bar, uint32_t parity, unsigned* status) {
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = global_ns();
    while (global_ns() - t0 < kGWaitNs) {
        if (mbar_try_wait_sleep(bar, parity, 20000)) return true;
        if (*reinterpret_cast<volatile int*>(&B->abort)) return false;
    }
    *reinterpret_cast<volatile int*>(&B->abort) = 1;
    atomicOr(status, 64u);
    return false;
}

__device__ __forceinline__ uint64_t f2_pack(float lo, float hi) {
    return (uint64_t)__float_as_uint(lo) | ((uint64_t)__float_as_uint(hi) << 32);
}

// Weights q * s of bytes b0, b1 of u (each byte q + 128) as bf16 pairs
// w_hi + w_lo: q comes out of the byte exactly as (2^23 + byte) - (2^23 + 128),
// w = q * s rounded once as in fp32, w_hi = w with its low 16 bits cleared,
// w_lo = bf16(w - w_hi) (the difference is exact in fp32). Packed f32x2
// arithmetic: two weights per instruction.
__device__ __forceinline__ void dequant_pair(uint32_t u, int b0, int b1, uint64_t s2, uint32_t& hi2, uint32_t& lo2) {
    const uint64_t magic = f2_pack(8388736.0f, 8388736.0f);
    uint64_t q = (uint64_t)__byte_perm(u, 0x4B000000u, 0x7650 | b0) |
                 ((uint64_t)__byte_perm(u, 0x4B000000u, 0x7650 | b1) << 32);
    uint64_t w, l;
    asm("sub.rn.f32x2 %0, %1, %2;" : "=l"(q) : "l"(q), "l"(magic));
    asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(w) : "l"(q), "l"(s2));
    const uint32_t x0 = (uint32_t)w, x1 = (uint32_t)(w >> 32);
    hi2 = __byte_perm(x0, x1, 0x7632);
    const uint64_t h = (uint64_t)(x0 & 0xFFFF0000u) | ((uint64_t)(x1 & 0xFFFF0000u) << 32);
    asm("sub.rn.f32x2 %0, %1, %2;" : "=l"(l) : "l"(w), "l"(h));
    asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(lo2) : "f"(__uint_as_float((uint32_t)(l >> 32))),
        "f"(__uint_as_float((uint32_t)l)));
}

__global__ void __launch_bounds__(kGemmThreads, 1)
    q8_group_gemm_kernel(const __grid_constant__ GemmMaps maps, const __grid_constant__ GroupGemmArgs a) {
    extern __shared__ __align__(1024) unsigned char gsm_raw[];
    unsigned char* sm = gsm_raw + ((1024u - (smem_addr(gsm_raw) & 1023u)) & 1023u);
    GemmBars* B = reinterpret_cast<GemmBars*>(sm + GemmLayout::bars);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int mode = a.mode;
    const int n_items = a.counts[mode == 0 ? 1 : 2];
    const int4* items = mode == 0 ? a.items1 : a.items2;
    const int Kd = a.K, nk = Kd / kTK, E = a.E, Mtot = a.Mtot;
    const int tile_rows = mode == 0 ? kTM / 2 : kTM;  // rows of one weight matrix per tile

    if (tid == 0) {
        for (int i = 0; i < kRawSlots; ++i) {
            mbar_init(&B->raw_full[i], 1);
            mbar_init(&B->raw_empty[i], 8);  // the 8 dequant warps
        }
        for (int i = 0; i < kASlots; ++i) {
            mbar_init(&B->a_full[i], 8);
            mbar_init(&B->a_empty[i], 1);    // tcgen05.commit
        }
        for (int i = 0; i < kBSlots; ++i) {
            mbar_init(&B->b_full[i], 1);
            mbar_init(&B->b_empty[i], 1);
        }
        mbar_init(&B->acc_full, 1);
        mbar_init(&B->acc_empty, 4);  // the 4 epilogue warps
        B->abort = 0;
        mbar_init_fence();
    }
    if (warp == 5) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], 512;\n" ::"r"(smem_addr(&B->tmem))
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;\n" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = B->tmem;

    if (warp == 4) {
        // ---- weight producer
        if (lane == 0) {
            uint32_t rs = 0;
            for (int item = blockIdx.x; item < n_items; item += gridDim.x) {
                const int4 it = items[item];
                const bool sh = it.x == E;
                const int wrow = (sh ? 0 : it.x * Mtot) + it.w * tile_rows;
                for (int ks = 0; ks < nk; ++ks, ++rs) {
                    const int slot = rs % kRawSlots;
                    if (!role_wait(B, &B->raw_empty[slot], ((rs / kRawSlots) & 1) ^ 1, a.status)) goto done;
                    mbar_arrive_expect_tx(&B->raw_full[slot], kRawBytes + kScBytes);
                    const uint32_t dst = smem_addr(sm + GemmLayout::raw + slot * kRawSlotBytes);
                    // scales: a 16-byte box of 4 groups: gs = 32 -> groups 4 * (ks / 2) .. + 3 (both k-slices
                    // of the pair); gs = 16 -> groups 4 * ks .. + 3 (this k-slice)
                    const int sx = a.gs == 16 ? 4 * ks : 4 * (ks >> 1);
                    if (mode == 0) {
                        tma_load_2d(dst, sh ? &maps.w_sh[0] : &maps.w[0], ks * kTK, wrow, &B->raw_full[slot]);
                        tma_load_2d(dst + 64 * kTK, sh ? &maps.w_sh[1] : &maps.w[1], ks * kTK, wrow,
                                    &B->raw_full[slot]);
                        tma_load_2d(dst + kRawBytes, sh ? &maps.s_sh[0] : &maps.s[0], sx, wrow, &B->raw_full[slot]);
                        tma_load_2d(dst + kRawBytes + 64 * 16, sh ? &maps.s_sh[1] : &maps.s[1], sx, wrow,
                                    &B->raw_full[slot]);
                    } else {
                        tma_load_2d(dst, sh ? &maps.w_sh[0] : &maps.w[0], ks * kTK, wrow, &B->raw_full[slot]);
                        tma_load_2d(dst + kRawBytes, sh ? &maps.s_sh[0] : &maps.s[0], sx, wrow, &B->raw_full[slot]);
                    }
                }
            }
        }
    } else if (warp == 6) {
        // ---- activation producer: rows [row0, row0 + n) high parts, then low parts
        if (lane == 0) {
            uint32_t bs = 0;
            for (int item = blockIdx.x; item < n_items; item += gridDim.x) {
                const int4 it = items[item];
                const int n_eff = (it.z + 31) & ~31, nb = n_eff >> 5;
                for (int ks = 0; ks < nk; ++ks, ++bs) {
                    const int slot = bs % kBSlots;
                    if (!role_wait(B, &B->b_empty[slot], ((bs / kBSlots) & 1) ^ 1, a.status)) goto done;
                    mbar_arrive_expect_tx(&B->b_full[slot], (uint32_t)n_eff * 128 * 2);
                    const uint32_t dst = smem_addr(sm + GemmLayout::b + slot * kBBytes);
                    for (int j = 0; j < nb; ++j) {
                        tma_load_2d(dst + j * 4096, &maps.bhi, ks * kTK, it.y + 32 * j, &B->b_full[slot]);
                        tma_load_2d(dst + n_eff * 128 + j * 4096, &maps.blo, ks * kTK, it.y + 32 * j,
                                    &B->b_full[slot]);
                    }
                }
            }
        }
    } else if (warp == 5) {
        // ---- MMA issuer
        if (lane == 0) {
            uint32_t as = 0, bs = 0, ac = 0;
            for (int item = blockIdx.x; item < n_items; item += gridDim.x, ++ac) {
                const int4 it = items[item];
                const uint32_t n_eff = (uint32_t)((it.z + 31) & ~31);
                const uint32_t id_base = (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(kTM >> 4) << 24);
                const uint32_t id_cat = id_base | ((2 * n_eff >> 3) << 17), id_hi = id_base | ((n_eff >> 3) << 17);
                if (!role_wait(B, &B->acc_empty, (ac & 1) ^ 1, a.status)) goto done;
                tc_fence_after();
                for (int ks = 0; ks < nk; ++ks, ++bs, ++as) {
                    const int bslot = bs % kBSlots, aslot = as % kASlots;
                    if (!role_wait(B, &B->b_full[bslot], (bs / kBSlots) & 1, a.status)) goto done;
                    if (!role_wait(B, &B->a_full[aslot], (as / kASlots) & 1, a.status)) goto done;
                    tc_fence_after();
                    const uint32_t bAddr = smem_addr(sm + GemmLayout::b + bslot * kBBytes);
                    const uint32_t aHi = tmem + kTmemA + aslot * 64, aLo = aHi + 32;
#pragma unroll
                    for (int kk = 0; kk < kTK / 16; ++kk) {
                        const uint64_t bd = umma_desc(bAddr + kk * 32);
                        tc_mma_ts(tmem, aHi + kk * 8, bd, id_cat, (ks | kk) ? 1u : 0u);
                        tc_mma_ts(tmem, aLo + kk * 8, bd, id_hi, 1u);
                    }
                    tc_commit(&B->a_empty[aslot]);
                    tc_commit(&B->b_empty[bslot]);
                }
                tc_commit(&B->acc_full);
            }
        }
    } else if (warp >= 8) {
        // ---- dequantisers
        const int quarter = warp & 3, h = (warp - 8) >> 2, r = quarter * 32 + lane;
        const uint32_t lane_base = (uint32_t)(quarter * 32) << 16;
        const int swz = (r >> 1) & 3;  // 64-byte swizzle of the raw tile: chunk c of row r at c ^ swz
        uint32_t rs = 0;
        for (int item = blockIdx.x; item < n_items; item += gridDim.x)
            for (int ks = 0; ks < nk; ++ks, ++rs) {
                const int rslot = rs % kRawSlots, aslot = rs % kASlots;
                if (!role_wait(B, &B->raw_full[rslot], (rs / kRawSlots) & 1, a.status)) goto done;
                const unsigned char* slotp = sm + GemmLayout::raw + rslot * kRawSlotBytes;
                const unsigned char* rowp = slotp + r * kTK;
                const int4 v0 = *reinterpret_cast<const int4*>(rowp + 16 * ((2 * h) ^ swz));
                const int4 v1 = *reinterpret_cast<const int4*>(rowp + 16 * ((2 * h + 1) ^ swz));
                // columns 32h .. 32h + 31 of the k-slice: one group (gs = 32) or two (gs = 16)
                const float* sct = reinterpret_cast<const float*>(slotp + kRawBytes) + r * 4;
                const float sa = a.gs == 16 ? sct[2 * h] : sct[2 * (ks & 1) + h];
                const float sb = a.gs == 16 ? sct[2 * h + 1] : sa;
                __syncwarp();
                if (lane == 0) mbar_arrive(&B->raw_empty[rslot]);
                const uint64_t s2a = f2_pack(sa, sa), s2b = f2_pack(sb, sb);
                uint32_t hv[16], lv[16];
                const uint32_t qw[8] = {(uint32_t)v0.x, (uint32_t)v0.y, (uint32_t)v0.z, (uint32_t)v0.w,
                                        (uint32_t)v1.x, (uint32_t)v1.y, (uint32_t)v1.z, (uint32_t)v1.w};
#pragma unroll
                for (int j = 0; j < 8; ++j) {
                    const uint32_t u = qw[j] ^ 0x80808080u;  // bytes q + 128
                    const uint64_t s2 = j < 4 ? s2a : s2b;   // words 0-3: columns 0-15, 4-7: 16-31
                    dequant_pair(u, 0, 1, s2, hv[2 * j], lv[2 * j]);
                    dequant_pair(u, 2, 3, s2, hv[2 * j + 1], lv[2 * j + 1]);
                }
                if (!role_wait(B, &B->a_empty[aslot], ((rs / kASlots) & 1) ^ 1, a.status)) goto done;
                const uint32_t ta = tmem + lane_base + kTmemA + aslot * 64 + h * 16;
                tc_st16(ta, hv);
                tc_st16(ta + 32, lv);
                asm volatile("tcgen05.wait::st.sync.aligned;\n" ::: "memory");
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(&B->a_full[aslot]);
            }
    } else if (warp < 4) {
        // ---- epilogue: thread = tile row (warp * 32 + lane)
        float* stage = reinterpret_cast<float*>(sm + GemmLayout::stage);  // [2][64][kStageLd]
        const int row = warp * 32 + lane;
        uint32_t ac = 0;
        for (int item = blockIdx.x; item < n_items; item += gridDim.x, ++ac) {
            const int4 it = items[item];
            const int row0 = it.y, nrows = it.z, n_eff = (nrows + 31) & ~31;
            if (!role_wait(B, &B->acc_full, ac & 1, a.status)) goto done;
            tc_fence_after();
            const uint32_t tb = tmem + ((uint32_t)(warp * 32) << 16);
            for (int n0 = 0; n0 < nrows; n0 += 32) {
                float v[32], w2[32];
                tc_ld32(tb + n0, v);        // hi.hi + lo.hi
                tc_ld32(tb + n_eff + n0, w2);  // hi.lo (columns past 2 n_eff are never used)
#pragma unroll
                for (int j = 0; j < 32; ++j) v[j] += w2[j];
                if (n0 + 32 >= nrows) {  // accumulator read out: let the next item's MMAs start
                    tc_fence_before();
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&B->acc_empty);
                }
                if (mode == 0) {
                    // rows 0-63 gate, 64-127 up (same 64 features): exchange through shared memory
                    float* st = stage + (row >> 6) * 64 * kStageLd + (row & 63) * kStageLd;
#pragma unroll
                    for (int j = 0; j < 32; ++j) st[j] = v[j];
                    epi_bar();
                    const int f = tid & 63, j0 = (tid >> 6) * 16;
                    const int col = it.w * 64 + f;
                    const float* gs = stage + f * kStageLd;
                    const float* us = stage + 64 * kStageLd + f * kStageLd;
#pragma unroll
                    for (int j = j0; j < j0 + 16; ++j) {
                        if (n0 + j >= nrows) break;
                        const float g = gs[j];
                        const float hval = __fdividef(g, 1.0f + __expf(-g)) * us[j];  // infer.c:1184-1188, 1197-1201
                        __nv_bfloat16 hh, hl;
                        split_bf16(hval, hh, hl);
                        const size_t o = (size_t)(row0 + n0 + j) * Mtot + col;
                        static_cast<__nv_bfloat16*>(a.hhi)[o] = hh;
                        static_cast<__nv_bfloat16*>(a.hlo)[o] = hl;
                    }
                    epi_bar();  // stage is rewritten by the next chunk
                } else if (a.row_src) {
                    // expert parallelism: lane l finds where token row n0 + l goes (the
                    // sender's back_rows over NVLink, or y for this rank's own tokens)
                    const int col = it.w * kTM + row;
                    float* dst_l = nullptr;
                    if (n0 + lane < nrows) {
                        const int r = row0 + n0 + lane, src = a.row_src[r];
                        if (src < a.n_slots) {
                            const int q = src / a.cap, jj = src - q * a.cap;
                            dst_l = reinterpret_cast<float*>(a.peer[q] + a.back_off) +
                                    ((size_t)a.me * a.cap + jj) * Mtot;
                        } else {
                            dst_l = a.y + (size_t)r * Mtot;
                        }
                    }
#pragma unroll
                    for (int j = 0; j < 32; ++j) {
                        if (n0 + j >= nrows) break;
                        float* d = reinterpret_cast<float*>(
                            __shfl_sync(0xffffffffu, reinterpret_cast<unsigned long long>(dst_l), j));
                        d[col] = v[j];
                    }
                } else {
                    const int col = it.w * kTM + row;
#pragma unroll
                    for (int j = 0; j < 32; ++j) {
                        if (n0 + j >= nrows) break;
                        a.y[(size_t)(row0 + n0 + j) * Mtot + col] = v[j];
                    }
                }
            }
        }
    }
done:
    if (a.row_src) __threadfence_system();  // this thread's stores into the other ranks' regions
    __syncthreads();
    if (warp == 5) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, 512;\n" ::"r"(tmem) : "memory");
    }
    if (a.row_src && tid == 0 && atomicAdd(a.done, 1u) == gridDim.x - 1) {
        // every CTA's outputs are out: raise flag_back[me] in every region, unless
        // a CTA gave up (its rows would be missing; the senders then time out)
        __threadfence_system();
        if (!(*reinterpret_cast<volatile unsigned*>(a.status) & 64u))
            for (int q = 0; q < a.n_shards; ++q)
                st_release_sys(reinterpret_cast<unsigned*>(a.peer[q] + a.flag_off) + a.me, a.epoch);
        *reinterpret_cast<volatile unsigned*>(a.done) = 0u;
    }
}

// ------------------------------------------------------------------ combine

// x[t] += y_shared + sum_k (1.8 w_k) y_k in rank order (infer.c:1175,1192,
// 1212-1214), 4 elements per thread.
__global__ void prefill_combine_kernel(float* x, const float* __restrict__ Y, const int* __restrict__ tok_row,
                                       const float* __restrict__ topk_w, int T, int D, int K, int routed) {
    const int per_tok = D / 4;
    const size_t n = (size_t)T * per_tok;
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
        const int t = (int)(i / per_tok), c = (int)(i - (size_t)t * per_tok) * 4;
        const int* tr = tok_row + (size_t)t * (K + 1);
        float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
        if (routed)
            for (int k = 0; k < K; ++k) {
                const int r = tr[k];
                if (r < 0) continue;
                const float wk = __fmul_rn(topk_w[(size_t)t * K + k], 1.8f);
                const float4 y = *reinterpret_cast<const float4*>(Y + (size_t)r * D + c);
                acc.x = __fadd_rn(acc.x, __fmul_rn(wk, y.x));
                acc.y = __fadd_rn(acc.y, __fmul_rn(wk, y.y));
                acc.z = __fadd_rn(acc.z, __fmul_rn(wk, y.z));
                acc.w = __fadd_rn(acc.w, __fmul_rn(wk, y.w));
            }
        const float4 ys = *reinterpret_cast<const float4*>(Y + (size_t)tr[K] * D + c);
        float4* xp = reinterpret_cast<float4*>(x + (size_t)t * D + c);
        float4 xv = *xp;
        xv.x = __fadd_rn(xv.x, __fadd_rn(ys.x, acc.x));
        xv.y = __fadd_rn(xv.y, __fadd_rn(ys.y, acc.y));
        xv.z = __fadd_rn(xv.z, __fadd_rn(ys.z, acc.z));
        xv.w = __fadd_rn(xv.w, __fadd_rn(ys.w, acc.w));
        *xp = xv;
    }
}

// ------------------------------------------------------- expert parallelism
//
// Experts are sharded over n_shards ranks, e_local consecutive experts each;
// every rank routes its own tokens, sends each (token, slot) pair's xn row
// to the rank that holds its expert, runs its experts on what it received
// (plus the replicated shared expert on its own tokens), and gets the expert
// outputs back in the order it sent them.

constexpr int kMaxShards = kEpMaxShards;

// Send layout: pairs (t, k) in (token, slot) order within each destination,
// destinations in rank order. One CTA; thread i owns a contiguous chunk of
// the T*K pairs. send_pos[t*K + k] = row in the send buffer (-1: not sent).
__global__ void __launch_bounds__(1024) ep_pack_kernel(const int32_t* __restrict__ ids, int T, int K, int e_local,
                                                     int n_shards, int routed, int* send_pos, int* send_counts,
                                                     int32_t* send_expert) {
    __shared__ int pre[kMaxShards][1024];
    __shared__ int base[kMaxShards + 1];
    const int n = T * K, tid = threadIdx.x, nt = blockDim.x;
    const int chunk = (n + nt - 1) / nt, lo = min(n, tid * chunk), hi = min(n, lo + chunk);
    int c[kMaxShards];
#pragma unroll
    for (int d = 0; d < kMaxShards; ++d) c[d] = 0;
    for (int i = lo; i < hi; ++i) {
        const int e = ids[i];
        if (!routed || e < 0) continue;
        const int d = e / e_local;
#pragma unroll
        for (int q = 0; q < kMaxShards; ++q) c[q] += q == d;
    }
#pragma unroll
    for (int d = 0; d < kMaxShards; ++d) pre[d][tid] = c[d];
    __syncthreads();
    // inclusive scans over threads, one destination per pass (Hillis-Steele)
    for (int off = 1; off < nt; off <<= 1) {
        int v[kMaxShards];
#pragma unroll
        for (int d = 0; d < kMaxShards; ++d) v[d] = tid >= off ? pre[d][tid - off] : 0;
        __syncthreads();
#pragma unroll
        for (int d = 0; d < kMaxShards; ++d) pre[d][tid] += v[d];
        __syncthreads();
    }
    if (tid == 0) {
        int o = 0;
        for (int d = 0; d < n_shards; ++d) {
            base[d] = o;
            send_counts[d] = pre[d][nt - 1];
            o += pre[d][nt - 1];
        }
        base[n_shards] = o;
    }
    __syncthreads();
    int run[kMaxShards];
#pragma unroll
    for (int d = 0; d < kMaxShards; ++d) run[d] = 0;
    for (int i = lo; i < hi; ++i) {
        const int e = ids[i];
        if (!routed || e < 0) {
            send_pos[i] = -1;
            continue;
        }
        const int d = e / e_local;
        int r = 0;
#pragma unroll
        for (int q = 0; q < kMaxShards; ++q)
            if (q == d) r = run[q]++;
        const int pos = base[d] + pre[d][tid] - c[d] + r;
        send_pos[i] = pos;
        send_expert[pos] = e - d * e_local;
    }
}

// send_rows[send_pos[t*K + k]] = xn[t] (one warp per pair).
__global__ void ep_pack_rows_kernel(const float* __restrict__ xn, const int* __restrict__ send_pos, int T, int K, int D,
                                    float* send_rows) {
    const int warps = (gridDim.x * blockDim.x) >> 5, lane = threadIdx.x & 31;
    for (int i = (blockIdx.x * blockDim.x + threadIdx.x) >> 5; i < T * K; i += warps) {
        const int pos = send_pos[i];
        if (pos < 0) continue;
        const float4* src = reinterpret_cast<const float4*>(xn + (size_t)(i / K) * D);
        float4* dst = reinterpret_cast<float4*>(send_rows + (size_t)pos * D);
        for (int c = lane; c < D / 4; c += 32) dst[c] = src[c];
    }
}

// Rows of the local expert GEMMs: received rows grouped by local expert
// (groups 0 .. e_local - 1), then this rank's own tokens for the shared
// expert (group e_local). Sources: s < n_recv -> received slot s, else own
// token s - n_recv. row_src[row] = source; pos_of_src[source] = row.
// Received slots are [0, n_recv) when recv_cnt is null (the all-to-all
// layout), else the first recv_cnt[q] of each sender q's cap slots
// [q * cap, q * cap + cap) (the peer-region layout; n_recv = n_src * cap).
__global__ void __launch_bounds__(1024) ep_group_kernel(const int32_t* __restrict__ recv_expert, int n_recv, int T,
                                                      int e_local, int routed, int mt1, int mt2, int* counts,
                                                      int* row_src, int* pos_of_src, int4* items1, int4* items2,
                                                      const int* recv_cnt, int n_src, int cap) {
    const int G = e_local + 1;
    __shared__ int cnt[kMaxGroups], off[kMaxGroups + 1], cur[kMaxGroups], toff[kMaxGroups + 1];
    __shared__ int soff[kMaxShards + 1];
    const int nseg = recv_cnt ? n_src : 1;
    if (threadIdx.x == 0) {
        int o = 0;
        for (int q = 0; q < nseg; ++q) {
            soff[q] = o;
            o += recv_cnt ? min(max(__ldcg(recv_cnt + q), 0), cap) : n_recv;
        }
        soff[nseg] = o;
    }
    for (int g = threadIdx.x; g < G; g += blockDim.x) {
        cnt[g] = g == e_local ? T : 0;
        cur[g] = 0;
    }
    __syncthreads();
    const int n_rows = soff[nseg];
    auto slot_of = [&](int m) {
        if (!recv_cnt) return m;
        int q = 0;
        while (m >= soff[q + 1]) ++q;
        return q * cap + (m - soff[q]);
    };
    if (routed)
        for (int m = threadIdx.x; m < n_rows; m += blockDim.x) {
            const int e = recv_expert[slot_of(m)];
            if (e >= 0 && e < e_local) atomicAdd(&cnt[e], 1);
        }
    __syncthreads();
    if (threadIdx.x == 0) {
        int o = 0, to = 0;
        for (int g = 0; g < G; ++g) {
            off[g] = o;
            o += cnt[g];
            toff[g] = to;
            to += (cnt[g] + kTN - 1) / kTN;
        }
        off[G] = o;
        toff[G] = to;
        counts[0] = o;
        counts[1] = to * mt1;
        counts[2] = to * mt2;
    }
    __syncthreads();
    for (int m = threadIdx.x; m < n_rows; m += blockDim.x) {
        const int i = slot_of(m);
        const int e = recv_expert[i];
        if (!routed || e < 0 || e >= e_local) {
            pos_of_src[i] = -1;
            continue;
        }
        const int r = off[e] + atomicAdd(&cur[e], 1);
        row_src[r] = i;
        pos_of_src[i] = r;
    }
    for (int t = threadIdx.x; t < T; t += blockDim.x) {
        const int r = off[e_local] + t;
        row_src[r] = n_recv + t;
        pos_of_src[n_recv + t] = r;
    }
    const int ntiles = toff[G];
    for (int tile = threadIdx.x; tile < ntiles; tile += blockDim.x) {
        int lo = 0, hi = G - 1;
        while (lo < hi) {
            const int mid = (lo + hi + 1) >> 1;
            if (toff[mid] <= tile) lo = mid;
            else hi = mid - 1;
        }
        const int g = lo;
        const int row0 = off[g] + (tile - toff[g]) * kTN;
        const int nrows = min(kTN, off[g] + cnt[g] - row0);
        for (int mt = 0; mt < mt1; ++mt) items1[tile * mt1 + mt] = make_int4(g, row0, nrows, mt);
        for (int mt = 0; mt < mt2; ++mt) items2[tile * mt2 + mt] = make_int4(g, row0, nrows, mt);
    }
}

// Activation rows of the local GEMMs as bf16 hi + lo, 8 elements per thread.
__global__ void ep_gather_split_kernel(const float* __restrict__ recv_rows, const float* __restrict__ xn,
                                       const int* __restrict__ row_src, const int* __restrict__ counts, int n_recv,
                                       int D, __nv_bfloat16* hi, __nv_bfloat16* lo) {
    const int per_row = D / 8;
    const size_t n = (size_t)counts[0] * per_row;
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
        const int r = (int)(i / per_row), c = (int)(i - (size_t)r * per_row) * 8;
        const int sidx = row_src[r];
        const float* src = (sidx < n_recv ? recv_rows + (size_t)sidx * D : xn + (size_t)(sidx - n_recv) * D) + c;
        const float4 v0 = *reinterpret_cast<const float4*>(src), v1 = *reinterpret_cast<const float4*>(src + 4);
        const float v[8] = {v0.x, v0.y, v0.z, v0.w, v1.x, v1.y, v1.z, v1.w};
        __align__(16) __nv_bfloat16 h[8], l[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) split_bf16(v[j], h[j], l[j]);
        *reinterpret_cast<int4*>(hi + (size_t)r * D + c) = *reinterpret_cast<const int4*>(h);
        *reinterpret_cast<int4*>(lo + (size_t)r * D + c) = *reinterpret_cast<const int4*>(l);
    }
}

// out_rows[i] = Y[pos_of_src[i]] for the received rows (one warp per row).
__global__ void ep_scatter_kernel(const float* __restrict__ Y, const int* __restrict__ pos_of_src, int n_recv, int D,
                                  float* out_rows) {
    const int warps = (gridDim.x * blockDim.x) >> 5, lane = threadIdx.x & 31;
    for (int i = (blockIdx.x * blockDim.x + threadIdx.x) >> 5; i < n_recv; i += warps) {
        const int r = pos_of_src[i];
        float4* dst = reinterpret_cast<float4*>(out_rows + (size_t)i * D);
        if (r < 0) {
            for (int c = lane; c < D / 4; c += 32) dst[c] = make_float4(0.f, 0.f, 0.f, 0.f);
            continue;
        }
        const float4* src = reinterpret_cast<const float4*>(Y + (size_t)r * D);
        for (int c = lane; c < D / 4; c += 32) dst[c] = src[c];
    }
}

// x[t] += y_shared[t] + sum_k (1.8 w_k) y_k in rank order (infer.c:1175,1192,
// 1212-1214); y_k = back_rows[send_pos[t*K + k]] came back from the expert's
// rank, y_shared = Y[pos_of_src[n_recv + t]].
__global__ void ep_combine_kernel(float* x, const float* __restrict__ Y, const int* __restrict__ pos_of_src,
                                  const float* __restrict__ back_rows, const int* __restrict__ send_pos,
                                  const float* __restrict__ topk_w, int T, int D, int K, int n_recv) {
    const int per_tok = D / 4;
    const size_t n = (size_t)T * per_tok;
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
        const int t = (int)(i / per_tok), c = (int)(i - (size_t)t * per_tok) * 4;
        float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
        for (int k = 0; k < K; ++k) {
            const int pos = send_pos[t * K + k];
            if (pos < 0) continue;
            const float wk = __fmul_rn(topk_w[(size_t)t * K + k], 1.8f);
            const float4 y = *reinterpret_cast<const float4*>(back_rows + (size_t)pos * D + c);
            acc.x = __fadd_rn(acc.x, __fmul_rn(wk, y.x));
            acc.y = __fadd_rn(acc.y, __fmul_rn(wk, y.y));
            acc.z = __fadd_rn(acc.z, __fmul_rn(wk, y.z));
            acc.w = __fadd_rn(acc.w, __fmul_rn(wk, y.w));
        }
        const float4 ys = *reinterpret_cast<const float4*>(Y + (size_t)pos_of_src[n_recv + t] * D + c);
        float4* xp = reinterpret_cast<float4*>(x + (size_t)t * D + c);
        float4 xv = *xp;
        xv.x = __fadd_rn(xv.x, __fadd_rn(ys.x, acc.x));
        xv.y = __fadd_rn(xv.y, __fadd_rn(ys.y, acc.y));
        xv.z = __fadd_rn(xv.z, __fadd_rn(ys.z, acc.z));
        xv.w = __fadd_rn(xv.w, __fadd_rn(ys.w, acc.w));
        *xp = xv;
    }
}

// ------------------------------------------------------------ tensor maps

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    if (!fn) {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    }
    return fn;
}

// 2-D map over a row-major [rows][cols] matrix, box [box_rows][box_cols].
bool make_map(CUtensorMap* m, const void* base, CUtensorMapDataType type, int elem, uint64_t rows, uint64_t cols,
              uint32_t box_rows, uint32_t box_cols, CUtensorMapSwizzle swz) {
    auto fn = encode_fn();
    if (!fn || !base) return false;
    const cuuint64_t dims[2] = {cols, rows};
    const cuuint64_t strides[1] = {cols * (uint64_t)elem};
    const cuuint32_t box[2] = {box_cols, box_rows};
    const cuuint32_t estr[2] = {1, 1};
    return fn(m, type, 2, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, swz,
              CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

}  // namespace

cudaError_t prefill_check(const MoeDims& d) {
    if ((d.gs != 32 && d.gs != 16) || d.D % kTM || d.F % kTM || d.E < 1 || d.E + 1 > kMaxGroups || d.K < 1 || d.K > kMaxTopK ||
        d.K > d.E || d.D > 8192 || d.F > 16384)
        return cudaErrorInvalidValue;
    return cudaSuccess;
}

namespace {

struct PrefillWs {
    float* xn;
    double *cen, *bnd;  // router logit centre / bound [T][E]
    int32_t* ids;
    float* wts;
    int* row_tok;
    int* tok_row;
    int* counts;
    int4* items1;
    int4* items2;
    __nv_bfloat16 *xhi, *xlo, *hhi, *hlo;
    float* y;
    size_t bytes;
};

PrefillWs carve(unsigned char* base, const MoeDims& d, int T) {
    const size_t R = (size_t)T * (d.K + 1), tiles = R / kTN + d.E + 1;
    PrefillWs w{};
    size_t b = 0;
    auto take = [&](size_t n) {
        unsigned char* r = base ? base + b : nullptr;
        b += (n + 255) & ~(size_t)255;
        return r;
    };
    w.xn = reinterpret_cast<float*>(take((size_t)T * d.D * 4));
    w.cen = reinterpret_cast<double*>(take((size_t)T * d.E * 8));
    w.bnd = reinterpret_cast<double*>(take((size_t)T * d.E * 8));
    w.ids = reinterpret_cast<int32_t*>(take((size_t)T * d.K * 4));
    w.wts = reinterpret_cast<float*>(take((size_t)T * d.K * 4));
    w.row_tok = reinterpret_cast<int*>(take(R * 4));
    w.tok_row = reinterpret_cast<int*>(take(R * 4));
    w.counts = reinterpret_cast<int*>(take(16));
    w.items1 = reinterpret_cast<int4*>(take(tiles * (d.F / (kTM / 2)) * 16));
    w.items2 = reinterpret_cast<int4*>(take(tiles * (d.D / kTM) * 16));
    w.xhi = reinterpret_cast<__nv_bfloat16*>(take(R * d.D * 2));
    w.xlo = reinterpret_cast<__nv_bfloat16*>(take(R * d.D * 2));
    w.hhi = reinterpret_cast<__nv_bfloat16*>(take(R * d.F * 2));
    w.hlo = reinterpret_cast<__nv_bfloat16*>(take(R * d.F * 2));
    w.y = reinterpret_cast<float*>(take(R * d.D * 4));
    w.bytes = b;
    return w;
}

}  // namespace

size_t prefill_workspace_bytes(const MoeDims& d, int T) { return carve(nullptr, d, T).bytes; }

namespace {

cudaError_t launch_route(const PrefillRouteArgs& ra, int num_sms, cudaStream_t st) {
    return launch_route_batched(ra, num_sms, st);
}

// Gate/up + SwiGLU and down for grouped rows already split into xhi / xlo
// ([rows][D], rows <= R_cap): groups 0 .. d.E - 1 use the routed weights of
// `w` (d.E experts), group d.E the shared expert. Y = [rows][D].
cudaError_t launch_grouped_ffn(const MoeLayerDev& w, const MoeDims& d, bool use_routed, size_t R_cap,
                               const __nv_bfloat16* xhi, const __nv_bfloat16* xlo, __nv_bfloat16* hhi,
                               __nv_bfloat16* hlo, float* y, const int* counts, const int4* items1,
                               const int4* items2, int num_sms, unsigned* status, cudaStream_t st,
                               const GroupGemmArgs* peer_out = nullptr) {
    // tensor maps: weights (box rows x 64 bytes, 64-byte swizzle), their scales (box rows x 4 groups) and
    // activations (box 32 rows x 64 bf16, 128-byte swizzle)
    GemmMaps m1{}, m2{};
    const uint64_t er = (uint64_t)d.E;
    bool ok = true;
    // gate/up tiles stack 64 + 64 rows, down tiles 128 rows
    auto wmap = [&](CUtensorMap* mp, const int8_t* q, uint64_t rows, int cols, uint32_t box_rows,
                    const CUtensorMap* alt) {
        if (q) ok = ok && make_map(mp, q, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, rows, cols, box_rows, kTK,
                                   CU_TENSOR_MAP_SWIZZLE_64B);
        else if (alt) *mp = *alt;  // never read: no routed items
    };
    auto smap = [&](CUtensorMap* mp, const float* sc, uint64_t rows, int cols, uint32_t box_rows,
                    const CUtensorMap* alt) {
        if (sc) ok = ok && make_map(mp, sc, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, rows, cols / d.gs, box_rows, 4,
                                    CU_TENSOR_MAP_SWIZZLE_NONE);
        else if (alt) *mp = *alt;
    };
    const uint32_t r1 = kTM / 2, r2 = kTM;
    wmap(&m1.w_sh[0], w.gate_sh_q, d.F, d.D, r1, nullptr);
    wmap(&m1.w_sh[1], w.up_sh_q, d.F, d.D, r1, nullptr);
    wmap(&m1.w[0], use_routed ? w.gate_q : nullptr, er * d.F, d.D, r1, &m1.w_sh[0]);
    wmap(&m1.w[1], use_routed ? w.up_q : nullptr, er * d.F, d.D, r1, &m1.w_sh[1]);
    smap(&m1.s_sh[0], w.gate_sh_s, d.F, d.D, r1, nullptr);
    smap(&m1.s_sh[1], w.up_sh_s, d.F, d.D, r1, nullptr);
    smap(&m1.s[0], use_routed ? w.gate_s : nullptr, er * d.F, d.D, r1, &m1.s_sh[0]);
    smap(&m1.s[1], use_routed ? w.up_s : nullptr, er * d.F, d.D, r1, &m1.s_sh[1]);
    wmap(&m2.w_sh[0], w.down_sh_q, d.D, d.F, r2, nullptr);
    wmap(&m2.w[0], use_routed ? w.down_q : nullptr, er * d.D, d.F, r2, &m2.w_sh[0]);
    smap(&m2.s_sh[0], w.down_sh_s, d.D, d.F, r2, nullptr);
    smap(&m2.s[0], use_routed ? w.down_s : nullptr, er * d.D, d.F, r2, &m2.s_sh[0]);
    m2.w_sh[1] = m2.w_sh[0];
    m2.w[1] = m2.w[0];
    m2.s_sh[1] = m2.s_sh[0];
    m2.s[1] = m2.s[0];
    const auto bf = CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
    const auto sw = CU_TENSOR_MAP_SWIZZLE_128B;
    ok = ok && make_map(&m1.bhi, xhi, bf, 2, R_cap, d.D, 32, kTK, sw) && make_map(&m1.blo, xlo, bf, 2, R_cap, d.D, 32, kTK, sw);
    ok = ok && make_map(&m2.bhi, hhi, bf, 2, R_cap, d.F, 32, kTK, sw) && make_map(&m2.blo, hlo, bf, 2, R_cap, d.F, 32, kTK, sw);
    if (!ok) return cudaErrorInvalidValue;
    const int gsmem = (int)GemmLayout::total + 1024;
    cudaError_t err = ensure_smem_attr(reinterpret_cast<const void*>(q8_group_gemm_kernel), gsmem);
    if (err) return err;
    GroupGemmArgs g1{items1, items2, counts, hhi, hlo, nullptr, status, d.D, d.F, d.E, 0, d.gs};
    q8_group_gemm_kernel<<<num_sms, kGemmThreads, gsmem, st>>>(m1, g1);
    GroupGemmArgs g2{items1, items2, counts, nullptr, nullptr, y, status, d.F, d.D, d.E, 1, d.gs};
    if (peer_out) {
        g2.row_src = peer_out->row_src;
        for (int q = 0; q < kEpMaxShards; ++q) g2.peer[q] = peer_out->peer[q];
        g2.back_off = peer_out->back_off;
        g2.flag_off = peer_out->flag_off;
        g2.n_slots = peer_out->n_slots;
        g2.cap = peer_out->cap;
        g2.me = peer_out->me;
        g2.n_shards = peer_out->n_shards;
        g2.done = peer_out->done;
        g2.epoch = peer_out->epoch;
    }
    q8_group_gemm_kernel<<<num_sms, kGemmThreads, gsmem, st>>>(m2, g2);
    return cudaGetLastError();
}

}  // namespace

cudaError_t launch_moe_prefill(const MoeLayerDev& w, const MoeDims& d, unsigned char* ws, float* x, int T,
                               int32_t* topk_idx, float* topk_w, int routed, int num_sms, unsigned* status,
                               unsigned long long* stats, cudaStream_t st) {
    cudaError_t err = prefill_check(d);
    if (err != cudaSuccess) return err;
    if (T <= 0) return cudaErrorInvalidValue;
    const bool use_routed = routed && w.gate_q && w.up_q && w.down_q;
    const size_t R = (size_t)T * (d.K + 1);
    const int mt1 = d.F / (kTM / 2), mt2 = d.D / kTM;  // gate/up tiles: 64 features
    const PrefillWs p = carve(ws, d, T);
    // 1 routing
    PrefillRouteArgs ra{x, w.ffn_norm, w.router, w.router_bias, p.xn, p.ids, p.wts, stats, T, d.D, d.E, d.K,
                        p.cen, p.bnd};
    if ((err = launch_route(ra, num_sms, st))) return err;
    // 2 dispatch
    PrefillDispatchArgs da{p.ids, T, d.K, d.E, use_routed ? 1 : 0, mt1, mt2, p.counts, p.row_tok, p.tok_row,
                           p.items1, p.items2};
    prefill_dispatch_kernel<<<1, 1024, 0, st>>>(da);
    // 3 activations
    gather_split_kernel<<<num_sms * 4, 256, 0, st>>>(p.xn, p.row_tok, p.counts, d.D, p.xhi, p.xlo);
    // 4 gate/up + SwiGLU, 5 down
    if ((err = launch_grouped_ffn(w, d, use_routed, R, p.xhi, p.xlo, p.hhi, p.hlo, p.y, p.counts, p.items1, p.items2,
                                  num_sms, status, st)))
        return err;
    // 6 combine
    prefill_combine_kernel<<<num_sms * 4, 256, 0, st>>>(x, p.y, p.tok_row, p.wts, T, d.D, d.K, use_routed ? 1 : 0);
    if (topk_idx) cudaMemcpyAsync(topk_idx, p.ids, sizeof(int32_t) * T * d.K, cudaMemcpyDeviceToDevice, st);
    if (topk_w) cudaMemcpyAsync(topk_w, p.wts, sizeof(float) * T * d.K, cudaMemcpyDeviceToDevice, st);
    return cudaGetLastError();
}

// ---------------------------------------- expert parallelism, peer memory

constexpr uint64_t kEpWaitNs = 4000000000ull;  // a peer that has not answered in 4 s is taken as gone
constexpr unsigned kStatEpPeer = 128u;

// After every CTA's peer stores: the last CTA to finish raises flag `me` of
// every rank's region (flag_off) to `epoch`, after storing `cnt[d]` into
// slot `me` of the region's counts (cnt_off) when cnt is given. Every thread
// of the CTA calls it once, after its own stores.
__device__ void ep_signal_last(const EpPeers& peers, int n_shards, int me, size_t flag_off, size_t cnt_off,
                               const int* cnt, unsigned* done, unsigned epoch) {
    __threadfence_system();
    __syncthreads();
    if (threadIdx.x != 0) return;
    if (atomicAdd(done, 1u) != gridDim.x - 1) return;
    __threadfence_system();
    if (cnt)
        for (int d = 0; d < n_shards; ++d)
            reinterpret_cast<volatile int*>(peers.base[d] + cnt_off)[me] = cnt[d];
    __threadfence_system();
    for (int d = 0; d < n_shards; ++d) st_release_sys(reinterpret_cast<unsigned*>(peers.base[d] + flag_off) + me, epoch);
    *reinterpret_cast<volatile unsigned*>(done) = 0u;  // for the next launch (stream order)
}

// Rows of the last pack into the receivers' regions: pair i = (t, k) sent
// to rank d at position j of d's list lands in slot [me][j] of d's
// recv_rows / recv_expert; send_pos[i] becomes d * cap + j, where d will put
// the expert output in this rank's back_rows. One warp per pair.
__global__ void ep_push_kernel(const float* __restrict__ xn, int* send_pos, const int32_t* __restrict__ ids,
                               const int32_t* __restrict__ send_counts, int T, int K, int D, int e_local,
                               int n_shards, int me, const __grid_constant__ EpPeers peers, EpRegion R, unsigned* done,
                               unsigned epoch) {
    __shared__ int base[kMaxShards];
    __shared__ int cnt[kMaxShards];
    if (threadIdx.x == 0) {
        int o = 0;
        for (int d = 0; d < n_shards; ++d) {
            base[d] = o;
            cnt[d] = send_counts[d];
            o += cnt[d];
        }
    }
    __syncthreads();
    const int warps = (gridDim.x * blockDim.x) >> 5, lane = threadIdx.x & 31;
    for (int i = (blockIdx.x * blockDim.x + threadIdx.x) >> 5; i < T * K; i += warps) {
        const int pos = send_pos[i];
        if (pos < 0) continue;
        const int e = ids[i], d = e / e_local, j = pos - base[d];
        const size_t slot = (size_t)me * R.cap + j;
        const float4* src = reinterpret_cast<const float4*>(xn + (size_t)(i / K) * D);
        float4* dst = reinterpret_cast<float4*>(peers.base[d] + R.recv_rows) + slot * (size_t)(D / 4);
        for (int c = lane; c < D / 4; c += 32) dst[c] = src[c];
        if (lane == 0) {
            reinterpret_cast<int32_t*>(peers.base[d] + R.recv_expert)[slot] = e - d * e_local;
            send_pos[i] = d * R.cap + j;
        }
    }
    ep_signal_last(peers, n_shards, me, R.flag_rows, R.recv_cnt, cnt, done, epoch);
}

// Lane q waits until flags[q] has reached `epoch` (bounded: kEpWaitNs, then
// status bit kStatEpPeer and the kernel returns).
__global__ void ep_wait_kernel(const unsigned* flags, int n, unsigned epoch, unsigned* status) {
    const int q = threadIdx.x;
    if (q >= n) return;
    if ((int)(ld_acquire_sys(flags + q) - epoch) >= 0) return;
    const uint64_t t0 = global_ns();
    while ((int)(ld_acquire_sys(flags + q) - epoch) < 0) {
        if (global_ns() - t0 > kEpWaitNs) {
            atomicOr(status, kStatEpPeer);
            return;
        }
        __nanosleep(256);
    }
}

// Expert outputs back to their senders: received slot (q, j) -> row j of
// back_rows[me] in q's region (zeros for a row no local expert took). One
// warp per row; then flag_back[me] of every rank's region.
__global__ void ep_scatter_back_kernel(const float* __restrict__ Y, const int* __restrict__ pos_of_src,
                                       const int* recv_cnt, int n_shards, int D, int me,
                                       const __grid_constant__ EpPeers peers, EpRegion R, unsigned* done,
                                       unsigned epoch) {
    __shared__ int soff[kMaxShards + 1];
    if (threadIdx.x == 0) {
        int o = 0;
        for (int q = 0; q < n_shards; ++q) {
            soff[q] = o;
            o += min(max(__ldcg(recv_cnt + q), 0), R.cap);
        }
        soff[n_shards] = o;
    }
    __syncthreads();
    const int warps = (gridDim.x * blockDim.x) >> 5, lane = threadIdx.x & 31;
    for (int m = (blockIdx.x * blockDim.x + threadIdx.x) >> 5; m < soff[n_shards]; m += warps) {
        int q = 0;
        while (m >= soff[q + 1]) ++q;
        const int j = m - soff[q];
        const int r = pos_of_src[q * R.cap + j];
        float4* dst = reinterpret_cast<float4*>(peers.base[q] + R.back_rows) + ((size_t)me * R.cap + j) * (size_t)(D / 4);
        if (r < 0) {
            for (int c = lane; c < D / 4; c += 32) dst[c] = make_float4(0.f, 0.f, 0.f, 0.f);
            continue;
        }
        const float4* src = reinterpret_cast<const float4*>(Y + (size_t)r * D);
        for (int c = lane; c < D / 4; c += 32) dst[c] = src[c];
    }
    ep_signal_last(peers, n_shards, me, R.flag_back, 0, nullptr, done, epoch);
}

// ------------------------------------------------------- expert parallelism

namespace {

struct EpWs {
    float* xn;          // [T_max][D]
    double *cen, *bnd;  // [T_max][E] router logit centre / bound
    int32_t* ids;       // [T_max][K]
    float* wts;         // [T_max][K]
    int* send_pos;      // [T_max][K]
    int* row_src;       // [R_cap]
    int* pos_of_src;    // [R_cap]
    int* counts;        // [4]
    int4* items1;
    int4* items2;
    __nv_bfloat16 *xhi, *xlo, *hhi, *hlo;
    float* y;           // [R_cap][D]
    int32_t* send_counts;  // [kMaxShards] peer-memory path: rows for each receiver
    int32_t* send_expert;  // [T_max][K]   peer-memory path: pack's scratch
    unsigned* done;        // [2] last-CTA counters of the push and scatter-back kernels (zero between launches)
    size_t R_cap, bytes;
};

EpWs ep_carve(unsigned char* base, const EpShape& s) {
    const size_t R = (size_t)s.n_recv_cap + s.T_max, tiles = R / kTN + s.e_local + 1;
    EpWs w{};
    size_t b = 0;
    auto take = [&](size_t n) {
        unsigned char* r = base ? base + b : nullptr;
        b += (n + 255) & ~(size_t)255;
        return r;
    };
    w.xn = reinterpret_cast<float*>(take((size_t)s.T_max * s.D * 4));
    w.cen = reinterpret_cast<double*>(take((size_t)s.T_max * s.E * 8));
    w.bnd = reinterpret_cast<double*>(take((size_t)s.T_max * s.E * 8));
    w.ids = reinterpret_cast<int32_t*>(take((size_t)s.T_max * s.K * 4));
    w.wts = reinterpret_cast<float*>(take((size_t)s.T_max * s.K * 4));
    w.send_pos = reinterpret_cast<int*>(take((size_t)s.T_max * s.K * 4));
    w.row_src = reinterpret_cast<int*>(take(R * 4));
    w.pos_of_src = reinterpret_cast<int*>(take(R * 4));
    w.counts = reinterpret_cast<int*>(take(16));
    w.items1 = reinterpret_cast<int4*>(take(tiles * (s.F / (kTM / 2)) * 16));
    w.items2 = reinterpret_cast<int4*>(take(tiles * (s.D / kTM) * 16));
    w.xhi = reinterpret_cast<__nv_bfloat16*>(take(R * s.D * 2));
    w.xlo = reinterpret_cast<__nv_bfloat16*>(take(R * s.D * 2));
    w.hhi = reinterpret_cast<__nv_bfloat16*>(take(R * s.F * 2));
    w.hlo = reinterpret_cast<__nv_bfloat16*>(take(R * s.F * 2));
    w.y = reinterpret_cast<float*>(take(R * s.D * 4));
    w.send_counts = reinterpret_cast<int32_t*>(take(kMaxShards * 4));
    w.send_expert = reinterpret_cast<int32_t*>(take((size_t)s.T_max * s.K * 4));
    w.done = reinterpret_cast<unsigned*>(take(16));
    w.R_cap = R;
    w.bytes = b;
    return w;
}

}  // namespace

cudaError_t ep_check(const MoeDims& d, int n_shards) {
    if (n_shards < 1 || n_shards > kMaxShards || d.E % n_shards) return cudaErrorInvalidValue;
    MoeDims dl = d;
    dl.E = d.E / n_shards;
    dl.K = d.K < dl.E ? d.K : dl.E;
    return prefill_check(dl) == cudaSuccess && prefill_check(d) == cudaSuccess ? cudaSuccess : cudaErrorInvalidValue;
}

size_t ep_workspace_bytes(const EpShape& s) { return ep_carve(nullptr, s).bytes; }

cudaError_t launch_ep_dispatch(const MoeLayerDev& w, const MoeDims& d, const EpShape& s, unsigned char* ws,
                               const float* x, int T, float* send_rows, int32_t* send_expert, int32_t* send_counts,
                               int routed, int num_sms, unsigned long long* stats, cudaStream_t st) {
    if (T <= 0 || T > s.T_max) return cudaErrorInvalidValue;
    const EpWs p = ep_carve(ws, s);
    PrefillRouteArgs ra{x, w.ffn_norm, w.router, w.router_bias, p.xn, p.ids, p.wts, stats, T, d.D, d.E, d.K,
                        p.cen, p.bnd};
    cudaError_t err = launch_route(ra, num_sms, st);
    if (err) return err;
    ep_pack_kernel<<<1, 1024, 0, st>>>(p.ids, T, d.K, s.e_local, s.n_shards, routed && w.gate_q ? 1 : 0, p.send_pos,
                                       send_counts, send_expert);
    ep_pack_rows_kernel<<<num_sms * 4, 256, 0, st>>>(p.xn, p.send_pos, T, d.K, d.D, send_rows);
    return cudaGetLastError();
}

cudaError_t launch_ep_experts(const MoeLayerDev& w, const MoeDims& dl, const EpShape& s, unsigned char* ws, int T,
                              const float* recv_rows, const int32_t* recv_expert, int n_recv, float* out_rows,
                              int routed, int num_sms, unsigned* status, cudaStream_t st) {
    if (n_recv < 0 || n_recv > s.n_recv_cap || T <= 0 || T > s.T_max) return cudaErrorInvalidValue;
    const EpWs p = ep_carve(ws, s);
    const bool use_routed = routed && w.gate_q && w.up_q && w.down_q;
    const int mt1 = dl.F / (kTM / 2), mt2 = dl.D / kTM;
    ep_group_kernel<<<1, 1024, 0, st>>>(recv_expert, n_recv, T, dl.E, use_routed ? 1 : 0, mt1, mt2, p.counts,
                                        p.row_src, p.pos_of_src, p.items1, p.items2, nullptr, 0, 0);
    ep_gather_split_kernel<<<num_sms * 4, 256, 0, st>>>(recv_rows, p.xn, p.row_src, p.counts, n_recv, dl.D, p.xhi,
                                                        p.xlo);
    cudaError_t err = launch_grouped_ffn(w, dl, use_routed, p.R_cap, p.xhi, p.xlo, p.hhi, p.hlo, p.y, p.counts,
                                         p.items1, p.items2, num_sms, status, st);
    if (err) return err;
    if (n_recv > 0) ep_scatter_kernel<<<num_sms * 4, 256, 0, st>>>(p.y, p.pos_of_src, n_recv, dl.D, out_rows);
    return cudaGetLastError();
}

cudaError_t launch_ep_combine(const MoeDims& d, const EpShape& s, unsigned char* ws, float* x, int T, int n_recv,
                              const float* back_rows, int num_sms, cudaStream_t st) {
    if (T <= 0 || T > s.T_max) return cudaErrorInvalidValue;
    const EpWs p = ep_carve(ws, s);
    ep_combine_kernel<<<num_sms * 4, 256, 0, st>>>(x, p.y, p.pos_of_src, back_rows, p.send_pos, p.wts, T, d.D, d.K,
                                                   n_recv);
    return cudaGetLastError();
}

EpRegion ep_region_layout(const EpShape& s) {
    EpRegion r{};
    r.cap = s.n_recv_cap / s.n_shards;
    size_t b = 0;
    auto take = [&](size_t n) {
        const size_t o = b;
        b += (n + 255) & ~(size_t)255;
        return o;
    };
    const size_t slots = (size_t)s.n_shards * r.cap;
    r.header = take(sizeof(EpRegionHeader));
    r.recv_rows = take(slots * s.D * 4);
    r.recv_expert = take(slots * 4);
    r.back_rows = take(slots * s.D * 4);
    r.recv_cnt = take((size_t)s.n_shards * 4);
    r.flag_rows = take((size_t)s.n_shards * 4);
    r.flag_back = take((size_t)s.n_shards * 4);
    r.bytes = b;
    return r;
}

cudaError_t launch_ep_p2p_dispatch(const MoeLayerDev& w, const MoeDims& d, const EpShape& s, unsigned char* ws,
                                   const float* x, int T, int routed, int num_sms, unsigned long long* stats,
                                   const EpPeers& peers, int me, unsigned epoch, cudaStream_t st) {
    if (T <= 0 || T > s.T_max || me < 0 || me >= s.n_shards) return cudaErrorInvalidValue;
    const EpWs p = ep_carve(ws, s);
    const EpRegion R = ep_region_layout(s);
    PrefillRouteArgs ra{x, w.ffn_norm, w.router, w.router_bias, p.xn, p.ids, p.wts, stats, T, d.D, d.E, d.K,
                        p.cen, p.bnd};
    cudaError_t err = launch_route(ra, num_sms, st);
    if (err) return err;
    ep_pack_kernel<<<1, 1024, 0, st>>>(p.ids, T, d.K, s.e_local, s.n_shards, routed && w.gate_q ? 1 : 0, p.send_pos,
                                       p.send_counts, p.send_expert);
    ep_push_kernel<<<num_sms * 2, 256, 0, st>>>(p.xn, p.send_pos, p.ids, p.send_counts, T, d.K, d.D, s.e_local,
                                                s.n_shards, me, peers, R, p.done, epoch);
    return cudaGetLastError();
}

cudaError_t launch_ep_p2p_experts(const MoeLayerDev& w, const MoeDims& dl, const EpShape& s, unsigned char* ws,
                                  int T, int routed, int num_sms, unsigned* status, const EpPeers& peers, int me,
                                  unsigned epoch, cudaStream_t st) {
    if (T <= 0 || T > s.T_max || me < 0 || me >= s.n_shards) return cudaErrorInvalidValue;
    const EpWs p = ep_carve(ws, s);
    const EpRegion R = ep_region_layout(s);
    unsigned char* own = peers.base[me];
    const int n_slots = s.n_shards * R.cap;
    const bool use_routed = routed && w.gate_q && w.up_q && w.down_q;
    const int mt1 = dl.F / (kTM / 2), mt2 = dl.D / kTM;
    ep_wait_kernel<<<1, 32, 0, st>>>(reinterpret_cast<const unsigned*>(own + R.flag_rows), s.n_shards, epoch, status);
    const int* recv_cnt = reinterpret_cast<const int*>(own + R.recv_cnt);
    ep_group_kernel<<<1, 1024, 0, st>>>(reinterpret_cast<const int32_t*>(own + R.recv_expert), n_slots, T, dl.E,
                                        use_routed ? 1 : 0, mt1, mt2, p.counts, p.row_src, p.pos_of_src, p.items1,
                                        p.items2, recv_cnt, s.n_shards, R.cap);
    ep_gather_split_kernel<<<num_sms * 4, 256, 0, st>>>(reinterpret_cast<const float*>(own + R.recv_rows), p.xn,
                                                        p.row_src, p.counts, n_slots, dl.D, p.xhi, p.xlo);
    if (use_routed) {
        // the down GEMM's epilogue stores each received row's output straight
        // into its sender's region and raises the flags itself
        GroupGemmArgs pe{};
        pe.row_src = p.row_src;
        for (int q = 0; q < s.n_shards; ++q) pe.peer[q] = peers.base[q];
        pe.back_off = R.back_rows;
        pe.flag_off = R.flag_back;
        pe.n_slots = n_slots;
        pe.cap = R.cap;
        pe.me = me;
        pe.n_shards = s.n_shards;
        pe.done = p.done + 1;
        pe.epoch = epoch;
        return launch_grouped_ffn(w, dl, use_routed, p.R_cap, p.xhi, p.xlo, p.hhi, p.hlo, p.y, p.counts, p.items1,
                                  p.items2, num_sms, status, st, &pe);
    }
    // routed experts off on this rank: zero rows back for whatever was sent
    cudaError_t err = launch_grouped_ffn(w, dl, use_routed, p.R_cap, p.xhi, p.xlo, p.hhi, p.hlo, p.y, p.counts,
                                         p.items1, p.items2, num_sms, status, st);
    if (err) return err;
    ep_scatter_back_kernel<<<num_sms * 2, 256, 0, st>>>(p.y, p.pos_of_src, recv_cnt, s.n_shards, dl.D, me, peers, R,
                                                        p.done + 1, epoch);
    return cudaGetLastError();
}

cudaError_t launch_ep_p2p_combine(const MoeDims& d, const EpShape& s, unsigned char* ws, float* x, int T,
                                  int num_sms, unsigned* status, const EpPeers& peers, int me, unsigned epoch,
                                  cudaStream_t st) {
    if (T <= 0 || T > s.T_max || me < 0 || me >= s.n_shards) return cudaErrorInvalidValue;
    const EpWs p = ep_carve(ws, s);
    const EpRegion R = ep_region_layout(s);
    unsigned char* own = peers.base[me];
    ep_wait_kernel<<<1, 32, 0, st>>>(reinterpret_cast<const unsigned*>(own + R.flag_back), s.n_shards, epoch, status);
    ep_combine_kernel<<<num_sms * 4, 256, 0, st>>>(x, p.y, p.pos_of_src, reinterpret_cast<const float*>(own + R.back_rows),
                                                   p.send_pos, p.wts, T, d.D, d.K, s.n_shards * R.cap);
    return cudaGetLastError();
}

cudaError_t ep_p2p_counts(const EpShape& s, unsigned char* ws, const unsigned char* region, int32_t* send_counts,
                          int32_t* recv_counts, cudaStream_t st) {
    const EpWs p = ep_carve(ws, s);
    const EpRegion R = ep_region_layout(s);
    cudaError_t err = cudaMemcpyAsync(send_counts, p.send_counts, sizeof(int32_t) * s.n_shards,
                                      cudaMemcpyDeviceToHost, st);
    if (!err) err = cudaMemcpyAsync(recv_counts, region + R.recv_cnt, sizeof(int32_t) * s.n_shards,
                                    cudaMemcpyDeviceToHost, st);
    if (!err) err = cudaStreamSynchronize(st);
    return err;
}

cudaError_t ep_copy_routing(const EpShape& s, unsigned char* ws, int T, int32_t* topk_idx, float* topk_w,
                            cudaStream_t st) {
    const EpWs p = ep_carve(ws, s);
    cudaError_t err = cudaSuccess;
    if (topk_idx) err = cudaMemcpyAsync(topk_idx, p.ids, sizeof(int32_t) * T * s.K, cudaMemcpyDeviceToDevice, st);
    if (!err && topk_w) err = cudaMemcpyAsync(topk_w, p.wts, sizeof(float) * T * s.K, cudaMemcpyDeviceToDevice, st);
    return err;
}

}  // namespace glmq
