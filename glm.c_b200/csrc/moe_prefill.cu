// Batched MoE prefill on sm_100a: T tokens through one MoE FFN layer
// (apply_moe_shared_ffn_layer, infer.c:1087-1216, applied to every token),
// with the expert products as grouped GEMMs on the 5th-generation tensor
// cores (tcgen05, accumulators in TMEM).
//
//   1 prefill_route_kernel   one CTA per token: certified rmsnorm, router
//                            logit centre/bound per expert (one warp each),
//                            exact top-k (route_common.cuh) -> ids, weights
//   2 prefill_dispatch_kernel rows = (token, slot) pairs grouped by expert
//                            (+ the shared expert: every token), tile lists
//   3 gather_split_kernel    activation rows as bf16 hi + lo
//   4 q8_group_gemm_kernel   gate and up: G/U[row][f] = xn . W[f]
//   5 swiglu_split_kernel    h = silu(G) * U as bf16 hi + lo
//   6 q8_group_gemm_kernel   down: Y[row][d] = h . Wd[d]
//   7 prefill_combine_kernel x += y_shared + sum_k (1.8 w_k) y_k, rank order
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

#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include "glm_internal.h"
#include "q80_common.cuh"
#include "route_common.cuh"

namespace glmq {

namespace {

constexpr int kMaxGroups = 257;  // routed experts + the shared expert
constexpr int kTM = 128;     // weight rows per tile (MMA M)
constexpr int kTN = 64;      // token rows per tile (MMA N)
constexpr int kTK = 64;      // K per stage (bf16: 128 bytes per row = one swizzle atom)
constexpr int kGBufs = 3;    // operand buffers (two stages of loads in flight)
constexpr int kGThreads = 256;
constexpr uint64_t kGWaitNs = 2000000000ull;

// Byte offset of element (row, k) in a K-major tile with 64 bf16 per row,
// 128-byte swizzle (16-byte chunk index XOR row % 8).
__device__ __forceinline__ uint32_t sw128(int row, int chunk16) {
    return (uint32_t)row * 128u + ((uint32_t)(chunk16 ^ (row & 7)) << 4);
}

// tcgen05 shared-memory descriptor: K-major, 128-byte swizzle, 8-row groups
// 1024 bytes apart (SBO), LBO 16 bytes, descriptor version 1.
__device__ __forceinline__ uint64_t umma_desc(uint32_t saddr) {
    return (uint64_t)((saddr >> 4) & 0x3FFFu) | ((uint64_t)1 << 16) | ((uint64_t)(1024 >> 4) << 32) |
           ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}

// Instruction descriptor: bf16 x bf16 -> f32, both K-major, M = 128, N = 64.
constexpr uint32_t kIdesc = (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(kTN >> 3) << 17) |
                            ((uint32_t)(kTM >> 4) << 24);

__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src, bool valid) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(dst), "l"(src), "r"(valid ? 16 : 0)
                 : "memory");
}

__device__ __forceinline__ void cp_async8(uint32_t dst, const void* src) {
    asm volatile("cp.async.ca.shared.global [%0], [%1], 8;\n" ::"r"(dst), "l"(src) : "memory");
}

__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::: "memory"); }

__device__ __forceinline__ void cp_async_wait2() { asm volatile("cp.async.wait_group 2;\n" ::: "memory"); }

__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;\n" ::: "memory"); }
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;\n" ::: "memory"); }

__device__ __forceinline__ void tc_mma(uint32_t tmem, uint64_t ad, uint64_t bd, uint32_t acc) {
    asm volatile(
        "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}\n" ::"r"(
            tmem),
        "l"(ad), "l"(bd), "r"(kIdesc), "r"(acc)
        : "memory");
}

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

// Bounded wait on an mbarrier phase (2 s of wall time); false if it gave up.
__device__ __forceinline__ bool bar_wait(uint64_t* bar, uint32_t parity) {
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = global_ns();
    while (global_ns() - t0 < kGWaitNs)
        if (mbar_try_wait_sleep(bar, parity, 20000)) return true;
    return false;
}

__device__ __forceinline__ void split_bf16(float v, __nv_bfloat16& hi, __nv_bfloat16& lo) {
    hi = __float2bfloat16_rn(v);
    const float h = __bfloat162float(hi);
    lo = __float2bfloat16_rn(isinf(h) ? 0.0f : v - h);  // inf stays inf, not inf + NaN
}

// ------------------------------------------------------------------ routing

__global__ void __launch_bounds__(512) prefill_route_kernel(PrefillRouteArgs a) {
    extern __shared__ __align__(16) unsigned char smr[];
    const int D = a.D, E = a.E, K = a.K, t = blockIdx.x;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, nw = blockDim.x >> 5;
    float* xsp = reinterpret_cast<float*>(smr);                  // padded xn [pad64(D)]
    float* xs = xsp + ((pad64(D) + 3) & ~3);                      // flat xn [D]
    double* cen = reinterpret_cast<double*>(xs + D);              // [E]
    double* bnd = cen + E;                                        // [E]
    float* sel = reinterpret_cast<float*>(bnd + E);               // 4E floats + E ints
    int* misc = reinterpret_cast<int*>(sel + 5 * E);
    __shared__ double red[16];
    __shared__ float s_inv;
    SelectScratch S;
    S.sel_c = sel;
    S.sel_lo = sel + E;
    S.sel_hi = sel + 2 * E;
    S.p_c = sel + 3 * E;
    S.taken = reinterpret_cast<int*>(sel + 4 * E);
    S.rank = misc;            // [kMaxTopK + 1]
    S.cert = misc + 16;
    int* s_idx = misc + 32;   // [kMaxTopK]
    float* s_w = reinterpret_cast<float*>(misc + 48);

    const float* x = a.x + (size_t)t * D;
    double ss = 0.0;
    for (int i = tid; i < D; i += blockDim.x) ss += (double)x[i] * (double)x[i];
    ss = warp_sum_d(ss);
    if (lane == 0) red[warp] = ss;
    __syncthreads();
    if (tid == 0) {
        double tot = 0.0;
        for (int w = 0; w < nw; ++w) tot += red[w];
        s_inv = rms_inv_certified(tot, x, D, a.stats ? &a.stats[3] : nullptr);
    }
    __syncthreads();
    const float inv = s_inv;
    for (int i = tid; i < D; i += blockDim.x) {
        const float v = __fmul_rn(__fmul_rn(x[i], inv), a.norm[i]);  // infer.c:751
        xs[i] = v;
        xsp[pad64(i)] = v;
        a.xn[(size_t)t * D + i] = v;
    }
    __syncthreads();
    for (int e = warp; e < E; e += nw) {
        double C, B;
        warp_logit_bound_contig(a.router + (size_t)e * D, xsp, D, C, B);
        if (lane == 0) {
            cen[e] = C;
            bnd[e] = B;
        }
    }
    __syncthreads();
    block_select(cen, bnd, a.bias, E, K, a.router, xs, D, tid, (int)blockDim.x, S, s_idx, s_w, a.stats,
                 []() { __syncthreads(); });
    if (tid < K) {
        a.topk_idx[(size_t)t * K + tid] = s_idx[tid];
        a.topk_w[(size_t)t * K + tid] = s_w[tid];
    }
}

// ----------------------------------------------------------------- dispatch

// One CTA. Groups 0..E-1 are the routed experts, group E the shared expert.
__global__ void __launch_bounds__(1024) prefill_dispatch_kernel(PrefillDispatchArgs a) {
    const int T = a.T, K = a.K, E = a.E, G = E + 1;
    __shared__ int cnt[kMaxGroups], off[kMaxGroups + 1], cur[kMaxGroups], tiles[kMaxGroups], toff[kMaxGroups + 1];
    for (int g = threadIdx.x; g < G; g += blockDim.x) {
        cnt[g] = g == E ? T : 0;
        cur[g] = 0;
    }
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
            tiles[g] = (cnt[g] + kTN - 1) / kTN;
            toff[g] = to;
            to += tiles[g];
        }
        off[G] = o;
        toff[G] = to;
        a.counts[0] = o;                                    // rows
        a.counts[1] = to * 2 * a.mt1;                       // gate/up tiles
        a.counts[2] = to * a.mt2;                           // down tiles
    }
    __syncthreads();
    // rows: (token, slot); routed order inside a group does not matter (rows
    // are independent), the shared expert's rows follow token order
    for (int i = threadIdx.x; i < T * (K + 1); i += blockDim.x) a.tok_row[i] = -1;
    __syncthreads();
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
    // tiles: item = {group, row0, nrows, m-tile | mat << 16}
    for (int g = threadIdx.x; g < G; g += blockDim.x)
        for (int j = 0; j < tiles[g]; ++j) {
            const int row0 = off[g] + j * kTN;
            const int nrows = min(kTN, off[g] + cnt[g] - row0);
            const int tile = toff[g] + j;
            for (int mat = 0; mat < 2; ++mat)
                for (int mt = 0; mt < a.mt1; ++mt)
                    a.items1[(tile * 2 + mat) * a.mt1 + mt] = make_int4(g, row0, nrows, mt | (mat << 16));
            for (int mt = 0; mt < a.mt2; ++mt) a.items2[tile * a.mt2 + mt] = make_int4(g, row0, nrows, mt);
        }
}

// Activation rows (token xn) as bf16 hi + lo.
__global__ void gather_split_kernel(const float* xn, const int* row_tok, const int* counts, int D,
                                    __nv_bfloat16* hi, __nv_bfloat16* lo) {
    const int R = counts[0];
    for (int r = blockIdx.x; r < R; r += gridDim.x) {
        const float* src = xn + (size_t)row_tok[r] * D;
        for (int i = threadIdx.x; i < D; i += blockDim.x) split_bf16(src[i], hi[(size_t)r * D + i], lo[(size_t)r * D + i]);
    }
}

// h = silu(G) * U (infer.c:1184-1188, 1197-1201) as bf16 hi + lo.
__global__ void swiglu_split_kernel(const float* Gm, const float* Um, const int* counts, int F, __nv_bfloat16* hi,
                                    __nv_bfloat16* lo) {
    const size_t n = (size_t)counts[0] * F;
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
        const float g = Gm[i];
        split_bf16(g / (1.0f + expf(-g)) * Um[i], hi[i], lo[i]);
    }
}

// ------------------------------------------------------------- grouped GEMM

struct GemmSmem {
    // per buffer: A_hi, A_lo [128][64] bf16, B_hi, B_lo [64][64] bf16 (swizzled),
    // raw int8 weights [128][64] and their scales [128][2]
    static constexpr uint32_t kA = kTM * 128, kB = kTN * 128, kRaw = kTM * kTK, kSc = kTM * 8;
    static constexpr uint32_t kBuf = 2 * kA + 2 * kB + kRaw + kSc;  // multiple of 1024
    static constexpr uint32_t kBars = kGBufs * kBuf;
    static constexpr uint32_t kTotal = kBars + 128;
};
static_assert(GemmSmem::kBuf % 1024 == 0, "operand buffers must keep 1024-byte alignment");

__global__ void __launch_bounds__(kGThreads, 1) q8_group_gemm_kernel(GroupGemmArgs a) {
    extern __shared__ __align__(1024) unsigned char gsm_raw[];
    unsigned char* sm = gsm_raw + ((1024u - (smem_addr(gsm_raw) & 1023u)) & 1023u);
    uint64_t* mbar = reinterpret_cast<uint64_t*>(sm + GemmSmem::kBars);
    uint32_t* tslot = reinterpret_cast<uint32_t*>(sm + GemmSmem::kBars + 64);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int n_items = a.counts[a.mode == 0 ? 1 : 2];
    const int Kd = a.K, nst = Kd / kTK, sgrp = Kd >> 5;

    if (tid == 0) {
        for (int b = 0; b < kGBufs; ++b) mbar_init(&mbar[b], 1);
        mbar_init_fence();
    }
    if (warp == 0) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;\n" ::"r"(smem_addr(tslot)),
                     "r"(kTN)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;\n" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tslot;

    uint32_t ncommit[kGBufs] = {0, 0, 0};
    unsigned gstage = 0;  // running stage count: buffer = gstage % kGBufs
    bool failed = false;

    for (int item = blockIdx.x; item < n_items; item += gridDim.x) {
        const int4 it = (a.mode == 0 ? a.items1 : a.items2)[item];
        const int g = it.x, row0 = it.y, nrows = it.z, mt = it.w & 0xffff, mat = it.w >> 16;
        const int m0 = mt * kTM;
        const int8_t* wq;
        const float* ws;
        size_t moff;  // expert offset in rows of the weight matrix
        if (a.mode == 0) {
            const bool sh = g == a.E;
            wq = mat ? (sh ? a.w.up_sh_q : a.w.up_q) : (sh ? a.w.gate_sh_q : a.w.gate_q);
            ws = mat ? (sh ? a.w.up_sh_s : a.w.up_s) : (sh ? a.w.gate_sh_s : a.w.gate_s);
            moff = sh ? 0 : (size_t)g * a.Mtot;
        } else {
            const bool sh = g == a.E;
            wq = sh ? a.w.down_sh_q : a.w.down_q;
            ws = sh ? a.w.down_sh_s : a.w.down_s;
            moff = sh ? 0 : (size_t)g * a.Mtot;
        }
        const int8_t* wrow0 = wq + (moff + m0) * (size_t)Kd;
        const float* srow0 = ws + (moff + m0) * (size_t)sgrp;
        const __nv_bfloat16* bhi = static_cast<const __nv_bfloat16*>(a.bhi) + (size_t)row0 * Kd;
        const __nv_bfloat16* blo = static_cast<const __nv_bfloat16*>(a.blo) + (size_t)row0 * Kd;

        // stage s of this item -> copies into buffer b (weights raw, scales, token tiles)
        auto issue = [&](int s, int b) {
            unsigned char* buf = sm + (size_t)b * GemmSmem::kBuf;
            const uint32_t sA_raw = smem_addr(buf + 2 * GemmSmem::kA + 2 * GemmSmem::kB);
            const uint32_t sSc = sA_raw + GemmSmem::kRaw;
            const uint32_t sBhi = smem_addr(buf + 2 * GemmSmem::kA), sBlo = sBhi + GemmSmem::kB;
            const int k0 = s * kTK;
            for (int c = tid; c < kTM * 4; c += kGThreads) {  // 128 rows x 4 x 16 bytes
                const int r = c >> 2, p = c & 3;
                cp_async16(sA_raw + r * kTK + p * 16, wrow0 + (size_t)r * Kd + k0 + p * 16, true);
            }
            for (int r = tid; r < kTM; r += kGThreads) cp_async8(sSc + r * 8, srow0 + (size_t)r * sgrp + (k0 >> 5));
            for (int c = tid; c < kTN * 8; c += kGThreads) {  // 64 rows x 8 x 16 bytes, hi and lo
                const int n = c >> 3, p = c & 7;
                const bool valid = n < nrows;
                const size_t src = (size_t)(valid ? n : 0) * Kd + k0 + p * 8;
                cp_async16(sBhi + sw128(n, p), bhi + src, valid);
                cp_async16(sBlo + sw128(n, p), blo + src, valid);
            }
        };

        for (int s = 0; s < 2 && s < nst; ++s) {
            const unsigned gs = gstage + s;
            const int b = gs % kGBufs;
            if (ncommit[b]) failed |= !bar_wait(&mbar[b], (ncommit[b] - 1) & 1u);
            issue(s, b);
            cp_async_commit();
        }
        if (nst < 2) cp_async_commit();
        for (int s = 0; s < nst; ++s) {
            const unsigned gs = gstage + s;
            const int b = gs % kGBufs;
            if (s + 2 < nst) {
                const int b2 = (gs + 2) % kGBufs;
                if (ncommit[b2]) failed |= !bar_wait(&mbar[b2], (ncommit[b2] - 1) & 1u);
                issue(s + 2, b2);
            }
            cp_async_commit();  // (possibly empty) group: keeps "stage s landed" = wait_group 2
            cp_async_wait2();
            __syncthreads();
            // dequantise the weight tile: 128 rows x 64 int8 -> A_hi, A_lo
            unsigned char* buf = sm + (size_t)b * GemmSmem::kBuf;
            const int8_t* raw = reinterpret_cast<const int8_t*>(buf + 2 * GemmSmem::kA + 2 * GemmSmem::kB);
            const float* sc = reinterpret_cast<const float*>(buf + 2 * GemmSmem::kA + 2 * GemmSmem::kB +
                                                             GemmSmem::kRaw);
            for (int c = tid; c < kTM * 4; c += kGThreads) {  // 16 int8 per item
                const int r = c >> 2, p = c & 3;
                const int4 q = *reinterpret_cast<const int4*>(raw + r * kTK + p * 16);
                const float scale = sc[r * 2 + (p >> 1)];
                const int qw[4] = {q.x, q.y, q.z, q.w};
                __align__(16) __nv_bfloat16 h[16], l[16];
#pragma unroll
                for (int j = 0; j < 16; ++j) split_bf16((float)(int8_t)(qw[j >> 2] >> (8 * (j & 3))) * scale, h[j], l[j]);
                const int ch = p * 2;  // two 16-byte chunks (8 bf16 each)
                *reinterpret_cast<int4*>(buf + sw128(r, ch)) = *reinterpret_cast<const int4*>(h);
                *reinterpret_cast<int4*>(buf + sw128(r, ch + 1)) = *reinterpret_cast<const int4*>(h + 8);
                *reinterpret_cast<int4*>(buf + GemmSmem::kA + sw128(r, ch)) = *reinterpret_cast<const int4*>(l);
                *reinterpret_cast<int4*>(buf + GemmSmem::kA + sw128(r, ch + 1)) = *reinterpret_cast<const int4*>(l + 8);
            }
            asm volatile("fence.proxy.async.shared::cta;\n" ::: "memory");
            __syncthreads();
            if (tid == 0) {
                tc_fence_after();
                const uint32_t aHi = smem_addr(buf), aLo = aHi + GemmSmem::kA;
                const uint32_t bHi = aHi + 2 * GemmSmem::kA, bLo = bHi + GemmSmem::kB;
#pragma unroll
                for (int kk = 0; kk < kTK / 16; ++kk) {
                    const uint32_t o = kk * 32;
                    const uint32_t first = (s == 0 && kk == 0) ? 0u : 1u;
                    tc_mma(tmem, umma_desc(aHi + o), umma_desc(bHi + o), first);
                    tc_mma(tmem, umma_desc(aHi + o), umma_desc(bLo + o), 1u);
                    tc_mma(tmem, umma_desc(aLo + o), umma_desc(bHi + o), 1u);
                }
                tc_commit(&mbar[b]);
            }
            ++ncommit[b];
        }
        // the last commit covers every MMA of this tile
        const int blast = (gstage + nst - 1) % kGBufs;
        failed |= !bar_wait(&mbar[blast], (ncommit[blast] - 1) & 1u);
        gstage += nst;
        tc_fence_after();
        if (warp < 4) {
            float* out = a.mode == 0 ? (mat ? a.out1 : a.out0) : a.out0;
            const int m = warp * 32 + lane;
            for (int half = 0; half < kTN / 32; ++half) {
                float v[32];
                tc_ld32(tmem + ((uint32_t)(warp * 32) << 16) + half * 32, v);
#pragma unroll
                for (int j = 0; j < 32; ++j) {
                    const int n = half * 32 + j;
                    if (n < nrows) out[(size_t)(row0 + n) * a.Mtot + m0 + m] = v[j];
                }
            }
        }
        tc_fence_before();
        // a commit that never arrived stops this CTA (no further MMAs issued)
        if (__syncthreads_or(failed)) {
            failed = true;
            break;
        }
    }
    if (failed && tid == 0) atomicOr(a.status, 64u);
    __syncthreads();
    if (warp == 0) asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;\n" ::"r"(tmem), "r"(kTN) : "memory");
}

// ------------------------------------------------------------------ combine

// x[t] += y_shared + sum_k (1.8 w_k) y_k in rank order (infer.c:1175,1192,
// 1212-1214).
__global__ void prefill_combine_kernel(float* x, const float* Y, const int* tok_row, const float* topk_w, int D,
                                       int K, int routed) {
    const int t = blockIdx.x;
    const int* tr = tok_row + (size_t)t * (K + 1);
    for (int i = threadIdx.x; i < D; i += blockDim.x) {
        float acc = 0.0f;
        if (routed)
            for (int k = 0; k < K; ++k) {
                const int r = tr[k];
                if (r < 0) continue;
                acc = __fadd_rn(acc, __fmul_rn(__fmul_rn(topk_w[(size_t)t * K + k], 1.8f), Y[(size_t)r * D + i]));
            }
        const float ysh = Y[(size_t)tr[K] * D + i];
        x[(size_t)t * D + i] = __fadd_rn(x[(size_t)t * D + i], __fadd_rn(ysh, acc));
    }
}

}  // namespace

cudaError_t prefill_check(const MoeDims& d) {
    if (d.gs != 32 || d.D % kTM || d.F % kTM || d.D % kTK || d.F % kTK || d.E + 1 > kMaxGroups || d.K < 1 ||
        d.K > kMaxTopK || d.D > 8192)
        return cudaErrorInvalidValue;
    return cudaSuccess;
}

size_t prefill_workspace_bytes(const MoeDims& d, int T) {
    const size_t R = (size_t)T * (d.K + 1), tiles = R / kTN + d.E + 1;
    size_t b = 0;
    auto take = [&](size_t n) { b += (n + 255) & ~(size_t)255; };
    take((size_t)T * d.D * 4);              // xn
    take((size_t)T * d.K * 4 * 2);          // ids, weights
    take(R * 4);                            // row_tok
    take((size_t)T * (d.K + 1) * 4);        // tok_row
    take(4 * 4);                            // counts
    take(tiles * 2 * (d.F / kTM) * 16);     // items1
    take(tiles * (d.D / kTM) * 16);         // items2
    take(R * d.D * 2 * 2);                  // x hi/lo
    take(R * d.F * 4 * 2);                  // G, U
    take(R * d.F * 2 * 2);                  // h hi/lo
    take(R * d.D * 4);                      // Y
    return b;
}

cudaError_t launch_moe_prefill(const MoeLayerDev& w, const MoeDims& d, unsigned char* ws, float* x, int T,
                               int32_t* topk_idx, float* topk_w, int routed, int num_sms, unsigned* status,
                               unsigned long long* stats, cudaStream_t st) {
    cudaError_t err = prefill_check(d);
    if (err != cudaSuccess || T <= 0) return err != cudaSuccess ? err : cudaErrorInvalidValue;
    const size_t R = (size_t)T * (d.K + 1), tiles = R / kTN + d.E + 1;
    const int mt1 = d.F / kTM, mt2 = d.D / kTM;
    unsigned char* p = ws;
    auto take = [&](size_t n) {
        unsigned char* r = p;
        p += (n + 255) & ~(size_t)255;
        return r;
    };
    float* xn = reinterpret_cast<float*>(take((size_t)T * d.D * 4));
    int32_t* ids = reinterpret_cast<int32_t*>(take((size_t)T * d.K * 4 * 2));
    float* wts = reinterpret_cast<float*>(ids + (size_t)T * d.K);
    int* row_tok = reinterpret_cast<int*>(take(R * 4));
    int* tok_row = reinterpret_cast<int*>(take((size_t)T * (d.K + 1) * 4));
    int* counts = reinterpret_cast<int*>(take(16));
    int4* items1 = reinterpret_cast<int4*>(take(tiles * 2 * mt1 * 16));
    int4* items2 = reinterpret_cast<int4*>(take(tiles * mt2 * 16));
    __nv_bfloat16* xhi = reinterpret_cast<__nv_bfloat16*>(take(R * d.D * 2 * 2));
    __nv_bfloat16* xlo = xhi + R * d.D;
    float* Gm = reinterpret_cast<float*>(take(R * d.F * 4 * 2));
    float* Um = Gm + R * d.F;
    __nv_bfloat16* hhi = reinterpret_cast<__nv_bfloat16*>(take(R * d.F * 2 * 2));
    __nv_bfloat16* hlo = hhi + R * d.F;
    float* Y = reinterpret_cast<float*>(take(R * d.D * 4));

    // 1 routing
    PrefillRouteArgs ra{x, w.ffn_norm, w.router, w.router_bias, xn, ids, wts, stats, T, d.D, d.E, d.K};
    const size_t rsmem = sizeof(float) * ((pad64(d.D) + 3) & ~3) + sizeof(float) * d.D + 16 * (size_t)d.E +
                         20 * (size_t)d.E + 256;
    if ((err = cudaFuncSetAttribute(prefill_route_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)rsmem)))
        return err;
    prefill_route_kernel<<<T, 512, rsmem, st>>>(ra);
    // 2 dispatch
    PrefillDispatchArgs da{ids, T, d.K, d.E, routed && w.gate_q != nullptr, mt1, mt2, counts, row_tok, tok_row,
                           items1, items2};
    prefill_dispatch_kernel<<<1, 1024, 0, st>>>(da);
    // 3 activations
    gather_split_kernel<<<num_sms * 4, 256, 0, st>>>(xn, row_tok, counts, d.D, xhi, xlo);
    // 4 gate / up
    if ((err = cudaFuncSetAttribute(q8_group_gemm_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                    (int)(GemmSmem::kTotal + 1024))))
        return err;
    GroupGemmArgs g1{w, items1, items2, counts, xhi, xlo, Gm, Um, status, d.D, d.F, d.E, 0};
    q8_group_gemm_kernel<<<num_sms, kGThreads, GemmSmem::kTotal + 1024, st>>>(g1);
    // 5 SwiGLU
    swiglu_split_kernel<<<num_sms * 4, 256, 0, st>>>(Gm, Um, counts, d.F, hhi, hlo);
    // 6 down
    GroupGemmArgs g2{w, items1, items2, counts, hhi, hlo, Y, nullptr, status, d.F, d.D, d.E, 1};
    q8_group_gemm_kernel<<<num_sms, kGThreads, GemmSmem::kTotal + 1024, st>>>(g2);
    // 7 combine
    prefill_combine_kernel<<<T, 256, 0, st>>>(x, Y, tok_row, wts, d.D, d.K, routed && w.gate_q != nullptr);
    if (topk_idx) cudaMemcpyAsync(topk_idx, ids, sizeof(int32_t) * T * d.K, cudaMemcpyDeviceToDevice, st);
    if (topk_w) cudaMemcpyAsync(topk_w, wts, sizeof(float) * T * d.K, cudaMemcpyDeviceToDevice, st);
    return cudaGetLastError();
}

}  // namespace glmq
