// Device building blocks shared by the Q8 decode kernels (sm_100a).
//
// Q8 weights are glm.c's planar format (infer.c:765-786, model.h:65-84):
// int8 q[rows][cols] row-major plus fp32 s[rows][cols/gs] row-major.
//
// Dot-product engine. The int8 weights go straight from HBM into the A
// operand of the integer tensor-core MMA (mma.m16n8k32 .s8.s8.s32) -- no
// int8->float conversion per weight. The fp32 activation vector is
// re-expressed, per 32-element group g, as X = rint(x * 2^-e_g) with
// |X| <= 127*(65536+256+1), split into three balanced int8 digits
// (hi, mid, lo): x ~= 2^e_g * (hi*65536 + mid*256 + lo). Each digit plane is a
// column of the MMA's B operand, so one MMA yields exact int32 partial dots
// for all three planes; the epilogue rescales them by 2^(8p) * 2^e_g *
// s[row][g] in fp32. The only approximation is rounding x to 24 bits relative
// to its group maximum (<= 2^-23 of the group max), i.e. fp32-class accuracy.
//
// Chunk = 64 consecutive columns (two 32-column groups g0, g1). Lane
// (gid = lane>>2, t = lane&3) of a warp loads 16 bytes of row gid and of row
// gid+8 at column 16*t of the chunk; bytes 0-7 feed MMA #1, bytes 8-15 MMA #2.
// The k-slot permutation this implies is applied identically to B, so the
// dot products are unchanged. B column n carries (group, plane):
//   n: 0=(g0,hi) 1=(g0,mid) 2=(g1,hi) 3=(g1,mid) 4=(g0,lo) 5=(g1,lo) 6,7=0
// and is zero on the k-slots of the other group (lanes t<2 hold g0 columns,
// t>=2 hold g1 columns). The accumulator lane (gid, t) then holds columns
// 2t, 2t+1, whose scale factors are precomputed per chunk in `sxtab`.
#pragma once

#include <cstdint>
#include <utility>

#include <cuda_runtime.h>

namespace glmq {

constexpr int kChunkCols = 64;
constexpr int kChunkBytes = 192;       // 3 planes x 64 digit bytes, per chunk
constexpr int kChunkTab = 8;           // 4 lanes-in-quad x {colA, colB} scale factors
constexpr float kDigitMax = 8355711.0f;  // 127 * 65793: largest |X| with balanced digits

__device__ __forceinline__ float i2f_exact22(int v) {
    // Exact int->float for |v| < 2^22 with full-rate integer/FP ops.
    return __int_as_float(v + 0x4B400000) - 12582912.0f;
}

__device__ __forceinline__ void mma_s8(int (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                       uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 "
        "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};\n"
        : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// Streaming 16-byte weight load: read once per token, keep it out of L1.
__device__ __forceinline__ int4 ld_weights16(const int8_t* p) {
    int4 v;
    asm volatile("ld.global.nc.L1::no_allocate.v4.s32 {%0,%1,%2,%3}, [%4];\n"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "l"(p));
    return v;
}

__device__ __forceinline__ float2 ld_scales2(const float* p) {
    float2 v;
    asm volatile("ld.global.nc.v2.f32 {%0,%1}, [%2];\n" : "=f"(v.x), "=f"(v.y) : "l"(p));
    return v;
}

// Byte offset inside a chunk of this lane's B fragment, or -1 if the lane's
// B fragment is all zero (other group, or padding column).
__device__ __forceinline__ int b_frag_offset(int lane) {
    const int n = lane >> 2, t = lane & 3;
    if (n >= 6) return -1;
    const int group = (n == 2 || n == 3 || n == 5) ? 1 : 0;
    const int plane = (n < 4) ? (n & 1) : 2;
    if (group != (t >= 2 ? 1 : 0)) return -1;
    return plane * 64 + 16 * t;
}

// Accumulate one 16-row x 64-column chunk of a Q8 matrix into the lane's
// partial sums for rows gid (acc0) and gid+8 (acc1).
//   q0/q1: this lane's 16 weight bytes of row gid / gid+8
//   s0/s1: fp32 scales of row gid / gid+8 for the chunk's two groups
//   b:     this lane's B fragment (digit planes), tab: (colA, colB) factors
__device__ __forceinline__ void chunk_mma_accumulate(const int4& q0, const int4& q1, const float2& s0,
                                                     const float2& s1, const int4& b, const float2& tab,
                                                     int t, float& acc0, float& acc1) {
    // two independent MMAs (one per 8-byte half) so they issue back to back;
    // the int32 sum below is exact, as chaining them through C would be
    int d[4] = {0, 0, 0, 0}, e[4] = {0, 0, 0, 0};
    mma_s8(d, (uint32_t)q0.x, (uint32_t)q1.x, (uint32_t)q0.y, (uint32_t)q1.y, (uint32_t)b.x, (uint32_t)b.y);
    mma_s8(e, (uint32_t)q0.z, (uint32_t)q1.z, (uint32_t)q0.w, (uint32_t)q1.w, (uint32_t)b.z, (uint32_t)b.w);
#pragma unroll
    for (int i = 0; i < 4; ++i) d[i] += e[i];
    // Column A of lane t belongs to group g1 only for t==1; column B for t==1,2.
    const float swA0 = (t == 1) ? s0.y : s0.x, swB0 = (t == 1 || t == 2) ? s0.y : s0.x;
    const float swA1 = (t == 1) ? s1.y : s1.x, swB1 = (t == 1 || t == 2) ? s1.y : s1.x;
    acc0 = fmaf(i2f_exact22(d[0]), swA0 * tab.x, acc0);
    acc0 = fmaf(i2f_exact22(d[1]), swB0 * tab.y, acc0);
    acc1 = fmaf(i2f_exact22(d[2]), swA1 * tab.x, acc1);
    acc1 = fmaf(i2f_exact22(d[3]), swB1 * tab.y, acc1);
}

// ------------------------------------------------- gs = 16 weight scales
//
// glm.c's own export uses 16-column weight groups (glm47_flash_export.py:36),
// so one MMA column may not sum a whole 32-column x group. Lane t of a quad
// holds exactly the k-slots of chunk columns [16t, 16t+16) in its A fragment
// (its 16 weight bytes), i.e. of weight group w = t. Each B column carries
// one (weight group w, digit plane p) and is zero outside group w, and the
// columns are placed so that accumulator lane t (which holds columns 2t and
// 2t+1) receives the three plane sums of its own group w = t:
//   set X: column n = (w = n/2, p = n%2)              (hi, mid planes)
//   set Y: column n = (w = n/2, p = 2) for even n,   (lo plane)
//          zero for odd n
// Each set takes both 8-byte halves of the lanes' weight bytes, so a chunk
// costs 4 MMAs; the lane then scales its group's value
// 65536 hi + 256 mid + lo by its own weight scale s[row][4j + t] and by the
// scale of x group 2j + t/2 (columns 0-31 or 32-63 of chunk j). No per-lane
// table or selection is involved.
struct G16Lane {
    int offX, offY;  // byte offsets of the lane's B fragments in a chunk's planes, -1 = zero
};

__device__ __forceinline__ G16Lane g16_lane(int lane) {
    const int n = lane >> 2, t = lane & 3;  // B column n, k-slots of group t
    G16Lane L;
    L.offX = (n >> 1) == t ? (n & 1) * 64 + 16 * t : -1;
    L.offY = ((n >> 1) == t && (n & 1) == 0) ? 128 + 16 * t : -1;
    return L;
}

// Accumulate one 16-row x 64-column chunk with gs = 16 weight scales into the
// lane's partial sums for rows gid (acc0) and gid+8 (acc1).
//   q0/q1: this lane's 16 weight bytes of row gid / gid+8
//   s0/s1: weight scale of group t (lane-in-quad) of row gid / gid+8
//   bX/bY: this lane's B fragments (zero where G16Lane offX / offY < 0)
//   sx:    scale of the x group that holds weight group t
__device__ __forceinline__ void chunk_mma_accumulate_g16(const int4& q0, const int4& q1, float s0, float s1,
                                                         const int4& bX, const int4& bY, float sx, float& acc0,
                                                         float& acc1) {
    // four independent MMAs (set x half), summed exactly in int32 after
    int dx[4] = {0, 0, 0, 0}, dy[4] = {0, 0, 0, 0}, ex[4] = {0, 0, 0, 0}, ey[4] = {0, 0, 0, 0};
    mma_s8(dx, (uint32_t)q0.x, (uint32_t)q1.x, (uint32_t)q0.y, (uint32_t)q1.y, (uint32_t)bX.x, (uint32_t)bX.y);
    mma_s8(dy, (uint32_t)q0.x, (uint32_t)q1.x, (uint32_t)q0.y, (uint32_t)q1.y, (uint32_t)bY.x, (uint32_t)bY.y);
    mma_s8(ex, (uint32_t)q0.z, (uint32_t)q1.z, (uint32_t)q0.w, (uint32_t)q1.w, (uint32_t)bX.z, (uint32_t)bX.w);
    mma_s8(ey, (uint32_t)q0.z, (uint32_t)q1.z, (uint32_t)q0.w, (uint32_t)q1.w, (uint32_t)bY.z, (uint32_t)bY.w);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        dx[i] += ex[i];
        dy[i] += ey[i];
    }
    // columns 2t (hi), 2t+1 (mid) of X and 2t (lo) of Y; dy[1], dy[3] are the zero columns
    const float v0 = fmaf(i2f_exact22(dx[0]), 65536.0f, fmaf(i2f_exact22(dx[1]), 256.0f, i2f_exact22(dy[0])));
    const float v1 = fmaf(i2f_exact22(dx[2]), 65536.0f, fmaf(i2f_exact22(dx[3]), 256.0f, i2f_exact22(dy[2])));
    acc0 = fmaf(v0, s0 * sx, acc0);
    acc1 = fmaf(v1, s1 * sx, acc1);
}

__device__ __forceinline__ float ld_scale1(const float* p) {
    float v;
    asm volatile("ld.global.nc.f32 %0, [%1];\n" : "=f"(v) : "l"(p));
    return v;
}

__device__ __forceinline__ float quad_sum(float v) {
    v += __shfl_xor_sync(0xffffffffu, v, 1);
    v += __shfl_xor_sync(0xffffffffu, v, 2);
    return v;
}

// ------------------------------------------------------------ L2 loads

// Loads of data another CTA wrote (read through L2, never L1) that the
// compiler must issue exactly where they are written: a batch of these goes
// out back to back instead of being sunk to its uses one round trip at a time.
__device__ __forceinline__ float ldcg_f32(const float* p) {
    float v;
    asm volatile("ld.global.cg.f32 %0, [%1];\n" : "=f"(v) : "l"(p) : "memory");
    return v;
}

__device__ __forceinline__ double ldcg_f64(const double* p) {
    double v;
    asm volatile("ld.global.cg.f64 %0, [%1];\n" : "=d"(v) : "l"(p) : "memory");
    return v;
}

__device__ __forceinline__ float4 ldcg_f4(const float* p) {
    float4 v;
    asm volatile("ld.global.cg.v4.f32 {%0,%1,%2,%3}, [%4];\n"
                 : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
                 : "l"(p)
                 : "memory");
    return v;
}

// ------------------------------------------------ vectorised quantisation
//
// Group quantisation of the activations: each 32-element group with
// maximum |x| = a gets the scale 2^e, e = ilogb(a) - 22, so that every
// X = rn(x * 2^-e) fits 24 bits and splits exactly into three balanced
// signed bytes hi, mid, lo (X = 65536 hi + 256 mid + lo); a group with a
// non-finite element gets a NaN scale and zero digits, an all-zero group
// scale 0. Laid out for throughput: 8 lanes per group, 4 consecutive
// elements per lane,
// so a warp step covers 4 groups with one 16-byte load and three 4-byte digit
// stores per lane. Step s covers groups 4s .. 4s+3; warp w of nwarps takes
// steps w, w + nwarps, ... q4_load fetches kB such steps (global memory
// through L2 when kGlobal), q4_store quantises and stores them. For a group
// maximum a >= 2^-100 the powers of two 2^e and 2^-e are formed from exponent
// bits (the scaling products are exact, so the digits equal the ldexpf form);
// e = ilogb(a) - 22, plus one when a * 2^-e = 2^22 + mant(a)/2 would exceed
// 127*65793, i.e. when the 23-bit mantissa field of a exceeds 8322814.
template <bool kGlobal, int kB>
__device__ __forceinline__ void q4_load(const float* src, int groups, int s0, int nwarps, int lane,
                                        float4 (&v)[kB]) {
#pragma unroll
    for (int u = 0; u < kB; ++u) {
        const int g = 4 * (s0 + u * nwarps) + (lane >> 3);
        const float* p = src + g * 32 + (lane & 7) * 4;
        v[u] = g < groups ? (kGlobal ? ldcg_f4(p) : *reinterpret_cast<const float4*>(p))
                          : make_float4(0.f, 0.f, 0.f, 0.f);
    }
}

__device__ __forceinline__ unsigned pack_digit_bytes(int a, int b, int c, int d) {
    return (unsigned)(a & 255) | ((unsigned)(b & 255) << 8) | ((unsigned)(c & 255) << 16) | ((unsigned)d << 24);
}

// A group whose maximum |x| is below 2^-100 (a rare case, kept out of line so
// that the quantiser's hot code stays small): its scale and integers with
// the library's exponent functions.
struct TinyGroupQ {
    int x0, x1, x2, x3;
    float sx;
};

static __device__ __noinline__ TinyGroupQ tiny_group_q(float x0, float x1, float x2, float x3, unsigned am) {
    const float a = __uint_as_float(am);
    int e = ilogbf(a) - 22;
    if (ldexpf(a, -e) > kDigitMax) e += 1;
    return TinyGroupQ{__float2int_rn(ldexpf(x0, -e)), __float2int_rn(ldexpf(x1, -e)), __float2int_rn(ldexpf(x2, -e)),
                      __float2int_rn(ldexpf(x3, -e)), ldexpf(1.0f, e)};
}

template <int kB>
__device__ __forceinline__ void q4_store(const float4 (&v)[kB], int groups, int s0, int nwarps, int lane,
                                         int8_t* planes, float* sxg) {
#pragma unroll
    for (int u = 0; u < kB; ++u) {
        const int g = 4 * (s0 + u * nwarps) + (lane >> 3);
        const float x[4] = {v[u].x, v[u].y, v[u].z, v[u].w};
        unsigned am = 0u;
#pragma unroll
        for (int j = 0; j < 4; ++j) am = max(am, __float_as_uint(x[j]) & 0x7fffffffu);
        am = max(am, __shfl_xor_sync(0xffffffffu, am, 1));
        am = max(am, __shfl_xor_sync(0xffffffffu, am, 2));
        am = max(am, __shfl_xor_sync(0xffffffffu, am, 4));
        int X[4] = {0, 0, 0, 0};
        float sx = 0.0f;
        if (am >= 0x7f800000u) {  // inf or NaN in the group
            sx = __int_as_float(0x7fc00000);
        } else if (am >= (27u << 23)) {
            const int e = (int)(am >> 23) - 149 + ((am & 0x7fffffu) > 8322814u ? 1 : 0);
            sx = __uint_as_float((unsigned)(e + 127) << 23);
            const float inv = __uint_as_float((unsigned)(127 - e) << 23);
#pragma unroll
            for (int j = 0; j < 4; ++j) X[j] = __float2int_rn(__fmul_rn(x[j], inv));
        } else if (am != 0u) {  // tiny group: library scaling, out of line
            const TinyGroupQ t = tiny_group_q(x[0], x[1], x[2], x[3], am);
            X[0] = t.x0;
            X[1] = t.x1;
            X[2] = t.x2;
            X[3] = t.x3;
            sx = t.sx;
        }
        int hi[4], mid[4], lo[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            lo[j] = ((X[j] + 128) & 255) - 128;
            const int x1 = (X[j] - lo[j]) >> 8;
            mid[j] = ((x1 + 128) & 255) - 128;
            hi[j] = (x1 - mid[j]) >> 8;
        }
        if (g < groups) {
            unsigned* c = reinterpret_cast<unsigned*>(planes + (g >> 1) * kChunkBytes + (g & 1) * 32 + (lane & 7) * 4);
            c[0] = pack_digit_bytes(hi[0], hi[1], hi[2], hi[3]);
            c[16] = pack_digit_bytes(mid[0], mid[1], mid[2], mid[3]);
            c[32] = pack_digit_bytes(lo[0], lo[1], lo[2], lo[3]);
            if ((lane & 7) == 0) sxg[g] = sx;
        }
    }
}

// Per-chunk epilogue factors from the group scales (threads [0, nthreads)):
// lane-in-quad t of the MMA output holds B columns 2t and 2t+1, i.e.
// (g0 hi, g0 mid), (g1 hi, g1 mid), (g0 lo, g1 lo), unused.
__device__ __forceinline__ void fill_sxtab(const float* sxg, float* sxtab, int chunks, int tid, int nthreads) {
    for (int i = tid; i < chunks * 4; i += nthreads) {
        const int c = i >> 2, t = i & 3;
        const float s0 = sxg[2 * c], s1 = sxg[2 * c + 1];
        float A, B;
        if (t == 0) { A = 65536.0f * s0; B = 256.0f * s0; }
        else if (t == 1) { A = 65536.0f * s1; B = 256.0f * s1; }
        else if (t == 2) { A = s0; B = s1; }
        else { A = 0.0f; B = 0.0f; }
        sxtab[c * kChunkTab + 2 * t] = A;
        sxtab[c * kChunkTab + 2 * t + 1] = B;
    }
}

// Quantise src[0, n) (n % 64 == 0) into planes/sxg/sxtab, run by threads
// [0, nthreads) of a block that synchronise with `sync()` (e.g. the consumer
// warps of a warp-specialised kernel). kGlobal: src is global memory written
// by other CTAs; otherwise shared memory. kG16: no sxtab (the gs = 16 engine
// reads sxg). Ends with sync().
template <bool kGlobal, bool kG16 = false, typename Sync>
__device__ __forceinline__ void quantize_planes_part(const float* src, int n, int8_t* planes, float* sxg,
                                                     float* sxtab, int tid, int nthreads, Sync sync) {
    constexpr int kB = 4;
    const int groups = n >> 5, warp = tid >> 5, nwarps = nthreads >> 5, lane = tid & 31;
    for (int s0 = warp; 4 * s0 < groups; s0 += nwarps * kB) {
        float4 v[kB];
        q4_load<kGlobal, kB>(src, groups, s0, nwarps, lane, v);
        q4_store<kB>(v, groups, s0, nwarps, lane, planes, sxg);
    }
    sync();
    if constexpr (!kG16) {  // gs = 16 reads the group scales sxg directly
        fill_sxtab(sxg, sxtab, n >> 6, tid, nthreads);
        sync();
    }
}

// Quantize n fp32 values (n % 64 == 0; src 16-byte aligned, global or
// shared memory) into digit planes + scale table in shared memory with every
// thread of the block: planes [n/64][3][64] int8, sxg [n/32], sxtab
// [n/64][4][2]. All of a warp's loads are in flight at once. Ends with
// __syncthreads(). A group with a non-finite element gets a NaN scale so the
// rows it feeds come out non-finite, as the fp32 reference's would.
__device__ __forceinline__ void quantize_to_planes(const float* src, int n, int8_t* planes, float* sxg,
                                                   float* sxtab) {
    quantize_planes_part<false>(src, n, planes, sxg, sxtab, (int)threadIdx.x, (int)blockDim.x,
                                [] { __syncthreads(); });
}

// ------------------------------------------------------- TMA and mbarriers

// L2 prefetch hint for the 16-byte-aligned part of [p, p + bytes) (the
// unaligned ends are left out), one bulk request per MiB.
__device__ __forceinline__ void bulk_prefetch_l2(const void* p, size_t bytes) {
    uintptr_t a = (reinterpret_cast<uintptr_t>(p) + 15) & ~(uintptr_t)15;
    const uintptr_t e = (reinterpret_cast<uintptr_t>(p) + bytes) & ~(uintptr_t)15;
    while (a < e) {
        const uint32_t n = (uint32_t)(e - a < ((uintptr_t)1 << 20) ? e - a : ((uintptr_t)1 << 20));
        asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;\n" ::"l"(a), "r"(n) : "memory");
        a += n;
    }
}

__device__ __forceinline__ uint32_t smem_addr(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;\n" ::"r"(smem_addr(bar)), "r"(count) : "memory");
}

// Make mbarrier initialisation visible to the async (TMA) proxy.
__device__ __forceinline__ void mbar_init_fence() {
    asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];\n" ::"r"(smem_addr(bar)) : "memory");
}

// Arrive and register `bytes` of expected TMA traffic on the same phase.
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;\n" ::"r"(smem_addr(bar)), "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(ok)
        : "r"(smem_addr(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

// Programmatic dependent launch. A kernel started with launch_pdl may be
// scheduled while the previous kernel of its stream is still draining;
// pdl_enter(), its first statement, waits until that kernel has completed
// and its writes are visible, then lets the next kernel of the stream be
// scheduled early in turn. Every kernel launched with launch_pdl calls it
// before touching memory another kernel wrote.
__device__ __forceinline__ void pdl_enter() {
    asm volatile("griddepcontrol.wait;\n" ::: "memory");
    asm volatile("griddepcontrol.launch_dependents;\n" ::: "memory");
}

template <typename... KArgs, typename... Args>
inline cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                              Args&&... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

__device__ __forceinline__ uint64_t global_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;\n" : "=l"(t));
    return t;
}

// try_wait that lets the hardware suspend the thread (up to `hint_ns`) until
// the phase completes, instead of spinning on the barrier and taking shared
// memory issue slots from the threads doing the work.
__device__ __forceinline__ bool mbar_try_wait_sleep(uint64_t* bar, uint32_t parity, uint32_t hint_ns) {
    uint32_t ok;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(ok)
        : "r"(smem_addr(bar)), "r"(parity), "r"(hint_ns)
        : "memory");
    return ok != 0;
}

// Bounded wait: gives up after kWaitNs of wall time (a copy that never lands
// becomes an error status instead of a hung GPU).
constexpr uint64_t kWaitNs = 2000000000ull;  // 2 s
constexpr uint32_t kSuspendNs = 100000;      // 100 us per try

__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar, uint32_t parity) {
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = global_ns();
    while (global_ns() - t0 < kWaitNs)
        if (mbar_try_wait_sleep(bar, parity, kSuspendNs)) return true;
    return false;
}

// One contiguous global->shared bulk copy (TMA engine, no registers used);
// completion is counted in bytes on `bar`. dst, src and bytes must be
// multiples of 16. No cluster multicast.
__device__ __forceinline__ void bulk_copy_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];\n" ::"r"(
            smem_addr(dst)),
        "l"(src), "r"(bytes), "r"(smem_addr(bar))
        : "memory");
}

// 16-byte shared-memory load of an A/B fragment.
__device__ __forceinline__ int4 lds16(const int8_t* p) { return *reinterpret_cast<const int4*>(p); }

}  // namespace glmq
