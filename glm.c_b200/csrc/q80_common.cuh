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

// Quantize `n` fp32 values (n % 64 == 0) into digit planes + scale table in
// shared memory. planes: [n/64][3][64] int8, sxg: [n/32] scratch,
// sxtab: [n/64][4][2]. Must be called by all threads of the block; ends with
// __syncthreads(). A group with a non-finite element gets a NaN scale so the
// rows it feeds come out non-finite, as the fp32 reference's would.
__device__ __forceinline__ void quantize_to_planes(const float* __restrict__ src, int n, int8_t* planes,
                                                   float* sxg, float* sxtab) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nwarps = blockDim.x >> 5;
    const int groups = n >> 5;
    for (int g = warp; g < groups; g += nwarps) {
        const float v = src[g * 32 + lane];
        float a = fabsf(v);
        const bool bad = __any_sync(0xffffffffu, !isfinite(v));
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) a = fmaxf(a, __shfl_xor_sync(0xffffffffu, a, off));
        int X = 0;
        float sx = 0.0f;
        if (bad) {
            sx = __int_as_float(0x7fc00000);
        } else if (a > 0.0f) {
            int e = ilogbf(a) - 22;  // a * 2^-e in [2^22, 2^23)
            if (ldexpf(a, -e) > kDigitMax) e += 1;
            sx = ldexpf(1.0f, e);
            X = __float2int_rn(ldexpf(v, -e));
        }
        const int lo = ((X + 128) & 255) - 128;
        const int x1 = (X - lo) >> 8;
        const int mid = ((x1 + 128) & 255) - 128;
        const int hi = (x1 - mid) >> 8;
        int8_t* c = planes + (g >> 1) * kChunkBytes + (g & 1) * 32 + lane;
        c[0] = (int8_t)hi;
        c[64] = (int8_t)mid;
        c[128] = (int8_t)lo;
        if (lane == 0) sxg[g] = sx;
    }
    __syncthreads();
    const int chunks = n >> 6;
    for (int i = threadIdx.x; i < chunks * 4; i += blockDim.x) {
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
    __syncthreads();
}

// Accumulate one 16-row x 64-column chunk of a Q8 matrix into the lane's
// partial sums for rows gid (acc0) and gid+8 (acc1).
//   q0/q1: this lane's 16 weight bytes of row gid / gid+8
//   s0/s1: fp32 scales of row gid / gid+8 for the chunk's two groups
//   b:     this lane's B fragment (digit planes), tab: (colA, colB) factors
__device__ __forceinline__ void chunk_mma_accumulate(const int4& q0, const int4& q1, const float2& s0,
                                                     const float2& s1, const int4& b, const float2& tab,
                                                     int t, float& acc0, float& acc1) {
    int d[4] = {0, 0, 0, 0};
    mma_s8(d, (uint32_t)q0.x, (uint32_t)q1.x, (uint32_t)q0.y, (uint32_t)q1.y, (uint32_t)b.x, (uint32_t)b.y);
    mma_s8(d, (uint32_t)q0.z, (uint32_t)q1.z, (uint32_t)q0.w, (uint32_t)q1.w, (uint32_t)b.z, (uint32_t)b.w);
    // Column A of lane t belongs to group g1 only for t==1; column B for t==1,2.
    const float swA0 = (t == 1) ? s0.y : s0.x, swB0 = (t == 1 || t == 2) ? s0.y : s0.x;
    const float swA1 = (t == 1) ? s1.y : s1.x, swB1 = (t == 1 || t == 2) ? s1.y : s1.x;
    acc0 = fmaf(i2f_exact22(d[0]), swA0 * tab.x, acc0);
    acc0 = fmaf(i2f_exact22(d[1]), swB0 * tab.y, acc0);
    acc1 = fmaf(i2f_exact22(d[2]), swA1 * tab.x, acc1);
    acc1 = fmaf(i2f_exact22(d[3]), swB1 * tab.y, acc1);
}

__device__ __forceinline__ float quad_sum(float v) {
    v += __shfl_xor_sync(0xffffffffu, v, 1);
    v += __shfl_xor_sync(0xffffffffu, v, 2);
    return v;
}

}  // namespace glmq
