// Persistent batch-1 MoE decode: one launch runs the MoE FFN of
// one or more consecutive layers for one token (apply_moe_shared_ffn_layer,
// infer.c:1087-1216, once per layer).
//
// Why persistent. Each MoE layer moves ~53.6 MB but only ~360 KB per SM; a
// kernel launch costs microseconds of start-up and tail, and a chain of
// small dependent kernels per layer spends most of its time there. Here one
// CTA per SM stays resident for all layers:
//
//   warp 15 (producer)  walks a fixed per-CTA schedule of weight tiles and
//                       streams each into a 5-slot shared-memory ring with
//                       TMA bulk copies (one copy per contiguous run of rows,
//                       completion counted on the slot's mbarrier). It runs
//                       ahead across phases and layers and stops only where
//                       data depends on routing: the routed gate/up and down
//                       rows of layer l wait for that layer's expert ids.
//   warps 0-14          consume the tiles phase by phase, in 5 groups of 3
//                       warps; group g owns ring slot g and processes the
//                       weight items that land there (a gate/up item holds
//                       8 gate rows and their 8 up rows, so SwiGLU finishes
//                       in-lane; a down item 16 output rows of one matrix):
//     P0  rmsnorm of x (every CTA), xn quantised to int8 digit planes
//     P1  CTA c < E: router logit centre/bound of expert c
//     --  grid barrier A
//     P2  every CTA ranks the experts itself (identical, certified result)
//         and hands the ids to its producer, which prefetches all of the
//         CTA's routed rows into L2; the shared gate/up items (already in
//         the ring) then the routed ones -> h
//     --  grid barrier B
//     P3  this CTA's output rows of the shared and the K routed down
//         matrices, each group quantising its slot's h first (group
//         barrier only); weighted combine in rank order + residual -> x
//     --  grid barrier C (between layers)
//
// While a layer's routing is decided, the producer also pulls the next
// layer's routing-independent weights (router row, shared expert rows) into
// L2.
//
// Grid barriers are a global arrival counter: after a block barrier one
// thread adds its arrival with a gpu-scope release (covering the CTA's
// writes ordered before it by that barrier) and polls with acquire loads;
// a block barrier then passes the others on. Every
// wait in this kernel (barriers, ring slots, routing hand-off) gives up after
// a bounded number of polls, records the reason in `status`, raises an abort
// flag, and the kernel leaves at its next grid barrier, so a fault cannot
// hang the GPU. One CTA per SM fits (checked at launch), so all CTAs are
// resident together.
#include <cstdint>

#include <cuda_runtime.h>

#include "glm_internal.h"
#include "q80_common.cuh"
#include "route_common.cuh"

namespace glmq {

constexpr int kPGroupWarps = 3;                // consumer warps per group; group g owns ring slot g
#ifndef GLM_P_INFLIGHT
#define GLM_P_INFLIGHT 5
#endif
// At most this many ring items in flight (issued, not landed); below the
// slot count it trades ring throughput for shorter queues behind the
// kernel's small critical-path loads (measured best: no limit, with the L2
// prefetches).
constexpr int kPInflight = GLM_P_INFLIGHT;

// Shape of the CTA for a weight group size. gs = 32: a 5-slot ring and 5
// consumer groups of 3 warps (+1 producer: 512 threads, 128 registers).
// gs = 16 doubles the scale bytes of every tile (16 rows of D = 2048 take
// 40 KB instead of 36 KB), so 5 slots no longer fit shared memory beside the
// activation planes: 4 slots and 4 groups (416 threads); its engine reads
// the x-group scales directly (no epilogue table).
template <int kGS>
struct PCfg {
    static constexpr int kSlots = kGS == 32 ? 5 : 4;
    static constexpr int kGroups = kSlots;  // one consumer group per ring slot
    static constexpr int kCons = kGroups * kPGroupWarps;
    static constexpr int kConsThreads = kCons * 32;
    static constexpr int kThreads = kConsThreads + 32;
    static constexpr int kTab = kGS == 32 ? kChunkTab : 0;  // epilogue-table floats per 64-column chunk
};
constexpr int kPMaxCons = PCfg<32>::kCons;
constexpr int kPTile = 16;                     // rows per ring item
constexpr int kPHRows = 8;                     // h rows per gate/up item (8 gate rows + their 8 up rows)
constexpr unsigned kStatBarrier = 4u, kStatFull = 8u, kStatEmpty = 16u, kStatRoute = 32u;
constexpr unsigned kStatAbort = kStatBarrier | kStatFull | kStatEmpty | kStatRoute;

struct PersistArgs {
    const MoeLayerDev* layers;  // device table
    int first, n_layers;
    float* x;
    float* h;
    double* center;
    double* bound;
    int32_t* topk_out;  // [n_layers][K] or null
    float* topkw_out;
    unsigned* bar;      // grid-barrier arrivals; zero at launch (the last CTA to exit resets it)
    unsigned* done;     // CTAs that have exited; zero at launch
    unsigned* status;
    unsigned long long* stats;
    int D, F, E, K, routed_enabled, slot_bytes;
    int next_layer;     // table index whose shared weights to pull into L2 during the last layer, or -1
    int gs;             // weight scale group (32 or 16)
    int sdiv;           // weight bytes per scale byte (gs / 4): a row of n weights has n / sdiv scale bytes
    int slots;          // ring slots
};

__host__ __device__ inline size_t p_take(size_t& o, size_t n) {
    const size_t r = o;
    o = (o + n + 127) & ~(size_t)127;
    return r;
}

// Dynamic shared memory layout (offsets in bytes).
struct PSmem {
    size_t bars, ring, xs, ph, px, tx, gx, th, gh, part, ys, bias, cen, bnd, sel, rscr, misc, total;
    // slots: ring slots (= consumer groups), tab: epilogue floats per chunk
    __host__ __device__ PSmem(int D, int F, int E, int K, int slot_bytes, int slots, int tab) {
        size_t o = 0;
        const int NS = K + 1, nchD = D >> 6, nchF = F >> 6;
        bars = p_take(o, 128);
        ring = p_take(o, (size_t)slots * slot_bytes);
        // xn (until routing is decided) and the h digit planes (after that)
        // are never live together.
        const size_t hpl = (size_t)NS * nchF * kChunkBytes;
        xs = p_take(o, hpl > (size_t)D * 4 ? hpl : (size_t)D * 4);
        ph = xs;
        px = p_take(o, (size_t)nchD * kChunkBytes);
        tx = p_take(o, (size_t)nchD * tab * 4);
        gx = p_take(o, (size_t)(D >> 5) * 4);
        th = p_take(o, (size_t)NS * nchF * tab * 4);
        gh = p_take(o, (size_t)NS * (F >> 5) * 4);
        part = p_take(o, (size_t)slots * 2 * kPGroupWarps * kPTile * 4);
        ys = p_take(o, (size_t)NS * kPTile * 4);
        bias = p_take(o, (size_t)E * 4);
        cen = p_take(o, (size_t)E * 8);
        bnd = p_take(o, (size_t)E * 8);
        sel = p_take(o, (size_t)E * 20);
        rscr = p_take(o, (size_t)(64 + 5 * kPMaxCons) * 4);
        misc = p_take(o, 512);
        total = o;
    }
};

// Ring slot: the largest of a gate/up tile (16 rows of D), a down tile (16
// rows of F) and the layer constants (norm + bias); weights plus their
// gs-group scales (4 bytes per gs weights).
__host__ __device__ inline int p_slot_bytes(int D, int F, int E, int gs) {
    int b = kPTile * (D + 4 * D / gs);
    const int bf = kPTile * (F + 4 * F / gs);
    if (bf > b) b = bf;
    if (D * 4 + E * 4 > b) b = D * 4 + E * 4;
    return (b + 127) & ~127;
}

// ------------------------------------------------------------ primitives

// Barrier 1 among the kN consumer threads (the producer warp never joins it).
template <int kN>
__device__ __forceinline__ void cons_sync() {
    asm volatile("bar.sync 1, %0;\n" ::"n"(kN) : "memory");
}

__device__ __forceinline__ unsigned ld_acquire_gpu(const unsigned* p) {
    unsigned v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];\n" : "=r"(v) : "l"(p) : "memory");
    return v;
}

__device__ __forceinline__ void red_release_gpu_add(unsigned* p, unsigned v) {
    asm volatile("red.release.gpu.global.add.u32 [%0], %1;\n" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ unsigned ld_relaxed_gpu(const unsigned* p) {
    unsigned v;
    asm volatile("ld.relaxed.gpu.global.u32 %0, [%1];\n" : "=r"(v) : "l"(p) : "memory");
    return v;
}

// ------------------------------------------------------------ row mapping

// This CTA's rows: shared gate/up rows [sh0, sh0+nsh), routed gate/up rows
// [rt0, rt0+nrt) of the slot-major K*F routed h, output rows [rb, re).
struct PRows {
    int sh0, nsh, rt0, nrt, rb, re;
    __device__ PRows(int c, int G, int D, int F, int K) {
        sh0 = (int)((long long)c * F / G);
        nsh = (int)((long long)(c + 1) * F / G) - sh0;
        rt0 = (int)((long long)c * K * F / G);
        nrt = (int)((long long)(c + 1) * K * F / G) - rt0;
        rb = (int)((long long)c * D / G);
        re = (int)((long long)(c + 1) * D / G);
    }
    __device__ int n_sh_items() const { return (nsh + kPHRows - 1) / kPHRows; }
    __device__ int n_rt_items() const { return (nrt + kPHRows - 1) / kPHRows; }
};

struct GRow {
    const int8_t* q = nullptr;  // null: row absent (zero contribution)
    const float* s = nullptr;
    int hidx = -1;              // index into h, -1 past the end of the tile
};

// Row j (0-15) of gate/up item t: rows 0-7 are the gate rows of this CTA's
// h entries 8t .. 8t+7 (shared rows, or routed rows once `topk` is known),
// rows 8-15 their up rows, so one MMA tile yields gate and up of an h entry
// in the same lane.
__device__ __forceinline__ GRow gate_row(const MoeLayerDev& W, const PersistArgs& a, const PRows& m, bool routed,
                                         int t, int j, const int* topk) {
    GRow r;
    const size_t D = (size_t)a.D, sgrp = D / a.gs;
    const int i = t * kPHRows + (j & (kPHRows - 1)), mat = j >= kPHRows;
    if (!routed) {
        if (i >= m.nsh) return r;
        const int rr = m.sh0 + i;
        r.hidx = a.K * a.F + rr;
        r.q = (mat ? W.up_sh_q : W.gate_sh_q) + (size_t)rr * D;
        r.s = (mat ? W.up_sh_s : W.gate_sh_s) + (size_t)rr * sgrp;
        return r;
    }
    if (i >= m.nrt) return r;
    const int flat = m.rt0 + i, slot = flat / a.F, rr = flat - slot * a.F;
    r.hidx = flat;
    if (!a.routed_enabled || !W.gate_q || !topk) return r;
    const int e = topk[slot];
    if (e < 0) return r;
    const size_t row = (size_t)e * a.F + rr;
    r.q = (mat ? W.up_q : W.gate_q) + row * D;
    r.s = (mat ? W.up_s : W.gate_s) + row * sgrp;
    return r;
}

// ------------------------------------------------------------ producer

// Producer lanes: gate/up item t into `buf`: each maximal run of rows with
// contiguous sources is one q copy and one s copy.
__device__ void produce_gate_item(const MoeLayerDev& W, const PersistArgs& a, const PRows& m, bool routed, int t,
                                  const int* topk, unsigned char* buf, uint64_t* bar) {
    const unsigned full = 0xffffffffu;
    const int lane = threadIdx.x & 31;
    const size_t D = (size_t)a.D, sgrp = D / a.gs, sbytes = D / a.sdiv;
    GRow r;
    if (lane < kPTile) r = gate_row(W, a, m, routed, t, lane, topk);
    const bool take = lane < kPTile && r.q != nullptr;
    const unsigned tmask = __ballot_sync(full, take);
    const auto pq = reinterpret_cast<const int8_t*>(__shfl_up_sync(full, reinterpret_cast<unsigned long long>(r.q), 1));
    const auto ps = reinterpret_cast<const float*>(__shfl_up_sync(full, reinterpret_cast<unsigned long long>(r.s), 1));
    const bool cont = take && lane > 0 && ((tmask >> (lane - 1)) & 1u) && pq + D == r.q && ps + sgrp == r.s;
    const unsigned cmask = __ballot_sync(full, cont);
    const uint32_t bytes = (uint32_t)__popc(tmask) * (uint32_t)(D + sbytes);
    if (lane == 0) {
        if (bytes)
            mbar_arrive_expect_tx(bar, bytes);
        else
            mbar_arrive(bar);
    }
    __syncwarp();
    if (take && !cont) {
        // run length: this lane plus the following lanes that continue it
        const int n = __ffs(~(cmask >> (lane + 1)));
        bulk_copy_g2s(buf + (size_t)lane * D, r.q, (uint32_t)(n * D), bar);
        bulk_copy_g2s(buf + kPTile * D + (size_t)lane * sbytes, r.s, (uint32_t)(n * sbytes), bar);
    }
}

// Producer lanes: this CTA's output rows of down matrix `slot` (K = shared).
__device__ void produce_down(const MoeLayerDev& W, const PersistArgs& a, const PRows& m, int slot, const int* topk,
                             unsigned char* buf, uint64_t* bar) {
    const int lane = threadIdx.x & 31;
    const int n = m.re - m.rb;
    const size_t F = (size_t)a.F, fgrp = F / a.gs, sbytes = F / a.sdiv;
    const int8_t* q = nullptr;
    const float* s = nullptr;
    if (n > 0) {
        if (slot == a.K) {
            q = W.down_sh_q + (size_t)m.rb * F;
            s = W.down_sh_s + (size_t)m.rb * fgrp;
        } else if (a.routed_enabled && W.down_q && topk[slot] >= 0) {
            const size_t row = (size_t)topk[slot] * a.D + m.rb;
            q = W.down_q + row * F;
            s = W.down_s + row * fgrp;
        }
    }
    if (lane == 0) {
        if (q) {
            mbar_arrive_expect_tx(bar, (uint32_t)(n * (F + sbytes)));
            bulk_copy_g2s(buf, q, (uint32_t)(n * F), bar);
            bulk_copy_g2s(buf + kPTile * F, s, (uint32_t)(n * sbytes), bar);
        } else {
            mbar_arrive(bar);
        }
    }
    __syncwarp();
}

// L2 prefetch of [p, p + bytes) (16-byte aligned, multiple of 16): the
// weights then stream from HBM at full rate while the ring, which holds only
// a few tiles, is refilled from L2.
__device__ __forceinline__ void prefetch_l2(const void* p, uint32_t bytes) {
    if (p && bytes) asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;\n" ::"l"(p), "r"(bytes) : "memory");
}

// Producer lanes: this CTA's routed gate and up rows of layer W (expert ids
// in topk) into L2, one range per lane.
__device__ void prefetch_routed_gate_up(const MoeLayerDev& W, const PersistArgs& a, const PRows& m, const int* topk) {
    const int lane = threadIdx.x & 31;
    if (!a.routed_enabled || !W.gate_q || m.nrt <= 0) return;
    const size_t D = (size_t)a.D, F = (size_t)a.F;
    // routed rows [rt0, rt0 + nrt) span at most a few slots
    const int s_first = m.rt0 / a.F, s_last = (m.rt0 + m.nrt - 1) / a.F;
    for (int sl = s_first; sl <= s_last; ++sl) {
        const int e = topk[sl];
        if (e < 0) continue;
        const int r0 = (m.rt0 > sl * a.F ? m.rt0 : sl * a.F) - sl * a.F;
        const int r1 = (m.rt0 + m.nrt < (sl + 1) * a.F ? m.rt0 + m.nrt : (sl + 1) * a.F) - sl * a.F;
        const size_t row = (size_t)e * F + r0, n = (size_t)(r1 - r0);
        const int base = 4 * (sl - s_first);
        if (lane == base) prefetch_l2(W.gate_q + row * D, (uint32_t)(n * D));
        if (lane == base + 1) prefetch_l2(W.gate_s + row * (D / a.gs), (uint32_t)(n * (D / a.sdiv)));
        if (lane == base + 2) prefetch_l2(W.up_q + row * D, (uint32_t)(n * D));
        if (lane == base + 3) prefetch_l2(W.up_s + row * (D / a.gs), (uint32_t)(n * (D / a.sdiv)));
    }
}

// Producer lanes: this CTA's output rows of the K routed down matrices into L2.
__device__ void prefetch_routed_down(const MoeLayerDev& W, const PersistArgs& a, const PRows& m, const int* topk) {
    const int lane = threadIdx.x & 31;
    const int n = m.re - m.rb;
    if (!a.routed_enabled || !W.down_q || n <= 0 || lane >= 2 * a.K) return;
    const size_t D = (size_t)a.D, F = (size_t)a.F;
    const int e = topk[lane >> 1];
    if (e < 0) return;
    const size_t row = (size_t)e * D + m.rb;
    if ((lane & 1) == 0)
        prefetch_l2(W.down_q + row * F, (uint32_t)(n * F));
    else
        prefetch_l2(W.down_s + row * (F / a.gs), (uint32_t)(n * (F / a.sdiv)));
}

// Producer lanes: the routing-independent weights this CTA needs of layer W
// (router row, shared expert rows, norm and bias) into L2.
__device__ void prefetch_shared(const MoeLayerDev& W, const PersistArgs& a, const PRows& m, int c) {
    const int lane = threadIdx.x & 31;
    const size_t D = (size_t)a.D, F = (size_t)a.F;
    const int n = m.re - m.rb;
    // (a table entry whose weights are absent has null pointers: skip those)
    switch (lane) {
        case 0: if (W.router && c < a.E) prefetch_l2(W.router + (size_t)c * D, (uint32_t)(D * 4)); break;
        case 1: if (W.gate_sh_q && m.nsh > 0) prefetch_l2(W.gate_sh_q + (size_t)m.sh0 * D, (uint32_t)(m.nsh * D)); break;
        case 2: if (W.gate_sh_s && m.nsh > 0) prefetch_l2(W.gate_sh_s + (size_t)m.sh0 * (D / a.gs), (uint32_t)(m.nsh * (D / a.sdiv))); break;
        case 3: if (W.up_sh_q && m.nsh > 0) prefetch_l2(W.up_sh_q + (size_t)m.sh0 * D, (uint32_t)(m.nsh * D)); break;
        case 4: if (W.up_sh_s && m.nsh > 0) prefetch_l2(W.up_sh_s + (size_t)m.sh0 * (D / a.gs), (uint32_t)(m.nsh * (D / a.sdiv))); break;
        case 5: if (W.down_sh_q && n > 0) prefetch_l2(W.down_sh_q + (size_t)m.rb * F, (uint32_t)(n * F)); break;
        case 6: if (W.down_sh_s && n > 0) prefetch_l2(W.down_sh_s + (size_t)m.rb * (F / a.gs), (uint32_t)(n * (F / a.sdiv))); break;
        case 7: if (c == 0) prefetch_l2(W.ffn_norm, (uint32_t)(D * 4)); break;
        case 8: if (c == 0) prefetch_l2(W.router_bias, (uint32_t)(a.E * 4)); break;
        default: break;
    }
}

// ------------------------------------------------------------ consumers

struct PCtx {
    unsigned char* ring;
    uint64_t* full;
    uint64_t* empty;
    int slot_bytes;
    int slots;
    volatile int* abort_flag;
    unsigned* status;
};

__device__ __forceinline__ unsigned char* slot_buf(const PCtx& P, uint32_t it) {
    return P.ring + (size_t)(it % P.slots) * P.slot_bytes;
}

// Every consumer thread waits for ring item `it` itself. A wait that gives up
// records why and raises the CTA's abort flag; the thread then carries on
// with whatever the slot holds (no block-wide agreement per item), and the
// CTA leaves at its next grid barrier, which checks the flag.
__device__ __forceinline__ void cons_wait(const PCtx& P, uint32_t it) {
    if (!mbar_wait_bounded(&P.full[it % P.slots], (it / P.slots) & 1u)) {
        atomicOr(P.status, kStatFull);
        *P.abort_flag = 1;
    }
}

// A consumer warp of the slot's group is done reading item `it`: one arrival
// per warp hands the slot back once the group's kPGroupWarps warps are done.
__device__ __forceinline__ void cons_release(const PCtx& P, uint32_t it) {
    __syncwarp();
    if ((threadIdx.x & 31) == 0) mbar_arrive(&P.empty[it % P.slots]);
}

// Thread 0: wait until the arrival count reaches target (acquire), polling
// 32 times between looks at the clock, the abort flag and the status word.
__device__ __forceinline__ int poll_barrier(const PersistArgs& a, const PCtx& P, unsigned target) {
    const uint64_t t0 = global_ns();
    for (uint32_t i = 0; !*P.abort_flag && global_ns() - t0 < kWaitNs; ++i) {
#pragma unroll 1
        for (int j = 0; j < 32; ++j)
            if (ld_acquire_gpu(a.bar) >= target) return 1;
        if ((i & 7u) == 7u && (ld_relaxed_gpu(a.status) & kStatAbort)) break;
    }
    atomicOr(a.status, kStatBarrier);
    *P.abort_flag = 1;
    return 0;
}

// Grid-wide barrier among the consumer warps of all CTAs; false when this
// CTA or another one has given up (every CTA then leaves).
template <int kN>
__device__ bool grid_sync(const PersistArgs& a, const PCtx& P, unsigned& nbar, int tid, volatile int* s_ok) {
    cons_sync<kN>();
    ++nbar;
    if (tid == 0) {
        if (!*P.abort_flag) red_release_gpu_add(a.bar, 1u);
        const int ok = poll_barrier(a, P, nbar * gridDim.x);
        *s_ok = ok;
    }
    cons_sync<kN>();
    return *s_ok != 0;
}

// grid_sync in two halves: grid_arrive (after this CTA's writes) and
// grid_wait (before reading the other CTAs'), with work in between.
template <int kN>
__device__ void grid_arrive(const PersistArgs& a, const PCtx& P, unsigned& nbar, int tid) {
    cons_sync<kN>();
    ++nbar;
    if (tid == 0 && !*P.abort_flag) red_release_gpu_add(a.bar, 1u);
}

template <int kN>
__device__ bool grid_wait(const PersistArgs& a, const PCtx& P, unsigned nbar, int tid, volatile int* s_ok) {
    cons_sync<kN>();
    if (tid == 0) *s_ok = poll_barrier(a, P, nbar * gridDim.x);
    cons_sync<kN>();
    return *s_ok != 0;
}

__device__ __forceinline__ float silu_p(float v) { return v / (1.0f + expf(-v)); }

template <int kGS>
__global__ void __launch_bounds__(PCfg<kGS>::kThreads, 1) moe_persistent_kernel(PersistArgs a) {
    using Cfg = PCfg<kGS>;
    constexpr int kPSlots = Cfg::kSlots, kPCons = Cfg::kCons, kPConsThreads = Cfg::kConsThreads, kTab = Cfg::kTab;
    auto cons_sync = []() { glmq::cons_sync<kPConsThreads>(); };
    extern __shared__ __align__(128) unsigned char sm[];
    const int D = a.D, F = a.F, E = a.E, K = a.K;
    const int nchF = F >> 6;
    const PSmem L(D, F, E, K, a.slot_bytes, kPSlots, kTab);
    uint64_t* full = reinterpret_cast<uint64_t*>(sm + L.bars);
    uint64_t* empty = full + kPSlots;
    uint64_t* route_ready = empty + kPSlots;
    float* xs = reinterpret_cast<float*>(sm + L.xs);
    int8_t* ph = reinterpret_cast<int8_t*>(sm + L.ph);
    int8_t* px = reinterpret_cast<int8_t*>(sm + L.px);
    float* tx = reinterpret_cast<float*>(sm + L.tx);
    float* gx = reinterpret_cast<float*>(sm + L.gx);
    float* th = reinterpret_cast<float*>(sm + L.th);
    float* gh = reinterpret_cast<float*>(sm + L.gh);
    float* part = reinterpret_cast<float*>(sm + L.part);
    float* ys = reinterpret_cast<float*>(sm + L.ys);
    float* s_bias = reinterpret_cast<float*>(sm + L.bias);
    double* s_cen = reinterpret_cast<double*>(sm + L.cen);
    double* s_bnd = reinterpret_cast<double*>(sm + L.bnd);
    float* rscr = reinterpret_cast<float*>(sm + L.rscr);
    int* misc = reinterpret_cast<int*>(sm + L.misc);
    int* s_rank = misc;                                   // [kMaxTopK + 1]
    int* s_cert = misc + 16;
    int* s_topk = misc + 32;                              // [kMaxTopK]
    float* s_topw = reinterpret_cast<float*>(misc + 48);  // [kMaxTopK]
    float* s_inv = reinterpret_cast<float*>(misc + 64);
    volatile int* s_ok = misc + 65;
    volatile int* s_abort = misc + 66;
    double* red = reinterpret_cast<double*>(misc + 72);   // [kPCons] (<= kPMaxCons)
    SelectScratch S;
    S.sel_c = reinterpret_cast<float*>(sm + L.sel);
    S.sel_lo = S.sel_c + E;
    S.sel_hi = S.sel_lo + E;
    S.p_c = S.sel_hi + E;
    S.taken = reinterpret_cast<int*>(S.p_c + E);
    S.rank = s_rank;
    S.cert = s_cert;

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int c = blockIdx.x, G = gridDim.x;
    const PRows m(c, G, D, F, K);
    const PCtx P{sm + L.ring, full, empty, a.slot_bytes, kPSlots, s_abort, a.status};

    if (tid == 0) {
        for (int i = 0; i < kPSlots; ++i) {
            mbar_init(&full[i], 1);
            mbar_init(&empty[i], kPGroupWarps);
        }
        mbar_init(route_ready, 1);
        *s_abort = 0;
        mbar_init_fence();
        // the next launch on this stream may start as SMs free up; it waits
        // (griddepcontrol.wait) for this grid's completion before it reads x
        asm volatile("griddepcontrol.launch_dependents;\n" ::: "memory");
    }
    __syncthreads();

    // ------------------------------------------------------------- producer
    if (warp == kPCons) {
        uint32_t it = 0;
        // Lane 0 waits (the hardware suspends it until the phase completes);
        // gives up after kWaitNs or when the consumers abort.
        auto wait_phase = [&](uint64_t* bar, uint32_t parity) -> bool {
            bool ok = false;
            if (lane == 0) {
                ok = mbar_try_wait(bar, parity);
                const uint64_t t0 = global_ns();
                while (!ok && !*s_abort && global_ns() - t0 < kWaitNs)
                    ok = mbar_try_wait_sleep(bar, parity, kSuspendNs);
            }
            return __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
        };
        // Ring slot of item i is free (its previous item was released) and
        // at most kPInflight items are in flight.
        auto acquire = [&](uint32_t i) -> bool {
            if (i >= (uint32_t)kPSlots && !wait_phase(&empty[i % kPSlots], ((i / kPSlots) - 1) & 1u)) return false;
            if (kPInflight < kPSlots && i >= (uint32_t)kPInflight) {
                const uint32_t j = i - kPInflight;
                if (!wait_phase(&full[j % kPSlots], (j / kPSlots) & 1u)) return false;
            }
            return true;
        };
        bool alive = true;
        for (int li = 0; li < a.n_layers && alive; ++li) {
            const MoeLayerDev W = a.layers[a.first + li];
            // layer constants: ffn_norm and the router bias
            if (!(alive = acquire(it))) break;
            if (lane == 0) {
                uint64_t* bar = &full[it % kPSlots];
                unsigned char* buf = slot_buf(P, it);
                mbar_arrive_expect_tx(bar, (uint32_t)(D * 4 + E * 4));
                bulk_copy_g2s(buf, W.ffn_norm, (uint32_t)(D * 4), bar);
                bulk_copy_g2s(buf + D * 4, W.router_bias, (uint32_t)(E * 4), bar);
            }
            __syncwarp();
            ++it;
            if (c < E) {  // this CTA's router row
                if (!(alive = acquire(it))) break;
                if (lane == 0) {
                    uint64_t* bar = &full[it % kPSlots];
                    mbar_arrive_expect_tx(bar, (uint32_t)(D * 4));
                    bulk_copy_g2s(slot_buf(P, it), W.router + (size_t)c * D, (uint32_t)(D * 4), bar);
                }
                __syncwarp();
                ++it;
            }
            for (int t = 0; t < m.n_sh_items() && alive; ++t) {
                if (!(alive = acquire(it))) break;
                produce_gate_item(W, a, m, false, t, nullptr, slot_buf(P, it), &full[it % kPSlots]);
                ++it;
            }
            if (!alive) break;
            // While this layer's routing is decided HBM is nearly idle: pull
            // the next layer's routing-independent weights into L2.
            const int nl = li + 1 < a.n_layers ? a.first + li + 1 : a.next_layer;
            if (nl >= 0) prefetch_shared(a.layers[nl], a, m, c);
            // routed rows need this layer's expert ids
            if (!(alive = wait_phase(route_ready, (uint32_t)li & 1u))) {
                if (lane == 0) atomicOr(a.status, kStatRoute);
                break;
            }
            // The first routed items go out first; then the CTA's remaining
            // routed gate/up rows go to L2 at once (HBM at full rate) and the
            // ring refills from L2; the down rows follow once every gate/up
            // item is issued, so they do not slow the gate/up stream.
            const int ngate = m.n_rt_items();
            for (int t = 0; t < ngate && alive; ++t) {
                if (t == 3) prefetch_routed_gate_up(W, a, m, s_topk);
                if (!(alive = acquire(it))) break;
                produce_gate_item(W, a, m, true, t, s_topk, slot_buf(P, it), &full[it % kPSlots]);
                ++it;
            }
            if (!alive) break;
            prefetch_routed_down(W, a, m, s_topk);
            // down rows: shared expert first, then the routed slots in rank order
            for (int q = 0; q <= K && alive; ++q) {
                if (!(alive = acquire(it))) break;
                produce_down(W, a, m, q == 0 ? K : q - 1, s_topk, slot_buf(P, it), &full[it % kPSlots]);
                ++it;
            }
        }
        if (!alive) {
            if (lane == 0) {
                atomicOr(a.status, kStatEmpty);
                *s_abort = 1;
            }
            // let copies still in flight land before the CTA can exit
            for (uint32_t j = (it > (uint32_t)kPSlots ? it - kPSlots : 0u); j < it; ++j)
                mbar_wait_bounded(&full[j % kPSlots], (j / kPSlots) & 1u);
        }
        return;
    }

    // ------------------------------------------------------------ consumers
    const int gid = lane >> 2, t4 = lane & 3;
    const int grp = warp / kPGroupWarps, gw = warp % kPGroupWarps;
    const int boff = b_frag_offset(lane);
    const G16Lane gl = g16_lane(lane);
    const int4 z4 = make_int4(0, 0, 0, 0);
    const float2 z2 = make_float2(0.f, 0.f);
    constexpr int kPart = kPGroupWarps * kPTile;
    float* gpart = part + (size_t)grp * 2 * kPart;  // this group's two partial buffers
    uint32_t it = 0;
    unsigned nbar = 0;
    int nlocal = 0;  // items this group has processed (parity picks the partial buffer)
    auto sync = []() { glmq::cons_sync<kPConsThreads>(); };
    auto grp_sync = [&]() { asm volatile("bar.sync %0, %1;\n" ::"r"(2 + grp), "n"(kPGroupWarps * 32) : "memory"); };

    // Items that every consumer reads (layer constants, router row): after
    // a block barrier the slot's group hands the slot back.
    auto release_shared_item = [&](uint32_t item) {
        if (grp == (int)(item % kPSlots)) cons_release(P, item);
    };

    // A weight item is processed by the group that owns its ring slot: each
    // of the group's warps dots its third of the 64-column chunks of the 16
    // rows with the activation planes and hands the slot back; after the
    // group barrier one warp adds the three partials of every row. tab: the
    // planes' epilogue table (gs = 32) or x-group scales (gs = 16).
    auto group_rows = [&](uint32_t item, const int8_t* planes, const float* tab, int cols, bool v0, bool v1) {
        cons_wait(P, item);
        const int nch = cols >> 6;
        const int8_t* qb = reinterpret_cast<const int8_t*>(slot_buf(P, item));
        const unsigned char* sb = slot_buf(P, item) + kPTile * cols;
        const int srow = cols * 4 / kGS;  // scale bytes per row
        float acc0 = 0.f, acc1 = 0.f;
#pragma unroll(kGS == 32 ? 2 : 1)
        for (int j = gw * nch / kPGroupWarps; j < (gw + 1) * nch / kPGroupWarps; ++j) {
            const int off = j * kChunkCols + 16 * t4;
            const int4 q0 = v0 ? lds16(qb + gid * cols + off) : z4;
            const int4 q1 = v1 ? lds16(qb + (gid + 8) * cols + off) : z4;
            if constexpr (kGS == 32) {
                const int4 b4 = boff >= 0 ? lds16(planes + j * kChunkBytes + boff) : z4;
                const float2 tb = *reinterpret_cast<const float2*>(tab + j * kTab + 2 * t4);
                const float2 s0 = v0 ? *reinterpret_cast<const float2*>(sb + gid * srow + 8 * j) : z2;
                const float2 s1 = v1 ? *reinterpret_cast<const float2*>(sb + (gid + 8) * srow + 8 * j) : z2;
                chunk_mma_accumulate(q0, q1, s0, s1, b4, tb, t4, acc0, acc1);
            } else {  // tab: the x-group scales
                const int8_t* pl = planes + j * kChunkBytes;
                const int4 bx = gl.offX >= 0 ? lds16(pl + gl.offX) : z4;
                const int4 by = gl.offY >= 0 ? lds16(pl + gl.offY) : z4;
                const float sx = tab[2 * j + (t4 >> 1)];
                const float s0 = v0 ? *reinterpret_cast<const float*>(sb + gid * srow + 16 * j + 4 * t4) : 0.f;
                const float s1 = v1 ? *reinterpret_cast<const float*>(sb + (gid + 8) * srow + 16 * j + 4 * t4) : 0.f;
                chunk_mma_accumulate_g16(q0, q1, s0, s1, bx, by, sx, acc0, acc1);
            }
        }
        cons_release(P, item);
        acc0 = quad_sum(acc0);
        acc1 = quad_sum(acc1);
        float* pt = gpart + (nlocal & 1) * kPart;
        if (t4 == 0) {
            pt[gw * kPTile + gid] = acc0;
            pt[gw * kPTile + gid + 8] = acc1;
        }
        ++nlocal;
        grp_sync();
        return static_cast<const float*>(pt);
    };
    auto row_total = [&](const float* pt, int r) {
        float tot = 0.f;
#pragma unroll
        for (int w = 0; w < kPGroupWarps; ++w) tot += pt[w * kPTile + r];
        return tot;
    };

    // Gate/up item t -> 8 entries of h, h = silu(gate) * up
    // (infer.c:1184-1188, 1197-1201).
    auto gate_item = [&](const MoeLayerDev& W, bool routed, int t, uint32_t item) {
        const int* tk = routed ? s_topk : nullptr;
        const float* pt = group_rows(item, px, kGS == 32 ? tx : gx, D, gate_row(W, a, m, routed, t, gid, tk).q != nullptr,
                                     gate_row(W, a, m, routed, t, gid + 8, tk).q != nullptr);
        if (gw == 0 && lane < kPHRows) {
            const int hidx = gate_row(W, a, m, routed, t, lane, tk).hidx;
            if (hidx >= 0) a.h[hidx] = silu_p(row_total(pt, lane)) * row_total(pt, lane + kPHRows);
        }
    };

    // This CTA's output rows of down matrix `slot` (K = shared) -> ys[slot]:
    // the group quantises that slot's h itself (its group barrier, no block
    // barrier), then dots the down tile with it.
    auto down_item = [&](const MoeLayerDev& W, int slot, uint32_t item) {
        const int n = m.re - m.rb;
        const bool live = slot == K || (a.routed_enabled && W.down_q && s_topk[slot] >= 0);
        int8_t* pl = ph + (size_t)slot * nchF * kChunkBytes;
        float* sg = gh + (size_t)slot * (F >> 5);
        float* tb = th + (size_t)slot * nchF * kTab;
        quantize_planes_part<true, kGS == 16>(a.h + (size_t)slot * F, F, pl, sg, tb, gw * 32 + lane,
                                              kPGroupWarps * 32, grp_sync);
        const float* pt = group_rows(item, pl, kGS == 32 ? tb : sg, F, live && gid < n, live && gid + 8 < n);
        if (gw == 0 && lane < kPTile) ys[slot * kPTile + lane] = row_total(pt, lane);
    };

    // First item index >= from that belongs to this group.
    auto first_mine = [&](uint32_t from) { return from + (uint32_t)((grp - (int)(from % kPSlots) + kPSlots) % kPSlots); };

    // x, the barrier words and the scratch may still be in use by the previous
    // launch on this stream (programmatic dependent launch): wait for it.
    asm volatile("griddepcontrol.wait;\n" ::: "memory");
    // Every consumer exit goes through here: the last CTA to leave resets the
    // barrier words for the next launch (no memset between launches).
    auto leave = [&]() {
        if (tid == 0) {
            // every CTA counted here has passed its last grid barrier: the
            // last one resets the words (the next launch reads them only
            // after this grid has completed)
            unsigned prev;
            asm volatile("atom.add.acq_rel.gpu.global.u32 %0, [%1], 1;\n" : "=r"(prev) : "l"(a.done) : "memory");
            if (prev == (unsigned)G - 1u) {
                *reinterpret_cast<volatile unsigned*>(a.bar) = 0u;
                *reinterpret_cast<volatile unsigned*>(a.done) = 0u;
            }
        }
    };

    for (int li = 0; li < a.n_layers; ++li) {
        const MoeLayerDev W = a.layers[a.first + li];

        // ---- P0: rmsnorm (infer.c:746-752, 1098), every CTA; xn -> planes
        cons_wait(P, it);
        {
            const float* norm = reinterpret_cast<const float*>(slot_buf(P, it));
            for (int i = tid; i < E; i += kPConsThreads) s_bias[i] = norm[D + i];
            constexpr int kXPer = (2048 + kPConsThreads - 1) / kPConsThreads;  // D <= 2048
            float xr[kXPer];
#pragma unroll
            for (int u = 0; u < kXPer; ++u)
                xr[u] = tid + u * kPConsThreads < D ? ldcg_f32(a.x + tid + u * kPConsThreads) : 0.0f;
            double ss = 0.0;
#pragma unroll
            for (int u = 0; u < kXPer; ++u) {
                const double v = (double)xr[u];
                ss = __dadd_rn(ss, __dmul_rn(v, v));
            }
            ss = warp_sum_d(ss);
            if (lane == 0) red[warp] = ss;
            cons_sync();
            if (tid == 0) {
                double tot = 0.0;
                for (int w = 0; w < kPCons; ++w) tot += red[w];
                float mean;
                *s_inv = rms_mean_certify(tot, D, mean) ? rms_inv_of_mean(mean) : __int_as_float(0x7fc00000);
            }
            cons_sync();
            if (isnan(*s_inv)) {
                // not certified (or non-finite x): glm.c's serial fp64 sum, over x
                // staged in shared memory instead of one L2 round trip per element
#pragma unroll
                for (int u = 0; u < kXPer; ++u)
                    if (tid + u * kPConsThreads < D) xs[tid + u * kPConsThreads] = xr[u];
                cons_sync();
                if (tid == 0) {
                    double seq = 0.0;
                    for (int i = 0; i < D; ++i) {
                        const double v = (double)xs[i];
                        seq = __dadd_rn(seq, __dmul_rn(v, v));
                    }
                    *s_inv = rms_inv_of_mean((float)(seq / (double)D));
                    if (c == 0) atomicAdd(&a.stats[3], 1ull);
                }
                cons_sync();
            }
            const float inv = *s_inv;
#pragma unroll
            for (int u = 0; u < kXPer; ++u) {
                const int i = tid + u * kPConsThreads;
                if (i < D) xs[i] = __fmul_rn(__fmul_rn(xr[u], inv), norm[i]);
            }
        }
        cons_sync();  // xs complete before any thread quantises it; the constants are read
        release_shared_item(it);
        ++it;

        // ---- P1: router logit of expert c (CTAs c < E)
        if (c < E) {
            cons_wait(P, it);
            double C = 0.0, B = 0.0;
            block_logit_bound_rows<(64 + kPCons - 1) / kPCons>(reinterpret_cast<const float*>(slot_buf(P, it)), xs, D,
                                                               tid, kPConsThreads, rscr, sync, C, B);
            release_shared_item(it);  // the row was read before the function's first barrier
            ++it;
            if (tid == 0) {
                __stcg(a.center + c, C);
                __stcg(a.bound + c, B);
            }
        }
        // arrive as soon as this CTA's router results are out, then turn xn
        // into digit planes for the gate/up products while the other CTAs'
        // results come in, then wait
        grid_arrive<kPConsThreads>(a, P, nbar, tid);
        quantize_planes_part<false, kGS == 16>(xs, D, px, gx, tx, tid, kPConsThreads, sync);
        if (!grid_wait<kPConsThreads>(a, P, nbar, tid, s_ok)) return leave();

        // ---- P2: routing (every CTA, identical); shared and routed gate/up
        for (int i = tid; i < E; i += kPConsThreads) {
            s_cen[i] = ldcg_f64(a.center + i);
            s_bnd[i] = ldcg_f64(a.bound + i);
        }
        cons_sync();
        block_select(s_cen, s_bnd, s_bias, E, K, W.router, xs, D, tid, kPConsThreads, S, s_topk, s_topw,
                     c == 0 ? a.stats : nullptr, sync);
        if (tid == 0) mbar_arrive(route_ready);  // the producer may fetch routed rows now
        if (c == 0 && tid < K) {
            if (a.topk_out) a.topk_out[li * K + tid] = s_topk[tid];
            if (a.topkw_out) a.topkw_out[li * K + tid] = s_topw[tid];
        }
        // Every group takes the items in its ring slot; the shared items are
        // already in the ring and fill the wait for the first routed rows.
        const int nsh = m.n_sh_items(), nitems = nsh + m.n_rt_items();
        for (uint32_t item = first_mine(it); item < it + (uint32_t)nitems; item += kPSlots) {
            const int u = (int)(item - it);
            gate_item(W, u >= nsh, u >= nsh ? u - nsh : u, item);
        }
        it += (uint32_t)nitems;
        if (!grid_sync<kPConsThreads>(a, P, nbar, tid, s_ok)) return leave();

        // ---- P3: down rows (each group quantises its slots' h: xs is dead); combine
        // down items in the order shared, routed 0 .. K-1; each group takes its own
        for (uint32_t item = first_mine(it); item < it + (uint32_t)(K + 1); item += kPSlots) {
            const int q = (int)(item - it);
            down_item(W, q == 0 ? K : q - 1, item);
        }
        it += (uint32_t)(K + 1);
        cons_sync();  // every group's ys written
        const int n = m.re - m.rb;
        if (tid < n) {
            // infer.c:1175,1192 then 1212-1214: acc += (1.8 w_k) y_k in rank
            // order, then x += y_shared + acc.
            const int r = m.rb + tid;
            float acc = 0.0f;
            for (int k = 0; k < K; ++k) {
                if (!a.routed_enabled || !W.down_q || s_topk[k] < 0) continue;
                acc = __fadd_rn(acc, __fmul_rn(__fmul_rn(s_topw[k], 1.8f), ys[k * kPTile + tid]));
            }
            a.x[r] = __fadd_rn(__ldcg(a.x + r), __fadd_rn(ys[K * kPTile + tid], acc));
        }
        if (li + 1 < a.n_layers && !grid_sync<kPConsThreads>(a, P, nbar, tid, s_ok)) return leave();
    }
    leave();
}

// ------------------------------------------------------------- launcher

cudaError_t persistent_check(const MoeDims& d, int num_sms, size_t* smem_out) {
    if (d.K < 1 || d.K > kMaxTopK || d.K > d.E || d.E > num_sms || d.E % 4 || (d.gs != 32 && d.gs != 16) ||
        d.D % 128 || d.D > 2048 || d.F % 128 || (d.D + kPTile - 1) / kPTile > num_sms)
        return cudaErrorInvalidValue;
    const int slot = p_slot_bytes(d.D, d.F, d.E, d.gs);
    const size_t smem = d.gs == 32 ? PSmem(d.D, d.F, d.E, d.K, slot, PCfg<32>::kSlots, PCfg<32>::kTab).total
                                   : PSmem(d.D, d.F, d.E, d.K, slot, PCfg<16>::kSlots, PCfg<16>::kTab).total;
    if (smem > 227 * 1024 - 1024) return cudaErrorInvalidValue;
    if (smem_out) *smem_out = smem;
    return cudaSuccess;
}

cudaError_t launch_moe_persistent(const MoeLayerDev* layers_dev, int first, int n_layers, const MoeDims& d,
                                  const MoeScratch& s, float* x, int32_t* topk_out, float* topkw_out,
                                  int routed_enabled, int num_sms, cudaStream_t stream, int next_layer) {
    size_t smem = 0;
    cudaError_t err = persistent_check(d, num_sms, &smem);
    if (err != cudaSuccess) return err;
    const bool g16 = d.gs == 16;
    auto kernel = g16 ? moe_persistent_kernel<16> : moe_persistent_kernel<32>;
    if ((err = ensure_smem_attr(reinterpret_cast<const void*>(kernel), (int)smem))) return err;
    PersistArgs a{layers_dev, first,    n_layers, x,           s.h,       s.center,
                  s.bound,    topk_out, topkw_out, s.grid_bar, s.grid_bar + 1, s.status, s.stats,
                  d.D,        d.F,      d.E,       d.K,        routed_enabled,
                  p_slot_bytes(d.D, d.F, d.E, d.gs), next_layer, d.gs, d.gs / 4,
                  g16 ? PCfg<16>::kSlots : PCfg<32>::kSlots};
    // The grid barriers need every CTA resident at once: one CTA per SM must
    // fit (checked here, as a cooperative launch would). The launch itself is
    // not cooperative: a plain programmatic dependent launch lets this grid's
    // CTAs start on the SMs that the previous kernel frees and stream their
    // first weight tiles while it drains (measured 1 us per layer faster than
    // the cooperative launch). Residency still holds: the previous kernel
    // never waits on this one, and the next kernel on the stream cannot start
    // before every CTA of this one has run its launch_dependents (the first
    // thing it does). A wait that still could not complete gives up after
    // kWaitNs and reports it in `status`.
    const int threads = g16 ? PCfg<16>::kThreads : PCfg<32>::kThreads;
    if ((err = ensure_resident(reinterpret_cast<const void*>(kernel), threads, (int)smem, num_sms))) return err;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(num_sms);
    cfg.blockDim = dim3(threads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kernel, a);
}

}  // namespace glmq
