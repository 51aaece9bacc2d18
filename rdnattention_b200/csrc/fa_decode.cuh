// Split-KV decode kernel (seq_len small: G * seq_len <= 64 query rows per KV
// head), FP16, HBM-bound.
//
// Work unit = (batch b, kv head). All G = H / Hkv query heads of the group
// and all seq_len query rows form the rows of the unit; each row group of 16
// is the M = 16 of one m16n8k16 tile, so every K/V byte read from HBM serves
// 16 rows (the reference re-reads K/V once per query head:
// src/rdna/fa2_forward_f16.hip:643-648).  Units with more than 16 rows have
// NRG = 2 or 4 row groups inside the CTA: warp w takes row group w % NRG, and
// each K/V tile is consumed by NRG warps (one per group), so the cache is
// still read once per unit.
//
// A cluster of CS CTAs (1..8) splits the unit's visible key range.  Per CTA:
//   warp 4       TMA producer: 32-key K and V tiles (strided [B, KS, Hkv, D]
//                caches included) through an NST-stage shared-memory ring;
//   warps 0..3   consumers, tile i -> warp i % 4: S = Q K^T and O += P V on
//                the tensor cores (mma.sync m16n8k16, fp32 accumulate) with
//                the online softmax in registers (quad shuffles).
// Partials (m, l, O) combine in shared memory across the 4 warps, then across
// the cluster over distributed shared memory; cluster rank 0 writes O.  No
// global scratch.  Masking (causal / both window forms / key tail) per
// element; rows with no visible key produce 0.
//
// The bound is HBM: per 32-key tile the warp moves 16 KB (D = 128) and
// issues 64 MMAs, far below the tensor and issue limits, so the mma.sync
// form costs nothing here while keeping the fragment-level softmax simple.
//
// RoPE (interleaved pairs, reference src/rdna/fa2_forward_f16.hip:63-77, Q
// row position = its index s within the sequence, K position = key index):
// Q is rotated as its fragments are loaded; each K tile is rotated in place in
// shared memory by one of NRW extra rotator warps (warps 5..8, tile i -> warp
// 5 + i % NRW; fp32 math, fp16 result), whose table loads for the tile are
// issued while its TMA is in flight; the consumers wait for the rotated tile.
// The KV cache is read once, as without RoPE; the cos/sin rows come from L2.
#pragma once

#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <math.h>

#include "rdna/forward.hpp"
#include "rope.cuh"
#include "sm100.cuh"

namespace rdna {
namespace decode {

using namespace sm100;

constexpr int KT = 32;         // keys per tile
constexpr int NCW = 4;         // consumer warps
// Ring stages.  Tile i lives in slot i % NST and is consumed by warp i % NCW;
// NST % NCW == 0 makes every slot's consumer the same warp, so no waiter can
// ever be more than one barrier phase ahead (parity waits cannot alias).
constexpr int NST = 8;
static_assert(NST % NCW == 0, "each ring slot needs a single consumer warp");
constexpr int NRW = 4;         // RoPE rotator warps (RoPE kernels only)
static_assert(NST % NRW == 0, "each ring slot needs a single rotator warp");
constexpr int THREADS = 32 * (NCW + 1);
constexpr int THREADS_ROPE = 32 * (NCW + 1 + NRW);
constexpr int MAX_ROWS = 16;   // rows per row group (one m16 tile)
constexpr int MAX_RG = 4;      // row groups per unit: G * seq_len <= 64
constexpr int MAX_CLUSTER = 8;

struct Params {
    const __half* q;
    __half* o;
    int64_t qsb, qsh, qss;
    int64_t osb, osh, oss;
    int B, H, Hkv, S, KS, G, R;  // R = G * S rows per unit
    int NRG;                     // row groups per unit: 1, 2 or 4 (divides the consumer warps)
    int delta;
    int causal;
    int window;
    float scale_log2;
    int rope;               // nonzero: rotate Q and K (tables [max(S, KS), D/2] fp32)
    const float* rope_cos;
    const float* rope_sin;
    int kv_bcast;  // K/V axes broadcast with stride 0 (prefill::KV_BCAST_* bits): coordinate 0
    // output replicas: n_peer other GPUs' counterparts of o (same strides, mapped
    // into this process), each written with the same 16-byte chunks as o (no
    // fence: the peers read them after this kernel has completed)
    int n_peer;
    __half* o_peer[7];
};

template <int D>
struct Layout {
    static constexpr int BOX = 64;  // fp16 elements per box row (128 B, SWIZZLE_128B)
    static constexpr int NBOX = D / BOX;
    static constexpr int BOX_BYTES = KT * 128;
    static constexpr int TILE = NBOX * BOX_BYTES;  // K or V tile
    static constexpr int STAGE = 2 * TILE;         // K then V
    static constexpr int OFF_RING = 1024;
    static constexpr int SMEM_BYTES = OFF_RING + NST * STAGE + 1024;  // + align slack
    // after the loop the ring is reused for partials
    static constexpr int WARP_PART = MAX_ROWS * (D + 2);              // floats per warp partial
    static_assert(NCW * WARP_PART * 4 + MAX_ROWS * MAX_RG * (D + 2) * 4 <= NST * STAGE, "partials fit in the ring");
};

// Byte offset of 16-byte chunk `c` (0..15 across boxes) of key row r in a tile.
template <int D>
__device__ __forceinline__ uint32_t tile_off(int r, int c) {
    const int box = c >> 3, cb = c & 7;
    return static_cast<uint32_t>(box * Layout<D>::BOX_BYTES + r * 128 + ((cb ^ (r & 7)) << 4));
}

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
                 : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
                 : "r"(addr));
}
__device__ __forceinline__ void mma16816(float* c, const uint32_t* a, uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
        "{%0, %1, %2, %3};"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

__device__ __forceinline__ uint32_t cluster_rank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}
__device__ __forceinline__ uint32_t cluster_size() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_nctarank;" : "=r"(r));
    return r;
}
// Cluster-wide barrier (non-.aligned form: callers reconverge their warp first
// anyway, but the barrier must not depend on it).
__device__ __forceinline__ void cluster_sync_all() {
    asm volatile("barrier.cluster.arrive.release;\n\tbarrier.cluster.wait.acquire;" ::: "memory");
}
__device__ __forceinline__ uint32_t map_to_rank(uint32_t saddr, uint32_t rank) {
    uint32_t r;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(saddr), "r"(rank));
    return r;
}
__device__ __forceinline__ float ld_dsmem(uint32_t addr) {
    float v;
    asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(v) : "r"(addr) : "memory");
    return v;
}

// Visible keys of decode row r (query position s = r % S): [lo, hi].
__device__ __forceinline__ void row_range(const Params& p, int s, int& lo, int& hi) {
    lo = 0;
    hi = p.KS - 1;
    const int qd = s + p.delta;
    if (p.causal) hi = min(hi, qd);
    if (p.window > 0) {
        if (p.causal) {
            lo = max(lo, qd - p.window + 1);
        } else {
            lo = max(lo, qd - p.window / 2);
            hi = min(hi, qd + p.window / 2);
        }
    }
}

// ROPE: compile-time, so the kernel without RoPE keeps the registers the
// rotation's table values would take.
template <int D, bool ROPE>
__global__ void __launch_bounds__(ROPE ? THREADS_ROPE : THREADS, 1) fa_decode_kernel(const __grid_constant__ CUtensorMap tmK,
                                                            const __grid_constant__ CUtensorMap tmV,
                                                            const __grid_constant__ Params p) {
    using L = Layout<D>;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
    const uint32_t bars = smem_u32(smem);
    auto full_bar = [&](int s) { return bars + 8u * s; };
    auto empty_bar = [&](int s) { return bars + 8u * (NST + s); };
    auto rot_bar = [&](int s) { return bars + 8u * (2 * NST + s); };  // RoPE: K tile of slot s rotated
    volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + 8 * 3 * NST);
    const Abort ab{abort_flag};
    uint8_t* ring = smem + L::OFF_RING;

    const int unit = blockIdx.y;
    const int b = unit / p.Hkv, kvh = unit % p.Hkv;
    // consumer warp -> (row group, tile class): tile i goes to the NRG warps of class i % NTG
    const int NRG = p.NRG, NTG = NCW / NRG;
    const int wrg = warp % NRG, wtg = warp / NRG;
    const int row0 = wrg * MAX_ROWS;  // first unit row of this warp's row group
    const uint32_t rank = cluster_rank(), csize = cluster_size();

    // visible key range of the unit (union over its rows), split across the cluster
    int ulo, uhi;
    {
        int lo0, hi0, lo1, hi1;
        row_range(p, 0, lo0, hi0);
        row_range(p, p.S - 1, lo1, hi1);
        ulo = lo0;
        uhi = hi1;
    }
    int t_begin = 0, t_end = 0;
    if (ulo <= uhi) {
        const int ta = ulo / KT, tb = uhi / KT + 1;
        const int n = tb - ta;
        t_begin = ta + static_cast<int>((static_cast<int64_t>(n) * rank) / csize);
        t_end = ta + static_cast<int>((static_cast<int64_t>(n) * (rank + 1)) / csize);
    }
    const int ntiles = t_end - t_begin;

    if (threadIdx.x == 0) {
        *abort_flag = 0;
        for (int s = 0; s < NST; ++s) {
            mbar_init(full_bar(s), 1);
            mbar_init(empty_bar(s), NRG);  // one arrive per row group's consumer warp
            mbar_init(rot_bar(s), 1);  // the tile's rotator warp
        }
        fence_barrier_init();
    }
    __syncthreads();

    float* part = reinterpret_cast<float*>(ring);                 // [NCW][MAX_ROWS][D + 2] after the loop
    float* cta = part + NCW * L::WARP_PART;                        // [R][D + 2]: O (D), m, l per unit row

    if (warp == NCW) {
        // ------------------------------------------------------------ producer
        if (lane == 0) {
            const uint64_t pol = policy_evict_first();
            const int kh = (p.kv_bcast & 2) ? 0 : kvh, kb = (p.kv_bcast & 1) ? 0 : b;  // broadcast axes: coordinate 0
            const int vh = (p.kv_bcast & 8) ? 0 : kvh, vb = (p.kv_bcast & 4) ? 0 : b;
            int filled[NST] = {0};
            bool ok = true;
            for (int i = 0; i < ntiles; ++i) {
                const int s = i % NST, n = i / NST;
                if (!mbar_wait(empty_bar(s), (n & 1) ^ 1, ab, 0x501)) {
                    ok = false;
                    break;
                }
                mbar_arrive_expect_tx(full_bar(s), L::STAGE);
                const uint32_t dst = smem_u32(ring + s * L::STAGE);
                const int k0 = (t_begin + i) * KT;
                for (int bx = 0; bx < L::NBOX; ++bx) {
                    tma_load_4d(dst + bx * L::BOX_BYTES, &tmK, full_bar(s), bx * L::BOX, k0, kh, kb, pol);
                    tma_load_4d(dst + L::TILE + bx * L::BOX_BYTES, &tmV, full_bar(s), bx * L::BOX, k0, vh, vb, pol);
                }
                filled[s]++;
            }
            if (!ok) {
                for (int s = 0; s < NST; ++s)
                    if (filled[s] > 0) mbar_wait_drain(full_bar(s), (filled[s] - 1) & 1);
            }
        }
        __syncwarp();  // lanes 1..31 wait here for lane 0's load loop
    } else if (ROPE && warp > NCW) {
        // ------------------------------------------------------------ rotators
        // Tile i -> rotator i % NRW: (key row, 16-byte chunk) tasks, chunk fastest
        // across the lanes, so 16 (D = 128) or 8 lanes read one whole cos/sin row
        // per load (coalesced); the first group of table loads is issued while
        // the tile is in flight.  The proxy fence orders the rotated rows before
        // the slot's next TMA write.
        constexpr int NCH = D / 8;   // 16-byte chunks per key row (= tasks per lane)
        constexpr int RG = 8;        // tasks per table-load group
        const int rw = warp - NCW - 1;
        bool aborted = false;
        for (int i = rw; i < ntiles; i += NRW) {
            const int s = i % NST, n = i / NST;
            const int k0 = (t_begin + i) * KT;
            float4 rc[RG], rs[RG];
            auto load_group = [&](int g0) {
#pragma unroll
                for (int u = 0; u < RG; ++u) {
                    const int task = (g0 + u) * 32 + lane, key = k0 + task / NCH;
                    if (g0 + u < NCH && key < p.KS) {  // rows past KS are zero fill
                        const int64_t ti = static_cast<int64_t>(key) * (D / 2) + 4 * (task % NCH);
                        rc[u] = __ldg(reinterpret_cast<const float4*>(p.rope_cos + ti));
                        rs[u] = __ldg(reinterpret_cast<const float4*>(p.rope_sin + ti));
                    }
                }
            };
            load_group(0);
            bool ok = !aborted && mbar_wait(full_bar(s), n & 1, ab, 0x504);
            ok = __all_sync(0xffffffffu, ok);
            if (!ok) {
                aborted = true;
                continue;
            }
            uint8_t* ktile = ring + s * L::STAGE;
#pragma unroll
            for (int g0 = 0; g0 < NCH; g0 += RG) {
                if (g0 > 0) load_group(g0);
#pragma unroll
                for (int u = 0; u < RG; ++u) {
                    const int task = (g0 + u) * 32 + lane, row = task / NCH;
                    if (g0 + u < NCH && k0 + row < p.KS)
                        rope::rotate_chunk(ktile + tile_off<D>(row, task % NCH), rc[u], rs[u]);
                }
            }
            fence_proxy_async_smem();
            __syncwarp();
            if (lane == 0) mbar_arrive(rot_bar(s));
        }
    } else {
        // ------------------------------------------------------------ consumers
        const int g = lane >> 2, t = lane & 3;
        // rows g and g + 8 of the 16-row tile: row r -> (head kvh*G + r / S, position r % S)
        const int rows[2] = {row0 + g, row0 + g + 8};  // unit rows
        int klo[2], khi[2];
        bool rvalid[2];
        for (int i = 0; i < 2; ++i) {
            rvalid[i] = rows[i] < p.R;
            const int s = rvalid[i] ? rows[i] % p.S : 0;
            row_range(p, s, klo[i], khi[i]);
            if (!rvalid[i]) {
                klo[i] = 1;
                khi[i] = 0;
            }
        }
        // Q fragments (A operand), straight from global memory, zero for padding rows
        uint32_t qa[D / 16][4];
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const int ri = j & 1;             // a0/a2: row g, a1/a3: row g+8
                const int dc = 16 * kk + 2 * t + ((j >> 1) << 3);
                uint32_t v = 0;
                if (rvalid[ri]) {
                    const int r = rows[ri];
                    const int h = kvh * p.G + r / p.S, s = r % p.S;
                    v = *reinterpret_cast<const uint32_t*>(p.q + b * p.qsb + h * p.qsh + s * p.qss + dc);
                    if constexpr (ROPE) {
                        const int64_t ti = static_cast<int64_t>(s) * (D / 2) + dc / 2;
                        v = rope::rotate_pair(v, __ldg(p.rope_cos + ti), __ldg(p.rope_sin + ti));
                    }
                }
                qa[kk][j] = v;
            }
        }
        float oacc[D / 8][4];
#pragma unroll
        for (int i = 0; i < D / 8; ++i) oacc[i][0] = oacc[i][1] = oacc[i][2] = oacc[i][3] = 0.f;
        float m_run[2] = {-INFINITY, -INFINITY};
        float l_run[2] = {0.f, 0.f};
        const float sl2 = p.scale_log2;
        bool aborted = false;

        for (int i = wtg; i < ntiles; i += NTG) {
            const int s = i % NST, n = i / NST;
            const int k0 = (t_begin + i) * KT;
            // RoPE: the tile's rotator warp signals when K is rotated
            bool ok = !aborted && mbar_wait(ROPE ? rot_bar(s) : full_bar(s), n & 1, ab, 0x502);
            ok = __all_sync(0xffffffffu, ok);
            if (!ok) {
                aborted = true;
                continue;
            }
            const uint32_t kb = smem_u32(ring + s * L::STAGE);
            const uint32_t vb = kb + L::TILE;

            // S = Q K^T over 32 keys: 4 n-tiles of 8 keys
            float sc[4][4];
#pragma unroll
            for (int nt = 0; nt < 4; ++nt) sc[nt][0] = sc[nt][1] = sc[nt][2] = sc[nt][3] = 0.f;
#pragma unroll
            for (int kk = 0; kk < D / 16; ++kk) {
#pragma unroll
                for (int np = 0; np < 2; ++np) {
                    const int mi = lane >> 3, ri = lane & 7;
                    const int key = 16 * np + ri + 8 * (mi >> 1);
                    const int chunk = 2 * kk + (mi & 1);
                    uint32_t b0, b1, b2, b3;
                    ldsm_x4(kb + tile_off<D>(key, chunk), b0, b1, b2, b3);
                    mma16816(sc[2 * np], qa[kk], b0, b1);
                    mma16816(sc[2 * np + 1], qa[kk], b2, b3);
                }
            }
            // mask, scale into the log2 domain, running max
            float mx[2] = {-INFINITY, -INFINITY};
#pragma unroll
            for (int nt = 0; nt < 4; ++nt) {
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    const int ri = e >> 1;
                    const int key = k0 + 8 * nt + 2 * t + (e & 1);
                    float v = sc[nt][e] * sl2;
                    if (key < klo[ri] || key > khi[ri]) v = -INFINITY;
                    sc[nt][e] = v;
                    mx[ri] = fmaxf(mx[ri], v);
                }
            }
            float corr[2], mref[2];
#pragma unroll
            for (int ri = 0; ri < 2; ++ri) {
                mx[ri] = fmaxf(mx[ri], __shfl_xor_sync(0xffffffffu, mx[ri], 1));
                mx[ri] = fmaxf(mx[ri], __shfl_xor_sync(0xffffffffu, mx[ri], 2));
                const float mn = fmaxf(m_run[ri], mx[ri]);
                corr[ri] = (mn == -INFINITY) ? 1.f : ex2(m_run[ri] - mn);
                m_run[ri] = mn;
                mref[ri] = (mn == -INFINITY) ? 0.f : mn;
                l_run[ri] *= corr[ri];
            }
#pragma unroll
            for (int i2 = 0; i2 < D / 8; ++i2) {
                oacc[i2][0] *= corr[0];
                oacc[i2][1] *= corr[0];
                oacc[i2][2] *= corr[1];
                oacc[i2][3] *= corr[1];
            }
            // P (fp16) as A fragments: k-step kk2 covers keys 16*kk2 .. +15
            uint32_t pa[2][4];
#pragma unroll
            for (int kk2 = 0; kk2 < 2; ++kk2) {
#pragma unroll
                for (int h2 = 0; h2 < 2; ++h2) {
                    const int nt = 2 * kk2 + h2;
                    const float p0 = ex2(sc[nt][0] - mref[0]);
                    const float p1 = ex2(sc[nt][1] - mref[0]);
                    const float p2 = ex2(sc[nt][2] - mref[1]);
                    const float p3 = ex2(sc[nt][3] - mref[1]);
                    l_run[0] += p0 + p1;
                    l_run[1] += p2 + p3;
                    pa[kk2][2 * h2 + 0] = pack_half2(p0, p1);
                    pa[kk2][2 * h2 + 1] = pack_half2(p2, p3);
                }
            }
            // O += P V: V tile [32 keys][D] is the K x N operand, transposed on load
#pragma unroll
            for (int kk2 = 0; kk2 < 2; ++kk2) {
#pragma unroll
                for (int dp = 0; dp < D / 16; ++dp) {
                    const int mi = lane >> 3, ri = lane & 7;
                    const int key = 16 * kk2 + ri + 8 * (mi & 1);
                    const int chunk = 2 * dp + (mi >> 1);
                    uint32_t b0, b1, b2, b3;
                    ldsm_x4_t(vb + tile_off<D>(key, chunk), b0, b1, b2, b3);
                    mma16816(oacc[2 * dp], pa[kk2], b0, b1);
                    mma16816(oacc[2 * dp + 1], pa[kk2], b2, b3);
                }
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(empty_bar(s));
        }
        // quad-reduce the row sums (partials scaled consistently with m_run)
#pragma unroll
        for (int ri = 0; ri < 2; ++ri) {
            l_run[ri] += __shfl_xor_sync(0xffffffffu, l_run[ri], 1);
            l_run[ri] += __shfl_xor_sync(0xffffffffu, l_run[ri], 2);
        }
        // all warps must be done with the ring before it holds partials
        named_bar_sync(1, 32 * NCW);
        float* wp = part + warp * L::WARP_PART;
#pragma unroll
        for (int ri = 0; ri < 2; ++ri) {
            const int r = rows[ri] - row0;  // row within the group
#pragma unroll
            for (int i2 = 0; i2 < D / 8; ++i2) {
                wp[r * (D + 2) + 8 * i2 + 2 * t] = oacc[i2][2 * ri];
                wp[r * (D + 2) + 8 * i2 + 2 * t + 1] = oacc[i2][2 * ri + 1];
            }
            if (t == 0) {
                wp[r * (D + 2) + D] = m_run[ri];
                wp[r * (D + 2) + D + 1] = l_run[ri];
            }
        }
        named_bar_sync(1, 32 * NCW);
        // combine the 4 warp partials into the CTA partial
        // combine, per unit row, the partials of the warps of its row group
        for (int idx = threadIdx.x; idx < p.R * D; idx += 32 * NCW) {
            const int ur = idx / D, d = idx % D;
            const int rgu = ur / MAX_ROWS, r = ur % MAX_ROWS;
            float M = -INFINITY;
            for (int k = 0; k < NTG; ++k) M = fmaxf(M, part[(rgu + k * NRG) * L::WARP_PART + r * (D + 2) + D]);
            float o = 0.f, l = 0.f;
            for (int k = 0; k < NTG; ++k) {
                const float* q = part + (rgu + k * NRG) * L::WARP_PART + r * (D + 2);
                const float f = (M == -INFINITY) ? 0.f : ex2(q[D] - M);
                o += q[d] * f;
                l += q[D + 1] * f;
            }
            cta[ur * (D + 2) + d] = o;
            if (d == 0) {
                cta[ur * (D + 2) + D] = M;
                cta[ur * (D + 2) + D + 1] = l;
            }
        }
    }
    // every thread of every CTA passes both cluster barriers, abort or not
    __syncwarp();
    cluster_sync_all();
    if (rank == 0 && warp < NCW) {
        const uint32_t cta_base = smem_u32(cta);
        for (int idx = threadIdx.x; idx < p.R * (D / 8); idx += 32 * NCW) {
            const int r = idx / (D / 8), c8 = idx % (D / 8);
            float M = -INFINITY;
            for (uint32_t cr = 0; cr < csize; ++cr)
                M = fmaxf(M, ld_dsmem(map_to_rank(cta_base + 4u * (r * (D + 2) + D), cr)));
            float o[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
            float l = 0.f;
            for (uint32_t cr = 0; cr < csize; ++cr) {
                const uint32_t rb = map_to_rank(cta_base + 4u * (r * (D + 2)), cr);
                const float mc = ld_dsmem(rb + 4u * D);
                const float f = (M == -INFINITY) ? 0.f : ex2(mc - M);
                l += ld_dsmem(rb + 4u * (D + 1)) * f;
#pragma unroll
                for (int e = 0; e < 8; ++e) o[e] += ld_dsmem(rb + 4u * (8 * c8 + e)) * f;
            }
            const float inv = l > 0.f ? 1.f / l : 0.f;
            uint4 v;
            v.x = pack_half2(o[0] * inv, o[1] * inv);
            v.y = pack_half2(o[2] * inv, o[3] * inv);
            v.z = pack_half2(o[4] * inv, o[5] * inv);
            v.w = pack_half2(o[6] * inv, o[7] * inv);
            const int h = kvh * p.G + r / p.S, s = r % p.S;
            if (!*abort_flag) {
                const int64_t off = b * p.osb + h * p.osh + s * p.oss + 8 * c8;
                *reinterpret_cast<uint4*>(p.o + off) = v;
#pragma unroll
                for (int k = 0; k < 7; ++k)
                    if (k < p.n_peer) *reinterpret_cast<uint4*>(p.o_peer[k] + off) = v;
            }
        }
    }
    __syncwarp();
    cluster_sync_all();
}

// ------------------------------------------------------------------ host
inline bool eligible(uint32_t seq_len, uint32_t group, uint32_t head_dim) {
    return (head_dim == 64 || head_dim == 128) && static_cast<uint64_t>(seq_len) * group <= MAX_ROWS * MAX_RG;
}

int launch_f16(char* err, const ForwardParams& a, cudaStream_t stream);

}  // namespace decode
}  // namespace rdna
