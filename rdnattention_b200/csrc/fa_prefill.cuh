// FlashAttention-2 forward for sm_100a: TMA -> shared memory, tcgen05.mma
// into TMEM, warp-specialised online softmax.
//
// One CTA owns NT (1 or 2) query tiles of 128 rows that share a KV head:
//   * NT = 2, pair_heads: two query heads of one GQA group, same rows, so
//     every K/V tile loaded into shared memory feeds two MMAs;
//   * NT = 2, row pairs: two consecutive 128-row blocks of one head (odd G);
//   * NT = 1: one tile (head_dim > 128, where TMEM holds a single O tile).
//
// Warp roles (THREADS = 128 * NT + 128):
//   warps [0, 4*NT)   softmax warpgroup t = warp / 4; thread = query row =
//                     TMEM lane.  Loads S from TMEM, masks boundary blocks,
//                     keeps the running max / row sum, writes P (fp16 or
//                     int8) back over S in TMEM, rescales O in TMEM when
//                     needed, and runs the epilogue (O / l -> fp16 -> TMA store).
//   warp 4*NT         TMA producer (one lane): a ring of K tiles and a ring
//                     of V tiles, across all of the CTA's work items.
//   warp 4*NT+1       MMA issuer (one lane): S_t = Q_t K^T (SS form),
//                     O_t += P_t V (TS form, P read from TMEM).
//   warp 4*NT+2       second MMA issuer when S is double-buffered (tile 1's
//                     MMAs), else idle.
//   warp 4*NT+3       Q producer (one lane): each item's Q tiles, once the
//                     previous item's Q K^T MMAs no longer read the buffer.
//
// One work item per CTA (items longest first for causal masks; the hardware
// block scheduler balances the tail).  The roles keep phase counters that
// would run on across items, so a role's loop body is written per item.
//
// Two schedules:
//   * single-buffered S (128-key blocks; INT8, head_dim > 128): per block j
//     and tile, PV(j) then QK(j+1) into the same TMEM columns, so a tile's
//     next S waits for its PV; the other tile's softmax fills the gap.
//   * double-buffered S (FP16 head_dim <= 128, 64-key blocks): S(t, j) lives
//     in buffer (j - first block) & 1; QK(j+2) is issued right after PV(j)
//     into the buffer PV(j) just read, so a tile's softmax only ever waits
//     for S itself.  An O rescale waits for PV(j-1) on its own barrier.
//     With two tiles each tile has its own MMA issuer thread.
//
// RoPE: rope.cuh rotates K once per launch and the kernel reads the rotated
// copy (rotating inside every CTA would repeat the K rotation once per query
// tile that reads the block); Q is rotated in shared memory by the softmax
// warps (T::ROPE_Q kernels) or by the same pre-pass.
//
// Output replicas (Params::n_peer > 0, the multi-GPU all-gather fused into the
// kernel): the staged tile of O is stored by TMA into the local output and into
// each peer GPU's output (one tensor map per peer, the same box coordinates),
// so the gather crosses NVLink while the CTAs after it compute.
//
// TMEM columns: S(t, b) at [(t*NSB + b)*BC, +BC) (P aliases its first
// columns); FP16: O_t (fp32) after all S.  INT8: ACC_t (s32 PV accumulator)
// then O_t (fp32, folded from ACC whenever the row max moves).
//
// Semantics follow the reference kernel (src/rdna/fa2_forward_f16.hip:633-741,
// src/rdna/fa2_forward_int8qk.hip:229-495): exp2-domain online softmax with
// scale*log2(e), P rounded to fp16 (or quantised min(127, lround(p*127)) for
// INT8) while the row sum uses the unrounded p, rows with no visible key
// produce 0, masks per src/rdna/fa2_forward_f16.hip:297-348.
#pragma once

#include <cuda_fp16.h>
#include <math.h>

#include "rope.cuh"
#include "sm100.cuh"

namespace rdna {
namespace prefill {

using namespace sm100;

constexpr int BM = 128;  // query rows per tile (= TMEM lanes)
constexpr int kMaxPeers = 7;  // output replicas on other GPUs (8 GPUs of one node)

// Tensor maps of the peers' outputs (PeerMaps::m[i] for i < Params::n_peer).
struct PeerMaps {
    CUtensorMap m[kMaxPeers];
};

struct Params {
    int B, H, Hkv, S, KS;
    int G;        // H / Hkv
    int delta;    // KS - S
    int causal;
    int window;   // <= 0: no window
    int pair_heads;
    int n_rb;     // ceil(S / BM)
    int n_rp;     // ceil(n_rb / 2)
    int n_split;  // output column slices per tile (head_dim > 256)
    int n_items;  // work items (CTA i handles items i, i + gridDim.x, ...)
    int dv_split; // output columns per slice (multiple of the box width)
    float scale_log2;
    // INT8 path
    float q_scale, k_scale, pv_scale;
    const float* q_vec;
    const float* k_vec;
    const float* v_chan;  // per-channel V scale (B, Hkv, D), or null
    // RoPE applied to Q inside the kernel (T::ROPE_Q kernels): Q tiles arrive
    // unrotated and the softmax warps rotate them in shared memory
    int rope_q;
    const float* rope_cos;  // [positions, D/2] fp32
    const float* rope_sin;
    // debug (T::DUMP_S kernels): the raw s32 Q K^T of every computed key block,
    // int32 [B, H, S, KS] contiguous
    int32_t* s_dump;
    // K/V axes broadcast with element stride 0 (KV_BCAST_* bits): their tensor
    // map has extent 1 there and the load coordinate is 0
    int kv_bcast;
    // debug (expired-wait test, off when dbg_withhold < 0): CTA 0 never loads the
    // K tile of its dbg_withhold-th key block and its waits give up after
    // dbg_wait_limit_ns, so the wait for that tile expires and the CTA unwinds
    int dbg_withhold;
    unsigned long long dbg_wait_limit_ns;
    // output replicas: n_peer other GPUs' counterparts of O (same strides, mapped
    // into this process; their tensor maps in PeerMaps), written with the same values as O
    int n_peer;
};

constexpr int KV_BCAST_KB = 1, KV_BCAST_KH = 2, KV_BCAST_VB = 4, KV_BCAST_VH = 8;

template <int D_, int DVMAX_, int BC_, int NT_, int NSK_, int NSV_, bool I8_, bool SDB_ = false,
          bool DUMP_S_ = false, bool TWOPASS_ = false>
struct Traits {
    static constexpr int D = D_;          // QK depth (head_dim)
    static constexpr int DVMAX = DVMAX_;  // output columns per CTA (<= 256)
    static constexpr int BC = BC_;        // keys per block
    static constexpr int NT = NT_;
    static constexpr int NSK = NSK_;
    static constexpr int NSV = NSV_;
    static constexpr bool I8 = I8_;
    // debug instantiations (INT8): write the raw s32 Q K^T to Params::s_dump
    static constexpr bool DUMP_S = DUMP_S_;
    // INT8 in two passes over the keys (S double-buffered): pass 1 only finds each
    // row's max, pass 2 quantises P against that final max, so the s32 P V
    // accumulator never needs rescaling and no fold into an fp32 O exists (valid
    // while 127 * 128 * key_seq_len < 2^31; longer sequences take the fold kernel).
    static constexpr bool TWOPASS = TWOPASS_;
    static_assert(!TWOPASS || I8_, "two-pass schedule is INT8-only");
    static_assert(!DUMP_S || I8, "score dump is INT8-only");
    // S double-buffered in TMEM: QK(j+2) is issued right after PV(j), while
    // the softmax works on S(j+1) from the other buffer.
    static constexpr bool SDB = SDB_;
    static constexpr int NSB = SDB ? 2 : 1;
    // MMA issuer threads: with double-buffered S and two tiles, each tile has
    // its own issuer (warps WARP_MMA and WARP_MMA + 1), so one tile's barrier
    // waits overlap the other tile's MMA issue.  K/V ring slots are released
    // once every issuer has committed.
    static constexpr int NI = ((SDB || TWOPASS) && NT == 2) ? 2 : 1;
    // Exp-phase token between the two softmax warpgroups, per scheduler: warp
    // w of one tile and warp w of the other (the pair that shares a MUFU) take
    // turns, without waiting for the other schedulers' warps.
    static constexpr bool TOKEN = NT == 2;
    // Kernels that can rotate Q themselves (one item per CTA: the softmax
    // warps are idle until the first S, so they rotate the Q tile that the
    // first Q K^T waits for); the RoPE pre-pass then only rotates K.
    static constexpr bool ROPE_Q = SDB && !I8;
    static_assert(NSK <= 8 && NSV <= 8 && (!SDB || NSV >= 2), "ring depth");
    static constexpr int ESZ = I8 ? 1 : 2;
    static constexpr int ROW_BYTES = D * ESZ;
    static constexpr int SW = (ROW_BYTES % 128 == 0) ? 128 : 64;  // swizzle span (bytes)
    static constexpr uint32_t LAYOUT = (SW == 128) ? 2u : 4u;    // UMMA layout code
    static constexpr int BOX = SW / ESZ;                          // elements per box row
    static constexpr int NBOX = D / BOX;
    static constexpr int NBOX_V = DVMAX / BOX;
    static constexpr int KSTEP = I8 ? 32 : 16;  // MMA K per instruction (elements)
    static constexpr int STEPS_PER_BOX = SW / 32;
    static constexpr int Q_BOX_BYTES = BM * SW;
    static constexpr int K_BOX_BYTES = BC * SW;
    static constexpr int Q_TILE = NBOX * Q_BOX_BYTES;
    static constexpr int K_TILE = NBOX * K_BOX_BYTES;
    static constexpr int V_TILE = NBOX_V * K_BOX_BYTES;
    static constexpr int THREADS = 128 * NT + 128;
    static constexpr int WARP_PROD = 4 * NT;
    static constexpr int WARP_MMA = 4 * NT + 1;
    static constexpr int WARP_QLOAD = 4 * NT + 3;
    // One-tile double-buffered kernels run two CTAs per SM (256 TMEM columns,
    // under half the shared memory each), so one CTA's prologue and epilogue
    // overlap the other's main loop.
    static constexpr int MIN_BLOCKS = (NT == 1 && SDB) ? 2 : 1;
    // Register split: launched at LAUNCH_REGS per thread (the most __launch_bounds__
    // allows for THREADS), then moved between warpgroups with setmaxnreg.
    static constexpr bool RESPLIT = NT == 2 || MIN_BLOCKS == 2;
    static constexpr int LAUNCH_REGS = MIN_BLOCKS == 2 ? 128 : (65536 / THREADS) / 8 * 8;
    // 128-key blocks hold 128 scores per softmax thread; 64-key blocks (S
    // double-buffered) need far fewer, and the two MMA issuer warps then keep
    // enough registers not to spill.
    // (splits at which ptxas spills nothing, checked by tests/test_resources_cpu.py)
    static constexpr int SOFTMAX_REGS = MIN_BLOCKS == 2 ? 184 : SDB ? 168 : (I8 && !TWOPASS) ? 208 : 216;
    static constexpr int CONTROL_REGS = MIN_BLOCKS == 2 ? 72 : SDB ? 168 : (I8 && !TWOPASS) ? 72 : 56;
    static_assert(!RESPLIT || 128 * NT * SOFTMAX_REGS + 128 * CONTROL_REGS <= THREADS * LAUNCH_REGS,
                  "register split exceeds the launch allocation");

    // TMEM columns
    static constexpr int S_COL0 = 0;                                 // S(t, b) at (t * NSB + b) * BC
    static constexpr int ACC_COL0 = NT * NSB * BC;                   // INT8 only
    // (the two-pass INT8 kernel has no fp32 O in TMEM: its output is ACC / l)
    static constexpr int O_COL0 = I8 ? NT * NSB * BC + (TWOPASS ? 0 : NT * DVMAX) : NT * NSB * BC;
    static_assert(!I8 || TWOPASS || !SDB, "the one-pass INT8 kernel keeps S single-buffered");
    static constexpr int TMEM_USED = O_COL0 + NT * DVMAX;
    static constexpr int TMEM_COLS = TMEM_USED <= 32 ? 32 : TMEM_USED <= 64 ? 64 : TMEM_USED <= 128 ? 128
                                     : TMEM_USED <= 256 ? 256 : 512;
    static_assert(TMEM_USED <= 512, "TMEM budget");
    static_assert(D % BOX == 0 && DVMAX % BOX == 0, "head_dim must tile into boxes");
    static_assert(BC % KSTEP == 0 && BC % 32 == 0, "key block");

    // Output (fp16) staging geometry.  FP16: O uses Q's swizzle and box and is
    // staged in Q_t's buffer.  INT8: fp16 rows are twice as wide as the int8 Q
    // rows, so O gets its own 128B-swizzled staging region.
    static constexpr int O_SW = I8 ? 128 : SW;
    static constexpr int O_BOX = O_SW / 2;
    static constexpr int O_BOX_BYTES = BM * O_SW;
    static constexpr int O_TILE = (DVMAX / O_BOX) * O_BOX_BYTES;
    static_assert(DVMAX % O_BOX == 0, "output slice tiles into boxes");

    // Shared memory: [misc 1 KB (+ INT8 key scales)][Q tiles][K ring][V ring]
    // (+ INT8 O staging), tiles 1024-aligned.
    static constexpr int OFF_KSCALE = 1024;  // INT8: [NT][2][BC] fp32 per-key scales
    static constexpr int MISC_BYTES = I8 ? OFF_KSCALE + NT * 2 * BC * 4 : 1024;
    static constexpr int OFF_Q = ((MISC_BYTES + 1023) / 1024) * 1024;
    static constexpr int OFF_K = OFF_Q + NT * Q_TILE;
    static constexpr int OFF_V = OFF_K + NSK * K_TILE;
    static constexpr bool OWN_STAGE = I8;
    static constexpr int OFF_O = OWN_STAGE ? OFF_V + NSV * V_TILE : OFF_Q;
    static constexpr int O_STRIDE = OWN_STAGE ? O_TILE : Q_TILE;  // staging bytes between tiles
    static constexpr int SMEM_BYTES = OFF_V + NSV * V_TILE + (OWN_STAGE ? NT * O_TILE : 0) + 1024;  // + align slack
    static_assert(SMEM_BYTES <= 232448, "shared memory budget");
    static_assert(OWN_STAGE || O_TILE <= Q_TILE, "O staging fits in the Q tile");

    static constexpr uint32_t IDESC_QK = instr_desc(I8 ? 2u : 1u, I8 ? 1u : 0u, 0u, BM, BC);
    static constexpr float THRESH = I8 ? 0.0f : 8.0f;  // log2-domain slack before O is rescaled
    // INT8: the s32 accumulator is folded into O with the exact-below-2^22 conversion
    // (i2f_biased), so a row folds before its bound on sum(Pq) can pass 2^15 (|V| <= 128
    // gives |ACC| < 2^22).  One block adds at most 127 * sum(p) + BC/2 <= 128 * BC + BC/2.
    static constexpr float PQ_FOLD = 32768.f - (128.f * BC + 0.5f * BC);
    static_assert(!I8 || PQ_FOLD > 0.f, "one block's P keeps the accumulator below 2^22");
};

// Barrier slots inside the misc region.
struct Bars {
    static constexpr int Q_FULL = 0, DRAIN = 2;
    static constexpr int K_FULL = 4;      // +NSK
    static constexpr int K_EMPTY = 12;    // +NSK
    static constexpr int V_FULL = 20;     // +NSV
    static constexpr int V_EMPTY = 28;    // +NSV
    static constexpr int S_FULL = 36;     // +t*NSB+b
    static constexpr int P_FULL = 40;     // +t*NSB+b
    static constexpr int O_FULL = 44;     // +NT
    static constexpr int PV_DONE = 46;    // +NT (each PV(t, j) complete; SDB only)
    static constexpr int KS_FULL = 48;    // +2*NT (INT8 per-key scale handoff, by block parity)
    static constexpr int EPI = 52;        // +NT (O staging written)
    static constexpr int EXPD = 63;       // +t*4+q: exp phase of tile t's warp in TMEM lane quadrant q finished
    static constexpr int Q_EMPTY = 56;    // Q tiles no longer read (every issuer commits once per item)
    static constexpr int O_EMPTY = 57;    // +NT (O read out of TMEM by the epilogue, one arrive per warp)
    static constexpr int STG_FREE = 59;   // +NT (O store has read the staging buffer)
    static constexpr int Q_ROT = 61;      // Q tiles rotated in place (one arrive per softmax warp)
    static constexpr int COUNT = 71;
    static constexpr int TMEM_SLOT = COUNT * 8;      // u32 TMEM base
    static constexpr int ABORT_SLOT = COUNT * 8 + 4; // int abort flag
};

// Error sites recorded in the status word (debug aid).
enum Site : int {
    SITE_PROD_KEMPTY = 0x101, SITE_PROD_VEMPTY = 0x102,
    SITE_MMA_Q = 0x201, SITE_MMA_K = 0x202, SITE_MMA_V = 0x203, SITE_MMA_P = 0x204,
    SITE_SM_S = 0x301, SITE_SM_O = 0x302, SITE_SM_Q = 0x303, SITE_SM_KS = 0x304, SITE_SM_EPI = 0x305,
    SITE_SM_TOKEN = 0x306, SITE_SM_PV = 0x307, SITE_SM_STG = 0x308,
    SITE_PROD_QEMPTY = 0x103, SITE_MMA_OEMPTY = 0x205, SITE_MMA_QROT = 0x206, SITE_SM_QROPE = 0x309,
};

struct Work {
    int b, kvh;
    int head[2];
    int row0[2];
    bool valid[2];
    int split;
};

template <class T>
__device__ __forceinline__ Work decode_work(const Params& p, int item) {
    Work w;
    w.split = item % p.n_split;
    item /= p.n_split;
    // Causal items differ in length: row blocks slowest, longest rows first
    // (the block scheduler then balances the tail).  Otherwise every item has
    // the same length and row blocks vary fastest, so the items that read one
    // (batch, KV head)'s K/V run in the same wave and find it in L2.
    const bool rows_fast = p.causal == 0;
    if constexpr (T::NT == 1) {
        const int per = p.B * p.H;
        int rb, rem;
        if (rows_fast) {
            rb = item % p.n_rb;
            rem = item / p.n_rb;
        } else {
            rb = p.n_rb - 1 - item / per;
            rem = item % per;
        }
        w.b = rem / p.H;
        const int h = rem % p.H;
        w.kvh = h / p.G;
        w.head[0] = w.head[1] = h;
        w.row0[0] = rb * BM;
        w.row0[1] = 0;
        w.valid[0] = true;
        w.valid[1] = false;
    } else if (p.pair_heads) {
        const int np = p.G / 2;
        const int per = p.B * p.Hkv * np;
        int rb, rem;
        if (rows_fast) {
            rb = item % p.n_rb;
            rem = item / p.n_rb;
        } else {
            rb = p.n_rb - 1 - item / per;
            rem = item % per;
        }
        w.b = rem / (p.Hkv * np);
        rem %= p.Hkv * np;
        w.kvh = rem / np;
        const int hp = rem % np;
        w.head[0] = w.kvh * p.G + 2 * hp;
        w.head[1] = w.head[0] + 1;
        w.row0[0] = w.row0[1] = rb * BM;
        w.valid[0] = w.valid[1] = true;
    } else {
        const int per = p.B * p.H;
        int rp, rem;
        if (rows_fast) {
            rp = item % p.n_rp;
            rem = item / p.n_rp;
        } else {
            rp = p.n_rp - 1 - item / per;
            rem = item % per;
        }
        w.b = rem / p.H;
        const int h = rem % p.H;
        w.kvh = h / p.G;
        w.head[0] = w.head[1] = h;
        w.row0[0] = 2 * rp * BM;
        w.row0[1] = (2 * rp + 1) * BM;
        w.valid[0] = true;
        w.valid[1] = w.row0[1] < p.S;
    }
    return w;
}

// Visible key interval of query row q (clamped to [0, KS-1]); empty if lo > hi.
__device__ __forceinline__ void row_keys(const Params& p, int q, int& lo, int& hi) {
    lo = 0;
    hi = p.KS - 1;
    const int qd = q + p.delta;
    if (p.causal) hi = min(hi, qd);
    if (p.window > 0) {
        if (p.causal) {
            lo = max(lo, qd - p.window + 1);
        } else {
            const int half = p.window / 2;
            lo = max(lo, qd - half);
            hi = min(hi, qd + half);
        }
    }
}

// [a, e) range of key blocks tile rows [row0, row0+BM) can touch.
template <class T>
__device__ __forceinline__ void tile_blocks(const Params& p, int row0, bool valid, int& a, int& e) {
    a = e = 0;
    if (!valid) return;
    const int rlast = min(row0 + BM - 1, p.S - 1);
    int lo0, hi0, lo1, hi1;
    row_keys(p, row0, lo0, hi0);
    row_keys(p, rlast, lo1, hi1);
    const int lo = lo0, hi = hi1;
    if (lo > hi || hi < 0 || lo > p.KS - 1) return;
    a = lo / T::BC;
    e = hi / T::BC + 1;
}

// The work item of this CTA (one item per CTA, items numbered longest first),
// or -1 past the end.  r counts the CTA's items (always 0 here).
__device__ __forceinline__ int item_at(const Params& p, int r) {
    const int64_t item = static_cast<int64_t>(r) * gridDim.x + blockIdx.x;
    return item < p.n_items ? static_cast<int>(item) : -1;
}

// Everything a role needs to know about one work item.
struct Item {
    Work w;
    int ta[2], te[2];  // per-tile key-block ranges [ta, te)
    int jlo, jhi;      // union of the tiles' ranges (the blocks the producer loads)
    int dv, dv0;       // output columns of this CTA: [dv0, dv0 + dv)
};

template <class T>
__device__ __forceinline__ Item make_item(const Params& p, int item) {
    Item I;
    I.w = decode_work<T>(p, item);
    if (p.n_split > 1) {
        I.dv0 = I.w.split * p.dv_split;
        I.dv = min(p.dv_split, T::D - I.dv0);
    } else {
        I.dv0 = 0;
        I.dv = T::D < T::DVMAX ? T::D : T::DVMAX;
    }
    I.ta[0] = I.te[0] = I.ta[1] = I.te[1] = 0;
    for (int t = 0; t < T::NT; ++t) tile_blocks<T>(p, I.w.row0[t], I.w.valid[t], I.ta[t], I.te[t]);
    I.jlo = 1 << 30;
    I.jhi = -1;
    for (int t = 0; t < T::NT; ++t) {
        if (I.te[t] > I.ta[t]) {
            I.jlo = min(I.jlo, I.ta[t]);
            I.jhi = max(I.jhi, I.te[t]);
        }
    }
    if (I.jhi < 0) I.jlo = I.jhi = 0;
    return I;
}

// Whether block j needs no per-element mask for any row of the tile.
template <class T>
__device__ __forceinline__ bool block_full(const Params& p, int row0, int j) {
    int loA, hiA, loB, hiB;
    row_keys(p, row0, loA, hiA);           // smallest hi
    row_keys(p, row0 + BM - 1, loB, hiB);  // largest lo
    const int k0 = j * T::BC, k1 = j * T::BC + T::BC - 1;
    return k0 >= loB && k1 <= hiA;
}

// Byte offset of 16-byte chunk `chunk` of row `row` inside one swizzled box.
template <int SW>
__device__ __forceinline__ uint32_t swz_off(int row, int chunk) {
    const uint32_t off = static_cast<uint32_t>(row * SW + chunk * 16);
    return off ^ (((off >> 7) & (SW / 16 - 1)) << 4);
}

// --------------------------------------------------------------- softmax
template <class T>
__device__ __forceinline__ void load_s_row(uint32_t taddr, uint32_t* r) {
    if constexpr (T::BC == 128) {
        if constexpr (T::LAUNCH_REGS <= 128) {
            // two 64-column loads, one wait: a 128-register destination does not fit
            // a kernel launched at 128 registers per thread
            tmem_ld_x64_nowait(taddr, r);
            tmem_ld_x64_nowait(taddr + 64, r + 64);
            tmem_wait_ld();
        } else {
            tmem_ld_x128(taddr, r);
        }
    } else if constexpr (T::BC == 64) {
        tmem_ld_x64(taddr, r);
    } else {
        tmem_ld_x32(taddr, r);
    }
}


// Row max of N values with 8 independent chains of 3-input max (dependency
// depth ~N/16 instead of N).
template <int N>
__device__ __forceinline__ float row_max(const float* x) {
    static_assert(N % 16 == 0, "row length");
    float m[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) m[i] = fmaxf(x[i], x[i + 8]);
#pragma unroll
    for (int c = 16; c < N; c += 16) {
#pragma unroll
        for (int i = 0; i < 8; ++i) m[i] = fmax3(m[i], x[c + i], x[c + 8 + i]);
    }
    return fmax3(fmax3(m[0], m[1], m[2]), fmax3(m[3], m[4], m[5]), fmaxf(m[6], m[7]));
}

// Warp-uniform bounded wait: every lane of the warp gets the same answer, so
// the warp-collective tcgen05.ld/st that follow never diverge.
__device__ __forceinline__ bool warp_wait(uint32_t bar, uint32_t parity, const Abort& ab, int site) {
    bool ok = mbar_wait(bar, parity, ab, site);
    return __all_sync(0xffffffffu, ok);
}

// RoPE on the item's Q tiles, in place in shared memory (ROPE_Q kernels),
// by all 4*NT softmax warps together: warp sw takes rows [RPW*sw, RPW*sw+RPW)
// of every tile as (row, 16-byte chunk) tasks, consecutive lanes on
// consecutive chunks, so each table load instruction reads whole rows of the
// cos/sin tables (coalesced) and, when the tiles sit at the same positions
// (two heads of a GQA group), one table fetch serves both tiles.  The loads
// are issued before Q_FULL, so their latency overlaps the tiles' TMA; rows
// past the sequence (TMA zero fill) are left alone.  Ends with a proxy fence:
// the tensor core reads the rotated tiles through the async proxy.
template <class T>
__device__ __forceinline__ bool rotate_q_tiles(const Params& p, const Work& w, uint8_t* smem, int sw, int lane,
                                               const Abort& ab) {
    constexpr int NCH = T::D / 8;              // 16-byte chunks (4 pairs) per row
    constexpr int CPB = T::BOX / 8;            // chunks per box row
    constexpr int RPW = BM / (4 * T::NT);      // rows per warp
    constexpr int TPL = RPW * NCH / 32;        // tasks per lane
    static_assert(RPW * NCH % 32 == 0, "task split");
    // tile 1 needs its own table rows unless it sits at tile 0's positions
    const bool own1 = T::NT == 2 && w.valid[1] && !(w.valid[0] && w.row0[0] == w.row0[1]);
    // table entries for tile 0's positions, and for tile 1's when they differ
    // (fixed register arrays: no runtime indexing, so nothing goes to local memory)
    float4 c0[TPL], s0[TPL], c1[TPL], s1[TPL];
#pragma unroll
    for (int k = 0; k < TPL; ++k) {
        const int task = k * 32 + lane;
        const int row = RPW * sw + task / NCH, ch = task % NCH;
        const int64_t off = static_cast<int64_t>(row) * (T::D / 2) + ch * 4;
        if (w.valid[0] && w.row0[0] + row < p.S) {
            const int64_t o = static_cast<int64_t>(w.row0[0]) * (T::D / 2) + off;
            c0[k] = __ldg(reinterpret_cast<const float4*>(p.rope_cos + o));
            s0[k] = __ldg(reinterpret_cast<const float4*>(p.rope_sin + o));
        }
        if (own1 && w.row0[1] + row < p.S) {
            const int64_t o = static_cast<int64_t>(w.row0[1]) * (T::D / 2) + off;
            c1[k] = __ldg(reinterpret_cast<const float4*>(p.rope_cos + o));
            s1[k] = __ldg(reinterpret_cast<const float4*>(p.rope_sin + o));
        }
    }
    if (!warp_wait(smem_u32(smem) + 8u * Bars::Q_FULL, 0, ab, SITE_SM_QROPE)) return false;
#pragma unroll
    for (int k = 0; k < TPL; ++k) {
        const int task = k * 32 + lane;
        const int row = RPW * sw + task / NCH, ch = task % NCH;
        const uint32_t off = (ch / CPB) * T::Q_BOX_BYTES + swz_off<T::SW>(row, ch % CPB);
        if (w.valid[0] && w.row0[0] + row < p.S) rope::rotate_chunk(smem + T::OFF_Q + off, c0[k], s0[k]);
        if (T::NT == 2 && w.valid[1] && w.row0[1] + row < p.S)
            rope::rotate_chunk(smem + T::OFF_Q + T::Q_TILE + off, own1 ? c1[k] : c0[k], own1 ? s1[k] : s0[k]);
    }
    fence_proxy_async_smem();
    return true;
}

// Softmax warpgroup for tile t.  Loops never exit early and no named
// barriers are used: after an abort every remaining wait returns false at
// once and the work is skipped, so all threads reach the kernel's final
// __syncthreads.
template <class T>
__device__ void softmax_role(const Params& p, const CUtensorMap* tmO, int t, uint8_t* smem, uint32_t tmem,
                             const Abort& ab, const PeerMaps* pm) {
    const int warp = threadIdx.x / 32;
    const int lane = threadIdx.x % 32;
    const int wq = warp % 4;
    const int r = wq * 32 + lane;
    const uint32_t lane_base = static_cast<uint32_t>(wq * 32) << 16;
    const uint32_t tS0 = tmem + lane_base + T::S_COL0 + t * T::NSB * T::BC;
    const uint32_t tO = tmem + lane_base + T::O_COL0 + t * T::DVMAX;
    const uint32_t tACC = tmem + lane_base + T::ACC_COL0 + t * T::DVMAX;
    const uint32_t bars = smem_u32(smem);
    auto bar = [&](int i) { return bars + 8u * static_cast<uint32_t>(i); };
    const float sl2 = p.scale_log2;
    bool aborted = false;
    // phase counters carried across this CTA's items
    int g = 0;     // key blocks of tile t done in earlier items (S / P / PV_DONE / KS phases)
    int n_o = 0;   // earlier items in which tile t accumulated O (O_FULL / O_EMPTY phases)
    int n_st = 0;  // earlier O stores of tile t (EPI / STG_FREE phases)

    // exactly one item per CTA (a trip count the compiler can see)
    for (int n_it = 0; n_it < 1; ++n_it) {
    const int item = item_at(p, n_it);
    if (item < 0) break;
    const Item I = make_item<T>(p, item);
    const Work& w = I.w;
    const int dv = I.dv, dv0 = I.dv0;
    if constexpr (T::ROPE_Q) {
        if (p.rope_q) {
            // every softmax warp rotates its rows of all tiles (one item per CTA: Q_FULL phase 0)
            if (!rotate_q_tiles<T>(p, w, smem, warp, lane, ab)) aborted = true;
            __syncwarp();
            if (lane == 0) mbar_arrive(bar(Bars::Q_ROT));
        }
    }
    if (!w.valid[t]) continue;  // uniform for the warpgroup (no O store, no phases used)
    const int row0 = w.row0[t];
    const int q = row0 + r;
    const int a = I.ta[t], e = I.te[t];
    int klo, khi;
    row_keys(p, q, klo, khi);
    // Exp-phase order between the two warps on this scheduler (warp w of WG0 and
    // of WG1): WG0 k, WG1 k, WG0 k+1, ... (k = each tile's own iteration count),
    // so the scheduler's MUFU serves one of them at a time.
    const int other_iters = T::TOKEN ? I.te[1 - t] - I.ta[1 - t] : 0;

    float m_ref = -INFINITY;
    float l = 0.f;

    // INT8 state
    float rowscale = 1.f;
    bool oflushed = false;  // O holds folded blocks
    float pq_acc = 0.f;     // bound on sum(Pq) held in ACC since the last fold
    float* ksbuf = nullptr;
    const bool kvec = T::I8 && p.k_vec != nullptr;
    if constexpr (T::I8) {
        float qs = p.q_scale;
        if (p.q_vec != nullptr && q < p.S) qs = p.q_vec[(static_cast<int64_t>(w.b) * p.H + w.head[t]) * p.S + q];
        rowscale = qs * sl2;
        if (!kvec) rowscale *= p.k_scale;
        ksbuf = reinterpret_cast<float*>(smem + T::OFF_KSCALE) + t * 2 * T::BC;
    }

    // per-key K scales of the next block are fetched one block ahead, so the
    // global-load latency never sits on the softmax critical path
    const float* kvec_row = kvec ? p.k_vec + (static_cast<int64_t>(w.b) * p.Hkv + w.kvh) * p.KS : nullptr;
    auto load_ks = [&](int jb) {
        const int key = jb * T::BC + r;
        return (kvec && r < T::BC && jb < e && key < p.KS) ? __ldg(kvec_row + key) : 0.f;
    };
    float ks_next = load_ks(a);

    int it = 0;
    for (int j = a; j < e; ++j, ++it) {
        const int gg = g + it;  // this block's index among all blocks of tile t in this CTA
        if constexpr (T::I8) {
            if (kvec) {
                // stage this block's per-key scales; buffer (gg & 1) is reused every second block
                const int buf = gg & 1;
                if (r < T::BC) ksbuf[buf * T::BC + r] = ks_next;
                mbar_arrive(bar(Bars::KS_FULL + 2 * t + buf));
                ks_next = load_ks(j + 1);
                if (!aborted && !warp_wait(bar(Bars::KS_FULL + 2 * t + buf), (gg >> 1) & 1, ab, SITE_SM_KS))
                    aborted = true;
            }
        }
        // S buffer of this block, and the phase of its barrier
        const int sb = T::SDB ? (gg & 1) : 0;
        const uint32_t tS = tS0 + sb * T::BC;
        const uint32_t s_par = T::SDB ? ((gg >> 1) & 1) : (gg & 1);
        if (!aborted && !warp_wait(bar(Bars::S_FULL + t * T::NSB + sb), s_par, ab, SITE_SM_S)) aborted = true;
        if (aborted) continue;
        tc_fence_after();

        if constexpr (T::DUMP_S) {
            // debug: the raw s32 scores, re-read 16 columns at a time (warp-wide loads)
            int32_t* dst = p.s_dump + ((static_cast<int64_t>(w.b) * p.H + w.head[t]) * p.S + q) * p.KS;
            for (int c0 = 0; c0 < T::BC; c0 += 16) {
                uint32_t d16[16];
                tmem_ld_x16(tS + c0, d16);
#pragma unroll
                for (int c = 0; c < 16; ++c)
                    if (q < p.S && j * T::BC + c0 + c < p.KS) dst[j * T::BC + c0 + c] = static_cast<int32_t>(d16[c]);
            }
        }
        uint32_t raw[T::BC];
        load_s_row<T>(tS, raw);
        float* x = reinterpret_cast<float*>(raw);
        const bool full = block_full<T>(p, row0, j);
        const int lo = klo - j * T::BC, hi = khi - j * T::BC;

        float mx;
        if constexpr (T::I8) {
            // s32 -> float by cvt.rn (exact: |q.k| <= 127*127*D < 2^22; one instruction
            // per score, measured 5 % faster at head_dim 64 than the add-and-subtract
            // bias trick).  x holds float(acc) * k_scale; the per-row q_scale * scale *
            // log2(e) (rowscale) is applied to the max and folded into the exponent's FMA.
            const float* ksb = ksbuf + (gg & 1) * T::BC;
            // the key-scale product on sm_100's paired fp32 instructions, two at a time
            // (mb2 is not read here: with the definition in place ptxas allocates this
            // kernel at 168 registers without spills, without it 4 bytes spill)
            [[maybe_unused]] const uint64_t mb2 = f2(-12582912.0f, -12582912.0f);
            if (kvec) {
#pragma unroll
                for (int c = 0; c < T::BC; c += 2) {
                    const uint64_t v = f2(s32_to_f32(raw[c]), s32_to_f32(raw[c + 1]));
                    f2_split(fmul2(v, *reinterpret_cast<const uint64_t*>(ksb + c)), x[c], x[c + 1]);
                }
            } else {
#pragma unroll
                for (int c = 0; c < T::BC; c += 2) f2_split(f2(s32_to_f32(raw[c]), s32_to_f32(raw[c + 1])), x[c], x[c + 1]);
            }
            if (!full) {
#pragma unroll
                for (int c = 0; c < T::BC; ++c)
                    if (c < lo || c > hi) x[c] = rowscale >= 0.f ? -INFINITY : INFINITY;
            }
            // max of x * rowscale: max(x) * rowscale for rowscale >= 0, else min(x) * rowscale
            if (rowscale >= 0.f) {
                mx = row_max<T::BC>(x) * rowscale;
            } else {
#pragma unroll
                for (int c = 0; c < T::BC; ++c) x[c] = -x[c];
                mx = row_max<T::BC>(x) * -rowscale;
            }
            if (mx != mx) mx = -INFINITY;  // fully masked row with rowscale == 0
        } else {
            if (sl2 > 0.f) {
                if (!full) {
#pragma unroll
                    for (int c = 0; c < T::BC; ++c)
                        if (c < lo || c > hi) x[c] = -INFINITY;
                }
                mx = row_max<T::BC>(x) * sl2;
            } else {
                // non-positive scale: scale first, then mask (rare; keeps max semantics exact)
#pragma unroll
                for (int c = 0; c < T::BC; ++c) {
                    float v = x[c] * sl2;
                    if (!full && (c < lo || c > hi)) v = -INFINITY;
                    x[c] = v;
                }
                mx = row_max<T::BC>(x);
            }
        }

        const float m_new = fmaxf(m_ref, mx);
        float corr = 1.f;
        bool rescale = false;
        if (m_new > m_ref + T::THRESH) {
            corr = ex2(m_ref - m_new);  // 0 when m_ref = -inf
            l *= corr;
            rescale = (it > 0);
            m_ref = m_new;
        }

        if constexpr (!T::I8) {
            // O(tmem) *= corr once PV(j-1) is complete.  Single-buffered S: S_FULL(j)
            // was committed after PV(j-1).  Double-buffered: wait for PV_DONE phase
            // gg-1; PV(j) cannot have been issued yet (it needs this warp's P), so
            // the barrier is at most one phase ahead and the parity is unambiguous.
            if (__any_sync(0xffffffffu, rescale)) {
                if constexpr (T::SDB) {
                    if (!warp_wait(bar(Bars::PV_DONE + t), (gg - 1) & 1, ab, SITE_SM_PV)) {
                        aborted = true;
                        continue;
                    }
                    tc_fence_after();
                }
                const float c = rescale ? corr : 1.f;
                for (int c0 = 0; c0 < dv; c0 += 32) {
                    uint32_t o[32];
                    tmem_ld_x32(tO + c0, o);
#pragma unroll
                    for (int i = 0; i < 32; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * c);
                    tmem_st_x32(tO + c0, o);
                }
                tmem_wait_st();
            }
        } else {
            // INT8: the accumulator fold runs after the exponent phase (below), when the
            // block's scores no longer hold registers; P V(j) waits for both anyway
        }

        // P = exp2(s*scale*log2e - m); the row sum uses the unrounded values
        const float neg_m = (m_ref == -INFINITY) ? 0.f : -m_ref;
        float lsum = 0.f;
        if constexpr (T::TOKEN) {
            const int need = it - 1 + t;  // the other warpgroup's exp phase that comes first
            if (need >= 0 && need < other_iters &&
                !warp_wait(bar(Bars::EXPD + (1 - t) * 4 + wq), need & 1, ab, SITE_SM_TOKEN)) {
                aborted = true;
                continue;
            }
        }
        // P goes back over S in 32-key chunks (S is already in registers), so only
        // one chunk of packed P is live at a time.  8 independent partial sums keep
        // the row-sum dependency chain short.
        float ls[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
        if constexpr (!T::I8) {
            const float mul = (sl2 > 0.f) ? sl2 : 1.f;
            const uint64_t mul2 = f2(mul, mul), nm2 = f2(neg_m, neg_m);
            uint64_t ls2[4] = {0ull, 0ull, 0ull, 0ull};  // (0.f, 0.f)
            // the scale-and-shift FMAs and row sums on sm_100's paired fp32 instructions
            // (two per issue); all exponentials on the MUFU: moving a share to the FMA
            // pipe (polynomial exp2) costs about as many issue slots as it saves
#pragma unroll
            for (int c0 = 0; c0 < T::BC; c0 += 32) {
                uint32_t pk[16];
#pragma unroll
                for (int c = 0; c < 32; c += 2) {
                    float a0, a1;
                    f2_split(ffma2(f2(x[c0 + c], x[c0 + c + 1]), mul2, nm2), a0, a1);
                    const float p0 = ex2(a0);
                    const float p1 = ex2(a1);
                    ls2[(c >> 1) & 3] = fadd2(ls2[(c >> 1) & 3], f2(p0, p1));
                    pk[c / 2] = pack_half2(p0, p1);
                }
                tmem_st_x16(tS + c0 / 2, pk);
            }
#pragma unroll
            for (int i = 0; i < 4; ++i) f2_split(ls2[i], ls[2 * i], ls[2 * i + 1]);
        } else {
            // p in [0, 1] against the running max, computed two at a time in half
            // precision (P only keeps 7 bits): fma(p, 127, 1024) in fp16 has unit
            // spacing, so its low byte is round(p * 127) (round-to-nearest-even; the
            // reference's lround differs only at exact .5 ties).  Row sums accumulate
            // in 8 f16x2 partials (<= 8 values each) and finish in fp32.
            const float ars = fabsf(rowscale);       // x was negated when rowscale < 0
            constexpr uint32_t k127 = 0x57F057F0u;   // (127, 127) in f16x2
            constexpr uint32_t k1024 = 0x64006400u;  // (1024, 1024)
            uint32_t hs[8] = {0u, 0u, 0u, 0u, 0u, 0u, 0u, 0u};
#pragma unroll
            for (int c0 = 0; c0 < T::BC; c0 += 32) {
                uint32_t pk[8];
#pragma unroll
                for (int c = 0; c < 32; c += 4) {
                    float a0, a1, a2, a3;
                    const uint64_t ars2 = f2(ars, ars), nm2 = f2(neg_m, neg_m);
                    f2_split(ffma2(f2(x[c0 + c], x[c0 + c + 1]), ars2, nm2), a0, a1);
                    f2_split(ffma2(f2(x[c0 + c + 2], x[c0 + c + 3]), ars2, nm2), a2, a3);
                    const uint32_t e0 = ex2_h2(pack_half2(a0, a1));
                    const uint32_t e1 = ex2_h2(pack_half2(a2, a3));
                    hs[(c >> 2) & 7] = hadd2(hs[(c >> 2) & 7], hadd2(e0, e1));
                    pk[c / 4] = pack_half_low_bytes(hfma2(e0, k127, k1024), hfma2(e1, k127, k1024));
                }
                tmem_st_x8(tS + c0 / 4, pk);
            }
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                const __half2 h = *reinterpret_cast<const __half2*>(&hs[i]);
                ls[i] = __low2float(h) + __high2float(h);
            }
        }
        lsum = ((ls[0] + ls[1]) + (ls[2] + ls[3])) + ((ls[4] + ls[5]) + (ls[6] + ls[7]));
        l += lsum;
        // sum(Pq) <= 127 * sum(p) + BC/2; the factor 128 covers the f16 partial sums' rounding
        if constexpr (T::I8) {
            // INT8: the s32 accumulator holds sum(Pq * V) quantised against the running
            // max.  A warp folds it into the fp32 O when any of its rows' max moves, and
            // before a row's |ACC| can reach 2^22 (the limit of the conversion below):
            // after this block's PV, ACC holds at most pq_acc + 128 * BC + BC/2 < 2^15
            // times max|V| <= 128.  Every lane folds (factor 1 where its max did not
            // move), so the fold has no per-element selects; 16 columns at a time keep
            // the fold's registers beside the block's scores.
            const bool flush = rescale || (it > 0 && pq_acc >= T::PQ_FOLD);
            if (__any_sync(0xffffffffu, flush)) {
                const float c = rescale ? corr : 1.f;
                const float psc = p.pv_scale * c;
                const uint64_t psc2 = f2(psc, psc), c2 = f2(c, c), mb2 = f2(-12582912.0f, -12582912.0f);
                for (int c0 = 0; c0 < dv; c0 += 16) {
                    uint32_t acc[16], o[16];
                    tmem_ld_x16(tACC + c0, acc);
                    if (oflushed) {
                        tmem_ld_x16(tO + c0, o);
#pragma unroll
                        for (int i = 0; i < 16; i += 2) {
                            const uint64_t af = fadd2(f2(i2f_biased(acc[i]), i2f_biased(acc[i + 1])), mb2);
                            const uint64_t oc = fmul2(f2(__uint_as_float(o[i]), __uint_as_float(o[i + 1])), c2);
                            float a0, a1;
                            f2_split(ffma2(af, psc2, oc), a0, a1);
                            o[i] = __float_as_uint(a0);
                            o[i + 1] = __float_as_uint(a1);
                        }
                    } else {
#pragma unroll
                        for (int i = 0; i < 16; i += 2) {
                            const uint64_t af = fadd2(f2(i2f_biased(acc[i]), i2f_biased(acc[i + 1])), mb2);
                            float a0, a1;
                            f2_split(fmul2(af, psc2), a0, a1);
                            o[i] = __float_as_uint(a0);
                            o[i + 1] = __float_as_uint(a1);
                        }
                    }
                    tmem_st_x16(tO + c0, o);
                }
                for (int c0 = 0; c0 < dv; c0 += 32) tmem_zero_x32(tACC + c0);
                tmem_wait_st();
                oflushed = true;
                pq_acc = 0.f;
            }
            pq_acc += fmaf(lsum, 128.f, 0.5f * T::BC);
        }
        if constexpr (T::TOKEN) {
            __syncwarp();
            if (lane == 0) mbar_arrive(bar(Bars::EXPD + t * 4 + wq));
        }
        tmem_wait_st();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(bar(Bars::P_FULL + t * T::NSB + sb));
    }

    // ---------------------------------------------------------------- epilogue
    const bool has_blocks = e > a;
    if (!aborted && has_blocks && !warp_wait(bar(Bars::O_FULL + t), n_o & 1, ab, SITE_SM_O)) aborted = true;
    if (!aborted) tc_fence_after();
    if constexpr (!T::OWN_STAGE) {
        // FP16 with one item per CTA stages O in Q_t's buffer: its TMA load must have landed
        if (!aborted && !warp_wait(bar(Bars::Q_FULL), 0, ab, SITE_SM_Q)) aborted = true;
    } else if (n_st > 0) {
        // the previous item's store must have finished reading the staging buffer
        // (issued an item ago, so the wait is normally already satisfied)
        if (r == 0) {
            bulk_wait_read_all();
            mbar_arrive(bar(Bars::STG_FREE + t));
        }
        if (!aborted && !warp_wait(bar(Bars::STG_FREE + t), (n_st - 1) & 1, ab, SITE_SM_STG)) aborted = true;
    }

    uint8_t* stage = smem + T::OFF_O + t * T::O_STRIDE;
    if (!aborted) {
        const float inv = (l > 0.f) ? 1.f / l : 0.f;
        for (int c0 = 0; c0 < dv; c0 += 32) {
            float o[32];
            if (has_blocks) {
                uint32_t ov[32];
                tmem_ld_x32(tO + c0, ov);
                if constexpr (T::I8) {
                    // O (the folded blocks, if any) plus the blocks in ACC since the last fold
                    uint32_t acc[32];
                    tmem_ld_x32(tACC + c0, acc);
#pragma unroll
                    for (int i = 0; i < 32; ++i) {
                        const float of = oflushed ? __uint_as_float(ov[i]) : 0.f;
                        o[i] = (of + static_cast<float>(static_cast<int>(acc[i])) * p.pv_scale) * inv;
                    }
                    if (p.v_chan != nullptr) {
                        // per-channel V dequantisation, folded in before the one fp16 rounding
                        const float* vc = p.v_chan + (static_cast<int64_t>(w.b) * p.Hkv + w.kvh) * T::D + dv0 + c0;
#pragma unroll
                        for (int i = 0; i < 32; ++i) o[i] *= __ldg(vc + i);
                    }
                } else {
#pragma unroll
                    for (int i = 0; i < 32; ++i) o[i] = __uint_as_float(ov[i]) * inv;
                }
            } else {
#pragma unroll
                for (int i = 0; i < 32; ++i) o[i] = 0.f;
            }
            // 32 fp16 = 4 chunks of 16 bytes
#pragma unroll
            for (int g4 = 0; g4 < 4; ++g4) {
                uint4 v;
                v.x = pack_half2(o[8 * g4 + 0], o[8 * g4 + 1]);
                v.y = pack_half2(o[8 * g4 + 2], o[8 * g4 + 3]);
                v.z = pack_half2(o[8 * g4 + 4], o[8 * g4 + 5]);
                v.w = pack_half2(o[8 * g4 + 6], o[8 * g4 + 7]);
                const int col = c0 + 8 * g4;
                const int box = col / T::O_BOX;
                const int chunk = (col % T::O_BOX) / 8;
                *reinterpret_cast<uint4*>(stage + box * T::O_BOX_BYTES + swz_off<T::O_SW>(r, chunk)) = v;
            }
        }
        fence_proxy_async_smem();
    }
    if (has_blocks) {
        // O (and the INT8 accumulator) are out of TMEM: the next item's first PV may overwrite them
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(bar(Bars::O_EMPTY + t));
    }
    mbar_arrive(bar(Bars::EPI + t));
    if (r == 0) {
        if (!aborted && mbar_wait(bar(Bars::EPI + t), n_st & 1, ab, SITE_SM_EPI) && !*ab.flag) {
            const int nbox = dv / T::O_BOX;
            for (int bx = 0; bx < nbox; ++bx)
                tma_store_4d(tmO, smem_u32(stage + bx * T::O_BOX_BYTES), dv0 + bx * T::O_BOX, row0, w.head[t], w.b);
            if constexpr (!T::DUMP_S) {  // (debug score dumps take no output replicas)
                // the same boxes into every peer's output: the TMA engine carries them
                // over NVLink while this CTA exits and the next one computes
                for (int k = 0; k < p.n_peer; ++k)
                    for (int bx = 0; bx < nbox; ++bx)
                        tma_store_4d(&pm->m[k], smem_u32(stage + bx * T::O_BOX_BYTES), dv0 + bx * T::O_BOX, row0,
                                     w.head[t], w.b);
            }
            bulk_commit();
            // FP16 stages O in Q's buffer: wait here; INT8 waits before the exit
            if constexpr (!T::OWN_STAGE) bulk_wait_read_all();
        }
    }
    g += e - a;
    n_o += has_blocks ? 1 : 0;
    ++n_st;
    }  // items
    if constexpr (T::OWN_STAGE) {
        // the stores have read the staging buffer before the CTA (and its shared
        // memory) goes; their writes complete before the kernel does
        if (r == 0) bulk_wait_read_all();
    }
}

// ------------------------------------------------------------- producers
// Two TMA producer lanes.  The K/V producer streams every item's K and V
// blocks through the rings, whose slot and phase counters run on across
// items, so the next item's first blocks load during the current item's tail.
// The Q producer loads an item's Q tiles once the previous item's Q K^T MMAs
// are done with the buffer (Q_EMPTY).
template <class T>
__device__ void producer_q_role(const Params& p, const CUtensorMap* tmQ, uint8_t* smem, const Abort& ab) {
    const uint32_t bars = smem_u32(smem);
    auto bar = [&](int i) { return bars + 8u * static_cast<uint32_t>(i); };
    prefetch_tmap(tmQ);
    const uint64_t pol_q = policy_evict_first();
    // Q comes from the RoPE pre-pass in the kernels that do not rotate it themselves
    if constexpr (!T::ROPE_Q) grid_dependency_wait();
    int qfill = 0;
    for (int r = 0; r < 1; ++r) {
        const int item = item_at(p, r);
        if (item < 0) break;
        const Work w = decode_work<T>(p, item);
        if (qfill > 0 && !mbar_wait(bar(Bars::Q_EMPTY), (qfill - 1) & 1, ab, SITE_PROD_QEMPTY)) break;
        mbar_arrive_expect_tx(bar(Bars::Q_FULL), T::NT * T::Q_TILE);
        for (int t = 0; t < T::NT; ++t) {
            const uint32_t dst = smem_u32(smem + T::OFF_Q + t * T::Q_TILE);
            for (int bx = 0; bx < T::NBOX; ++bx)
                tma_load_4d(dst + bx * T::Q_BOX_BYTES, tmQ, bar(Bars::Q_FULL), bx * T::BOX, w.row0[t], w.head[t],
                            w.b, pol_q);
        }
        ++qfill;
    }
    // every issued copy lands before the CTA can exit
    if (qfill > 0) mbar_wait_drain(bar(Bars::Q_FULL), (qfill - 1) & 1);
}

template <class T>
__device__ void producer_kv_role(const Params& p, const CUtensorMap* tmK, const CUtensorMap* tmV, uint8_t* smem,
                                 const Abort& ab) {
    const uint32_t bars = smem_u32(smem);
    auto bar = [&](int i) { return bars + 8u * static_cast<uint32_t>(i); };
    prefetch_tmap(tmK);
    prefetch_tmap(tmV);
    const uint64_t pol_kv = policy_evict_last();
    // K may be the RoPE pre-pass's output: a launch that overlaps the pre-pass
    // (programmatic dependent launch) waits here for it; otherwise a no-op
    grid_dependency_wait();

    int kfill[T::NSK] = {0};
    int vfill[T::NSV] = {0};
    bool ok = true;
    int i = 0;   // K blocks loaded so far
    int iv = 0;  // V blocks loaded so far
    for (int n = 0; ok && n < 1; ++n) {
        const int item = item_at(p, n);
        if (item < 0) break;
        const Item I = make_item<T>(p, item);
        const Work& w = I.w;
        const int nbox_v = I.dv / T::BOX;
        const int kh = (p.kv_bcast & KV_BCAST_KH) ? 0 : w.kvh, kb = (p.kv_bcast & KV_BCAST_KB) ? 0 : w.b;
        const int vh = (p.kv_bcast & KV_BCAST_VH) ? 0 : w.kvh, vb = (p.kv_bcast & KV_BCAST_VB) ? 0 : w.b;
        // two-pass INT8: every K block twice (pass 1 finds the row maxima), V in pass 2 only
        const int N = I.jhi - I.jlo;
        for (int u = 0; u < (T::TWOPASS ? 2 * N : N); ++u, ++i) {
            const int j = I.jlo + (u < N ? u : u - N);
            const int ks = i % T::NSK, kn = i / T::NSK;
            if (!mbar_wait(bar(Bars::K_EMPTY + ks), (kn & 1) ^ 1, ab, SITE_PROD_KEMPTY)) {
                ok = false;
                break;
            }
            if (p.dbg_withhold == i && blockIdx.x == 0) {
                // debug launch: this tile never arrives (its consumer's wait expires)
            } else {
                mbar_arrive_expect_tx(bar(Bars::K_FULL + ks), T::K_TILE);
                const uint32_t kdst = smem_u32(smem + T::OFF_K + ks * T::K_TILE);
                for (int bx = 0; bx < T::NBOX; ++bx)
                    tma_load_4d(kdst + bx * T::K_BOX_BYTES, tmK, bar(Bars::K_FULL + ks), bx * T::BOX, j * T::BC, kh,
                                kb, pol_kv);
                kfill[ks]++;
            }
            if (T::TWOPASS && u < N) continue;
            const int vs = iv % T::NSV, vn = iv / T::NSV;
            if (!mbar_wait(bar(Bars::V_EMPTY + vs), (vn & 1) ^ 1, ab, SITE_PROD_VEMPTY)) {
                ok = false;
                break;
            }
            mbar_arrive_expect_tx(bar(Bars::V_FULL + vs), nbox_v * T::K_BOX_BYTES);
            const uint32_t vdst = smem_u32(smem + T::OFF_V + vs * T::V_TILE);
            for (int bx = 0; bx < nbox_v; ++bx)
                tma_load_4d(vdst + bx * T::K_BOX_BYTES, tmV, bar(Bars::V_FULL + vs), I.dv0 + bx * T::BOX,
                            j * T::BC, vh, vb, pol_kv);
            vfill[vs]++;
            ++iv;
        }
    }
    if (!ok) {
        // unwind: let every issued copy land before the CTA can exit
        for (int s = 0; s < T::NSK; ++s)
            if (kfill[s] > 0) mbar_wait_drain(bar(Bars::K_FULL + s), (kfill[s] - 1) & 1);
        for (int s = 0; s < T::NSV; ++s)
            if (vfill[s] > 0) mbar_wait_drain(bar(Bars::V_FULL + s), (vfill[s] - 1) & 1);
    }
}

// ------------------------------------------------------------------- MMA
// Shared-memory descriptors of the MMA operands, built once per CTA: a tile's
// descriptor is its base descriptor plus (byte offset >> 4) in the 14-bit
// start-address field (shared addresses stay below 2^18 bytes, so the field
// never carries), which keeps the MMA issuer at one add per operand.
template <class T>
struct Descs {
    uint64_t q0;  // Q tile 0 (K-major)
    uint64_t k0;  // K ring slot 0 (K-major)
    uint64_t v0;  // V ring slot 0 (MN-major)
    __device__ __forceinline__ explicit Descs(uint8_t* smem) {
        q0 = smem_desc(smem_u32(smem + T::OFF_Q), 16, 8 * T::SW, T::LAYOUT);
        k0 = smem_desc(smem_u32(smem + T::OFF_K), 16, 8 * T::SW, T::LAYOUT);
        // MN-major V: 8-key atoms SBO = 8*SW apart, box (BOX columns) LBO = BC*SW apart
        v0 = smem_desc(smem_u32(smem + T::OFF_V), T::BC * T::SW, 8 * T::SW, T::LAYOUT);
    }
};

template <class T>
__device__ __forceinline__ void issue_qk(const Descs<T>& dz, uint32_t tmem, int t, int kslot, int sb = 0) {
    const uint64_t qa = dz.q0 + static_cast<uint32_t>(t * (T::Q_TILE >> 4));
    const uint64_t kb = dz.k0 + static_cast<uint32_t>(kslot * (T::K_TILE >> 4));
    const uint32_t d = tmem + T::S_COL0 + (t * T::NSB + sb) * T::BC;
#pragma unroll
    for (int kk = 0; kk < T::D / T::KSTEP; ++kk) {
        const int box = kk / T::STEPS_PER_BOX, sub = kk % T::STEPS_PER_BOX;
        const uint64_t ad = qa + static_cast<uint32_t>((box * T::Q_BOX_BYTES + sub * 32) >> 4);
        const uint64_t bd = kb + static_cast<uint32_t>((box * T::K_BOX_BYTES + sub * 32) >> 4);
        if constexpr (T::I8)
            mma_i8_ss(d, ad, bd, T::IDESC_QK, kk > 0 ? 1u : 0u);
        else
            mma_f16_ss(d, ad, bd, T::IDESC_QK, kk > 0 ? 1u : 0u);
    }
}

template <class T>
__device__ __forceinline__ void issue_pv(const Descs<T>& dz, uint32_t tmem, int t, int vslot, bool accumulate,
                                         uint32_t idesc_pv, int sb = 0) {
    const uint64_t vb = dz.v0 + static_cast<uint32_t>(vslot * (T::V_TILE >> 4));
    const uint32_t a_base = tmem + T::S_COL0 + (t * T::NSB + sb) * T::BC;  // P aliases S
    const uint32_t d = tmem + (T::I8 ? T::ACC_COL0 : T::O_COL0) + t * T::DVMAX;
#pragma unroll
    for (int kk = 0; kk < T::BC / T::KSTEP; ++kk) {
        const uint64_t bd = vb + static_cast<uint32_t>((kk * T::KSTEP * T::SW) >> 4);
        const uint32_t acc = (kk > 0 || accumulate) ? 1u : 0u;
        if constexpr (T::I8)
            mma_i8_ts(d, a_base + kk * 8, bd, idesc_pv, acc);
        else
            mma_f16_ts(d, a_base + kk * 8, bd, idesc_pv, acc);
    }
}

// Double-buffered S: S(t, j) lives in buffer (g + j - ta[t]) & 1, g = blocks of
// tile t in this CTA's earlier items.  Per item the prologue issues QK for the
// first two blocks; block j then issues, per tile, PV(j) (after P(t, j) is
// published) and QK(j+2) into the buffer PV(j) just read (tcgen05 MMAs from
// one thread run in issue order).  The softmax of block j+1 meanwhile works
// on the other buffer, so a tile's softmax never waits for the tensor core
// except for S itself.  An item's first PV overwrites O, so it waits until the
// epilogue of the tile's previous item has read O out of TMEM.
template <class T>
__device__ void mma_role_sdb(const Params& p, uint8_t* smem, uint32_t tmem, const Abort& ab, int issuer) {
    // issuer i serves tiles [t_begin, t_end)
    const int t_begin = T::NI == 1 ? 0 : issuer;
    const int t_end = T::NI == 1 ? T::NT : issuer + 1;
    const uint32_t bars = smem_u32(smem);
    auto bar = [&](int i) { return bars + 8u * static_cast<uint32_t>(i); };
    const Descs<T> dz(smem);
    int kc = 0, vc = 0, n = 0;
    int g[2] = {0, 0}, n_o[2] = {0, 0};
    bool ok = true;
    for (; ok && n < 1; ++n) {
        const int item = item_at(p, n);
        if (item < 0) break;
        const Item I = make_item<T>(p, item);
        const int* ta = I.ta;
        const int* te = I.te;
        const int jlo = I.jlo, jhi = I.jhi;
        const uint32_t idesc_pv =
            instr_desc(T::I8 ? 2u : 1u, T::I8 ? 1u : 0u, 1u, BM, static_cast<uint32_t>(I.dv));
        if (!mbar_wait(bar(Bars::Q_FULL), n & 1, ab, SITE_MMA_Q)) {
            ok = false;
            break;
        }
        if constexpr (T::ROPE_Q) {
            // the softmax warps rotate Q in place before the first Q K^T
            if (p.rope_q && !mbar_wait(bar(Bars::Q_ROT), n & 1, ab, SITE_MMA_QROT)) {
                ok = false;
                break;
            }
        }
        tc_fence_after();
        for (int jj = jlo; jj < jhi && jj < jlo + 2; ++jj) {
            const int ks = kc % T::NSK;
            if (!mbar_wait(bar(Bars::K_FULL + ks), (kc / T::NSK) & 1, ab, SITE_MMA_K)) {
                ok = false;
                break;
            }
            tc_fence_after();
            for (int t = t_begin; t < t_end; ++t) {
                if (ta[t] <= jj && jj < te[t]) {
                    const int sb = (g[t] + jj - ta[t]) & 1;
                    issue_qk<T>(dz, tmem, t, ks, sb);
                    tc_commit(bar(Bars::S_FULL + t * T::NSB + sb));
                }
            }
            tc_commit(bar(Bars::K_EMPTY + ks));
            kc++;
        }
        // Q is released as soon as this issuer's last Q K^T of the item is
        // issued (the commit fires when those MMAs complete), so the next
        // item's Q loads while the last PVs run
        if (ok && jhi - jlo <= 2) tc_commit(bar(Bars::Q_EMPTY));
        for (int j = jlo; ok && j < jhi; ++j) {
            const int vs = vc % T::NSV;
            if (!mbar_wait(bar(Bars::V_FULL + vs), (vc / T::NSV) & 1, ab, SITE_MMA_V)) {
                ok = false;
                break;
            }
            const bool has_k = j + 2 < jhi;
            const int ks = kc % T::NSK;
            if (has_k && !mbar_wait(bar(Bars::K_FULL + ks), (kc / T::NSK) & 1, ab, SITE_MMA_K)) {
                ok = false;
                break;
            }
            tc_fence_after();
            for (int t = t_begin; t < t_end; ++t) {
                if (ta[t] <= j && j < te[t]) {
                    const int it = j - ta[t];
                    const int gg = g[t] + it;
                    const int sb = gg & 1;
                    if (!mbar_wait(bar(Bars::P_FULL + t * T::NSB + sb), (gg >> 1) & 1, ab, SITE_MMA_P)) {
                        ok = false;
                        break;
                    }

                    if (it == 0 && n_o[t] > 0 &&
                        !mbar_wait(bar(Bars::O_EMPTY + t), (n_o[t] - 1) & 1, ab, SITE_MMA_OEMPTY)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    issue_pv<T>(dz, tmem, t, vs, it > 0, idesc_pv, sb);
                    tc_commit(bar(Bars::PV_DONE + t));
                    if (j == te[t] - 1) tc_commit(bar(Bars::O_FULL + t));
                }
                if (has_k && ta[t] <= j + 2 && j + 2 < te[t]) {
                    const int sb = (g[t] + j + 2 - ta[t]) & 1;
                    issue_qk<T>(dz, tmem, t, ks, sb);
                    tc_commit(bar(Bars::S_FULL + t * T::NSB + sb));
                }
            }
            if (!ok) break;
            tc_commit(bar(Bars::V_EMPTY + vs));
            vc++;
            if (has_k) {
                tc_commit(bar(Bars::K_EMPTY + ks));
                kc++;
                if (j + 2 == jhi - 1) tc_commit(bar(Bars::Q_EMPTY));
            }
        }
        if (!ok) break;
        for (int t = t_begin; t < t_end; ++t) {
            g[t] += te[t] - ta[t];
            n_o[t] += te[t] > ta[t] ? 1 : 0;
        }
    }
    tc_commit(bar(Bars::DRAIN + issuer));
    mbar_wait_drain(bar(Bars::DRAIN + issuer), 0);
}

template <class T>
__device__ void mma_role(const Params& p, uint8_t* smem, uint32_t tmem, const Abort& ab) {
    const uint32_t bars = smem_u32(smem);
    auto bar = [&](int i) { return bars + 8u * static_cast<uint32_t>(i); };
    const Descs<T> dz(smem);
    int kc = 0, vc = 0, n = 0;
    int pc[2] = {0, 0}, n_o[2] = {0, 0};
    bool ok = true;
    for (; ok && n < 1; ++n) {
        const int item = item_at(p, n);
        if (item < 0) break;
        const Item I = make_item<T>(p, item);
        const int* ta = I.ta;
        const int* te = I.te;
        const int jlo = I.jlo, jhi = I.jhi;
        const uint32_t idesc_pv =
            instr_desc(T::I8 ? 2u : 1u, T::I8 ? 1u : 0u, 1u, BM, static_cast<uint32_t>(I.dv));
        if (!mbar_wait(bar(Bars::Q_FULL), n & 1, ab, SITE_MMA_Q)) {
            ok = false;
            break;
        }
        tc_fence_after();
        if (jlo < jhi) {
            const int ks = kc % T::NSK;
            if (!mbar_wait(bar(Bars::K_FULL + ks), (kc / T::NSK) & 1, ab, SITE_MMA_K)) {
                ok = false;
                break;
            }
            tc_fence_after();
            for (int t = 0; t < T::NT; ++t) {
                if (ta[t] <= jlo && jlo < te[t]) {
                    issue_qk<T>(dz, tmem, t, ks);
                    tc_commit(bar(Bars::S_FULL + t));
                }
            }
            tc_commit(bar(Bars::K_EMPTY + ks));
            kc++;
        }
        if (ok && jhi - jlo <= 1) tc_commit(bar(Bars::Q_EMPTY));  // last Q K^T of the item issued
        for (int j = jlo; ok && j < jhi; ++j) {
            const int vs = vc % T::NSV;
            if (!mbar_wait(bar(Bars::V_FULL + vs), (vc / T::NSV) & 1, ab, SITE_MMA_V)) {
                ok = false;
                break;
            }
            const bool has_next = j + 1 < jhi;
            const int ks = kc % T::NSK;
            if (has_next && !mbar_wait(bar(Bars::K_FULL + ks), (kc / T::NSK) & 1, ab, SITE_MMA_K)) {
                ok = false;
                break;
            }
            tc_fence_after();
            for (int t = 0; t < T::NT; ++t) {
                const bool act = ta[t] <= j && j < te[t];
                const bool act_next = has_next && ta[t] <= j + 1 && j + 1 < te[t];
                if (act) {
                    if (!mbar_wait(bar(Bars::P_FULL + t), pc[t] & 1, ab, SITE_MMA_P)) {
                        ok = false;
                        break;
                    }
                    pc[t]++;
                    if (j == ta[t] && n_o[t] > 0 &&
                        !mbar_wait(bar(Bars::O_EMPTY + t), (n_o[t] - 1) & 1, ab, SITE_MMA_OEMPTY)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    issue_pv<T>(dz, tmem, t, vs, j > ta[t], idesc_pv);
                    if (j == te[t] - 1) tc_commit(bar(Bars::O_FULL + t));
                }
                if (act_next) {
                    issue_qk<T>(dz, tmem, t, ks);
                    tc_commit(bar(Bars::S_FULL + t));
                }
            }
            if (!ok) break;
            tc_commit(bar(Bars::V_EMPTY + vs));
            vc++;
            if (has_next) {
                tc_commit(bar(Bars::K_EMPTY + ks));
                kc++;
                if (j + 1 == jhi - 1) tc_commit(bar(Bars::Q_EMPTY));
            }
        }
        if (!ok) break;
        for (int t = 0; t < T::NT; ++t) n_o[t] += te[t] > ta[t] ? 1 : 0;
    }
    // drain: no MMA may still be writing TMEM when the CTA releases it
    tc_commit(bar(Bars::DRAIN));
    mbar_wait_drain(bar(Bars::DRAIN), 0);
}

// ------------------------------------------------- INT8, two passes over K
// Softmax warpgroup of tile t for T::TWOPASS.  Key blocks are visited twice in
// one sequence of S buffers (virtual block v = pass * n + it, S in buffer v & 1):
//   pass 1: S -> the row's exact max over every visible key (no exponentials);
//           the arrival on P_FULL only hands the S buffer back to the MMA issuer;
//   pass 2: S -> p = exp2(s * scale * log2(e) - max) <= 1, Pq = round(127 p)
//           written over S for the int8 P V MMA, row sum of the unrounded p.
// Pq is quantised against the row's global max (the reference gate's own
// semantics, tests/hip_forward_int8qk_gate.hip:69-120), so the s32 accumulator
// is never rescaled and O = ACC * v_scale / 127 / l at the end.
template <class T>
__device__ void softmax_role_i8x2(const Params& p, const CUtensorMap* tmO, int t, uint8_t* smem, uint32_t tmem,
                                  const Abort& ab, const PeerMaps* pm) {
    const int warp = threadIdx.x / 32;
    const int lane = threadIdx.x % 32;
    const int wq = warp % 4;
    const int r = wq * 32 + lane;
    const uint32_t lane_base = static_cast<uint32_t>(wq * 32) << 16;
    const uint32_t tS0 = tmem + lane_base + T::S_COL0 + t * T::NSB * T::BC;
    const uint32_t tACC = tmem + lane_base + T::ACC_COL0 + t * T::DVMAX;
    const uint32_t bars = smem_u32(smem);
    auto bar = [&](int i) { return bars + 8u * static_cast<uint32_t>(i); };
    bool aborted = false;

    const int item = item_at(p, 0);
    if (item < 0) return;
    const Item I = make_item<T>(p, item);
    const Work& w = I.w;
    if (!w.valid[t]) return;  // uniform for the warpgroup
    const int dv = I.dv, dv0 = I.dv0;
    const int row0 = w.row0[t];
    const int q = row0 + r;
    const int a = I.ta[t], e = I.te[t];
    const int n = e - a;
    int klo, khi;
    row_keys(p, q, klo, khi);
    const int other_iters = T::TOKEN ? I.te[1 - t] - I.ta[1 - t] : 0;

    const bool kvec = p.k_vec != nullptr;
    float qs = p.q_scale;
    if (p.q_vec != nullptr && q < p.S) qs = p.q_vec[(static_cast<int64_t>(w.b) * p.H + w.head[t]) * p.S + q];
    float rowscale = qs * p.scale_log2;
    if (!kvec) rowscale *= p.k_scale;
    const bool neg = rowscale < 0.f;  // then x is negated so that max(x) * |rowscale| is the max
    const float ars = fabsf(rowscale);
    float* ksbuf = reinterpret_cast<float*>(smem + T::OFF_KSCALE) + t * 2 * T::BC;
    const float* kvec_row = kvec ? p.k_vec + (static_cast<int64_t>(w.b) * p.Hkv + w.kvh) * p.KS : nullptr;
    auto load_ks = [&](int jb) {
        const int key = jb * T::BC + r;
        return (kvec && r < T::BC && jb < e && key < p.KS) ? __ldg(kvec_row + key) : 0.f;
    };
    float ks_next = load_ks(a);

    float m = -INFINITY;  // the row's max of s * rowscale (log2 domain), complete after pass 1
    float l = 0.f;
    for (int v = 0; v < 2 * n; ++v) {
        const bool second = v >= n;
        const int it = second ? v - n : v;
        const int j = a + it;
        if (kvec) {
            // stage this block's per-key scales; buffer (v & 1) is reused every second block
            const int buf = v & 1;
            if (r < T::BC) ksbuf[buf * T::BC + r] = ks_next;
            mbar_arrive(bar(Bars::KS_FULL + 2 * t + buf));
            ks_next = load_ks(it + 1 < n ? j + 1 : a);
            if (!aborted && !warp_wait(bar(Bars::KS_FULL + 2 * t + buf), (v >> 1) & 1, ab, SITE_SM_KS))
                aborted = true;
        }
        const int sb = v % T::NSB;
        const uint32_t tS = tS0 + sb * T::BC;
        if (!aborted && !warp_wait(bar(Bars::S_FULL + t * T::NSB + sb), (v / T::NSB) & 1, ab, SITE_SM_S))
            aborted = true;
        if (aborted) continue;
        tc_fence_after();

        if constexpr (T::DUMP_S) {
            if (second) {
                // debug: the raw s32 scores, read 16 columns at a time (warp-wide loads)
                int32_t* dst = p.s_dump + ((static_cast<int64_t>(w.b) * p.H + w.head[t]) * p.S + q) * p.KS;
                for (int c0 = 0; c0 < T::BC; c0 += 16) {
                    uint32_t d16[16];
                    tmem_ld_x16(tS + c0, d16);
#pragma unroll
                    for (int c = 0; c < 16; ++c)
                        if (q < p.S && j * T::BC + c0 + c < p.KS)
                            dst[j * T::BC + c0 + c] = static_cast<int32_t>(d16[c]);
                }
            }
        }
        uint32_t raw[T::BC];
        load_s_row<T>(tS, raw);
        // s32 -> float by cvt.rn (exact: |q.k| <= 127*127*D < 2^22), times the key
        // scale, negated for a negative row scale, masked outside the row's keys
        float* x = reinterpret_cast<float*>(raw);
        const float* ksb = ksbuf + (v & 1) * T::BC;
        if (kvec) {
#pragma unroll
            for (int c = 0; c < T::BC; c += 4) {
                const float4 k4 = *reinterpret_cast<const float4*>(ksb + c);
                const uint64_t u0 = f2(s32_to_f32(raw[c]), s32_to_f32(raw[c + 1]));
                const uint64_t u1 = f2(s32_to_f32(raw[c + 2]), s32_to_f32(raw[c + 3]));
                f2_split(fmul2(u0, f2(k4.x, k4.y)), x[c], x[c + 1]);
                f2_split(fmul2(u1, f2(k4.z, k4.w)), x[c + 2], x[c + 3]);
            }
        } else {
#pragma unroll
            for (int c = 0; c < T::BC; ++c) x[c] = s32_to_f32(raw[c]);
        }
        if (neg) {
#pragma unroll
            for (int c = 0; c < T::BC; ++c) x[c] = -x[c];
        }
        if (!block_full<T>(p, row0, j)) {
            const int lo = klo - j * T::BC, hi = khi - j * T::BC;
#pragma unroll
            for (int c = 0; c < T::BC; ++c)
                if (c < lo || c > hi) x[c] = -INFINITY;
        }

        if (!second) {
            float mx = row_max<T::BC>(x) * ars;
            if (mx != mx) mx = -INFINITY;  // fully masked with a zero row scale
            m = fmaxf(m, mx);
        } else {
            // exponent phases of the two tiles alternate on each scheduler's MUFU
            if constexpr (T::TOKEN) {
                const int need = it - 1 + t;
                if (need >= 0 && need < other_iters &&
                    !warp_wait(bar(Bars::EXPD + (1 - t) * 4 + wq), need & 1, ab, SITE_SM_TOKEN)) {
                    aborted = true;
                    continue;
                }
            }
            // p two at a time in half precision (P keeps 7 bits): fma(p, 127, 1024) in
            // fp16 has unit spacing, so its low byte is round(p * 127) (to nearest even; the
            // reference's lround differs only at exact .5 ties).  Row sums accumulate in 8
            // f16x2 partials (<= BC / 8 values each) and finish in fp32.
            const float neg_m = (m == -INFINITY) ? 0.f : -m;
            const uint64_t ars2 = f2(ars, ars), nm2 = f2(neg_m, neg_m);
            constexpr uint32_t k127 = 0x57F057F0u;   // (127, 127) in f16x2
            constexpr uint32_t k1024 = 0x64006400u;  // (1024, 1024)
            uint32_t hs[8] = {0u, 0u, 0u, 0u, 0u, 0u, 0u, 0u};
#pragma unroll
            for (int c0 = 0; c0 < T::BC; c0 += 32) {
                uint32_t pk[8];
#pragma unroll
                for (int c = 0; c < 32; c += 4) {
                    float a0, a1, a2, a3;
                    f2_split(ffma2(f2(x[c0 + c], x[c0 + c + 1]), ars2, nm2), a0, a1);
                    f2_split(ffma2(f2(x[c0 + c + 2], x[c0 + c + 3]), ars2, nm2), a2, a3);
                    const uint32_t e0 = ex2_h2(pack_half2(a0, a1));
                    const uint32_t e1 = ex2_h2(pack_half2(a2, a3));
                    hs[(c >> 2) & 7] = hadd2(hs[(c >> 2) & 7], hadd2(e0, e1));
                    pk[c / 4] = pack_half_low_bytes(hfma2(e0, k127, k1024), hfma2(e1, k127, k1024));
                }
                tmem_st_x8(tS + c0 / 4, pk);
            }
            float ls[8];
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                const __half2 h = *reinterpret_cast<const __half2*>(&hs[i]);
                ls[i] = __low2float(h) + __high2float(h);
            }
            l += ((ls[0] + ls[1]) + (ls[2] + ls[3])) + ((ls[4] + ls[5]) + (ls[6] + ls[7]));
            if constexpr (T::TOKEN) {
                __syncwarp();
                if (lane == 0) mbar_arrive(bar(Bars::EXPD + t * 4 + wq));
            }
            tmem_wait_st();
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(bar(Bars::P_FULL + t * T::NSB + sb));
    }

    // ---------------------------------------------------------------- epilogue
    const bool has_blocks = n > 0;
    if (!aborted && has_blocks && !warp_wait(bar(Bars::O_FULL + t), 0, ab, SITE_SM_O)) aborted = true;
    if (!aborted) tc_fence_after();
    uint8_t* stage = smem + T::OFF_O + t * T::O_STRIDE;
    if (!aborted) {
        // O = ACC * (v_scale / 127) / l (times the per-channel V scale when given)
        const float f = (l > 0.f) ? p.pv_scale / l : 0.f;
        for (int c0 = 0; c0 < dv; c0 += 32) {
            float o[32];
            if (has_blocks) {
                uint32_t acc[32];
                tmem_ld_x32(tACC + c0, acc);
#pragma unroll
                for (int i = 0; i < 32; ++i) o[i] = static_cast<float>(static_cast<int>(acc[i])) * f;
                if (p.v_chan != nullptr) {
                    // per-channel V dequantisation, folded in before the one fp16 rounding
                    const float* vc = p.v_chan + (static_cast<int64_t>(w.b) * p.Hkv + w.kvh) * T::D + dv0 + c0;
#pragma unroll
                    for (int i = 0; i < 32; ++i) o[i] *= __ldg(vc + i);
                }
            } else {
#pragma unroll
                for (int i = 0; i < 32; ++i) o[i] = 0.f;
            }
#pragma unroll
            for (int g4 = 0; g4 < 4; ++g4) {
                uint4 u;
                u.x = pack_half2(o[8 * g4 + 0], o[8 * g4 + 1]);
                u.y = pack_half2(o[8 * g4 + 2], o[8 * g4 + 3]);
                u.z = pack_half2(o[8 * g4 + 4], o[8 * g4 + 5]);
                u.w = pack_half2(o[8 * g4 + 6], o[8 * g4 + 7]);
                const int col = c0 + 8 * g4;
                const int box = col / T::O_BOX;
                const int chunk = (col % T::O_BOX) / 8;
                *reinterpret_cast<uint4*>(stage + box * T::O_BOX_BYTES + swz_off<T::O_SW>(r, chunk)) = u;
            }
        }
        fence_proxy_async_smem();
    }
    mbar_arrive(bar(Bars::EPI + t));
    if (r == 0) {
        if (!aborted && mbar_wait(bar(Bars::EPI + t), 0, ab, SITE_SM_EPI) && !*ab.flag) {
            const int nbox = dv / T::O_BOX;
            for (int bx = 0; bx < nbox; ++bx)
                tma_store_4d(tmO, smem_u32(stage + bx * T::O_BOX_BYTES), dv0 + bx * T::O_BOX, row0, w.head[t], w.b);
            if constexpr (!T::DUMP_S) {  // (debug score dumps take no output replicas)
                // the same boxes into every peer's output: the TMA engine carries them
                // over NVLink while this CTA exits and the next one computes
                for (int k = 0; k < p.n_peer; ++k)
                    for (int bx = 0; bx < nbox; ++bx)
                        tma_store_4d(&pm->m[k], smem_u32(stage + bx * T::O_BOX_BYTES), dv0 + bx * T::O_BOX, row0,
                                     w.head[t], w.b);
            }
            bulk_commit();
        }
        bulk_wait_read_all();  // the stores have read the staging buffer before the CTA exits
    }
}

// MMA issuer of the two-pass INT8 kernel (one per tile): Q K^T over the tile's
// key blocks twice, in the virtual-block order of softmax_role_i8x2, with S
// double-buffered; S(v + 2) is issued once the softmax has handed S(v) back
// (pass 1) or once P V(v) has been issued after it (pass 2: tcgen05 MMAs of
// one thread run in order, so P V(v) reads P before Q K^T(v + 2) overwrites).
// K ring slots are shared by both issuers and freed after both commit.
template <class T>
__device__ void mma_role_i8x2(const Params& p, uint8_t* smem, uint32_t tmem, const Abort& ab, int issuer) {
    const int t = T::NI == 1 ? 0 : issuer;  // tile of this issuer (NT == 1: issuer 0 only)
    const uint32_t bars = smem_u32(smem);
    auto bar = [&](int i) { return bars + 8u * static_cast<uint32_t>(i); };
    const Descs<T> dz(smem);
    bool ok = true;
    const int item = item_at(p, 0);
    if (item >= 0) {
        const Item I = make_item<T>(p, item);
        const int jlo = I.jlo, N = I.jhi - I.jlo;
        const int ta = I.ta[t], te = I.te[t];
        const uint32_t idesc_pv = instr_desc(2u, 1u, 1u, BM, static_cast<uint32_t>(I.dv));
        // virtual block u over the union of the tiles' ranges, twice; this tile's own
        // virtual block index (its S buffer sequence) is vt(u)
        auto active = [&](int u) { const int j = jlo + (u % N); return ta <= j && j < te; };
        auto vt = [&](int u) { const int j = jlo + (u % N); return (u >= N ? te - ta : 0) + (j - ta); };
        ok = mbar_wait(bar(Bars::Q_FULL), 0, ab, SITE_MMA_Q);
        if (ok) tc_fence_after();
        int kc = 0, vc = 0;
        auto issue_k = [&](int u) -> bool {  // Q K^T of virtual block u (K slot kc), if this tile has it
            const int ks = kc % T::NSK;
            if (!mbar_wait(bar(Bars::K_FULL + ks), (kc / T::NSK) & 1, ab, SITE_MMA_K)) return false;
            tc_fence_after();
            if (active(u)) {
                const int sb = vt(u) % T::NSB;
                issue_qk<T>(dz, tmem, t, ks, sb);
                tc_commit(bar(Bars::S_FULL + t * T::NSB + sb));
            }
            tc_commit(bar(Bars::K_EMPTY + ks));
            kc++;
            return true;
        };
        for (int u = 0; ok && u < T::NSB && u < 2 * N; ++u) ok = issue_k(u);
        for (int u = 0; ok && u < 2 * N; ++u) {
            const bool second = u >= N;
            int vs = 0;
            if (second) {
                vs = vc % T::NSV;
                if (!mbar_wait(bar(Bars::V_FULL + vs), (vc / T::NSV) & 1, ab, SITE_MMA_V)) {
                    ok = false;
                    break;
                }
            }
            if (active(u)) {
                const int v = vt(u), sb = v % T::NSB;
                if (!mbar_wait(bar(Bars::P_FULL + t * T::NSB + sb), (v / T::NSB) & 1, ab, SITE_MMA_P)) {
                    ok = false;
                    break;
                }
                if (second) {
                    tc_fence_after();
                    const int j = jlo + (u - N);
                    issue_pv<T>(dz, tmem, t, vs, j > ta, idesc_pv, sb);
                    if (j == te - 1) tc_commit(bar(Bars::O_FULL + t));
                }
            }
            if (second) {
                tc_commit(bar(Bars::V_EMPTY + vs));
                vc++;
            }
            if (u + T::NSB < 2 * N) ok = issue_k(u + T::NSB);
        }
        if (ok) tc_commit(bar(Bars::Q_EMPTY));
    }
    tc_commit(bar(Bars::DRAIN + issuer));
    mbar_wait_drain(bar(Bars::DRAIN + issuer), 0);
}

// ---------------------------------------------------------------- kernel
template <class T>
__global__ void __launch_bounds__(T::THREADS, T::MIN_BLOCKS)
    fa_prefill_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                      const __grid_constant__ CUtensorMap tmV, const __grid_constant__ CUtensorMap tmO,
                      const __grid_constant__ PeerMaps pm, const __grid_constant__ Params p) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    const int warp = threadIdx.x / 32;
    const uint32_t bars = smem_u32(smem);
    auto bar = [&](int i) { return bars + 8u * static_cast<uint32_t>(i); };
    volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + Bars::ABORT_SLOT);
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + Bars::TMEM_SLOT);

    if (threadIdx.x == 0) {
        *abort_flag = 0;
        mbar_init(bar(Bars::Q_FULL), 1);
        mbar_init(bar(Bars::DRAIN), 1);
        mbar_init(bar(Bars::DRAIN + 1), 1);
        for (int s = 0; s < T::NSK; ++s) {
            mbar_init(bar(Bars::K_FULL + s), 1);
            mbar_init(bar(Bars::K_EMPTY + s), T::NI);
        }
        for (int s = 0; s < T::NSV; ++s) {
            mbar_init(bar(Bars::V_FULL + s), 1);
            mbar_init(bar(Bars::V_EMPTY + s), T::NI);
        }
        for (int t = 0; t < T::NT; ++t) {
            for (int sb = 0; sb < T::NSB; ++sb) {
                mbar_init(bar(Bars::S_FULL + t * T::NSB + sb), 1);
                mbar_init(bar(Bars::P_FULL + t * T::NSB + sb), 4);
            }
            mbar_init(bar(Bars::O_FULL + t), 1);
            mbar_init(bar(Bars::PV_DONE + t), 1);
            mbar_init(bar(Bars::KS_FULL + 2 * t), 128);
            mbar_init(bar(Bars::KS_FULL + 2 * t + 1), 128);
            mbar_init(bar(Bars::EPI + t), 128);
            for (int q = 0; q < 4; ++q) mbar_init(bar(Bars::EXPD + t * 4 + q), 1);
        }
        mbar_init(bar(Bars::Q_EMPTY), T::NI);
        mbar_init(bar(Bars::Q_ROT), 4 * T::NT);
        for (int t = 0; t < T::NT; ++t) {
            mbar_init(bar(Bars::O_EMPTY + t), 4);
            mbar_init(bar(Bars::STG_FREE + t), 1);
        }
        fence_barrier_init();
    }
    if (warp == T::WARP_MMA) {
        tmem_alloc(smem_u32(tmem_slot), T::TMEM_COLS);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    const Abort ab{abort_flag, (p.dbg_withhold >= 0 && blockIdx.x == 0) ? p.dbg_wait_limit_ns : kWaitLimitNs};

    if constexpr (T::RESPLIT) {
        if (warp < 4 * T::NT)
            regs_increase<T::SOFTMAX_REGS>();
        else
            regs_decrease<T::CONTROL_REGS>();
    }
    if (warp < 4 * T::NT) {
        if constexpr (T::TWOPASS)
            softmax_role_i8x2<T>(p, &tmO, warp / 4, smem, tmem, ab, &pm);
        else
            softmax_role<T>(p, &tmO, warp / 4, smem, tmem, ab, &pm);
        tc_fence_before();
    } else if (warp == T::WARP_PROD) {
        if (sm100::lane_id() == 0) producer_kv_role<T>(p, &tmK, &tmV, smem, ab);
        __syncwarp();
    } else if (warp == T::WARP_QLOAD) {
        if (sm100::lane_id() == 0) producer_q_role<T>(p, &tmQ, smem, ab);
        __syncwarp();
    } else if (warp == T::WARP_MMA) {
        if (sm100::lane_id() == 0) {
            if constexpr (T::TWOPASS)
                mma_role_i8x2<T>(p, smem, tmem, ab, 0);
            else if constexpr (T::SDB)
                mma_role_sdb<T>(p, smem, tmem, ab, 0);
            else
                mma_role<T>(p, smem, tmem, ab);
        }
        __syncwarp();
    } else if (T::NI == 2 && warp == T::WARP_MMA + 1) {
        if constexpr (T::TWOPASS) {
            if (sm100::lane_id() == 0) mma_role_i8x2<T>(p, smem, tmem, ab, 1);
        } else if constexpr (T::SDB) {
            if (sm100::lane_id() == 0) mma_role_sdb<T>(p, smem, tmem, ab, 1);
        }
        __syncwarp();
    }
    __syncthreads();
    if (warp == T::WARP_MMA) {
        tc_fence_after();
        tmem_dealloc(tmem, T::TMEM_COLS);
    }
}

}  // namespace prefill
}  // namespace rdna
