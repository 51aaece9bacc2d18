// Thin inline-PTX wrappers for the sm_100a features the attention kernels use:
// mbarriers (with bounded waits), TMA tensor loads/stores, tcgen05 MMA / TMEM
// management, and the UMMA shared-memory / instruction descriptors.
//
// Descriptor bit layouts follow the PTX ISA "tcgen05 matrix descriptors"
// (shared-memory descriptor: start>>4 @[0,14), LBO>>4 @[16,30), SBO>>4
// @[32,46), version=1 @[46,48), layout @[61,64); instruction descriptor for
// kind::f16 / kind::i8: D format @[4,6), A/B format @[7,10)/[10,13), A/B
// major @15/@16, N>>3 @[17,23), M>>4 @[24,29)).
#pragma once

#include <cstdint>
#include <cuda.h>

#include "tmem_ldst.cuh"

namespace rdna {
namespace sm100 {

#define RDNA_DEV __device__ __forceinline__

RDNA_DEV uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

RDNA_DEV uint64_t globaltimer_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

RDNA_DEV uint32_t lane_id() {
    uint32_t l;
    asm volatile("mov.u32 %0, %%laneid;" : "=r"(l));
    return l;
}

// ------------------------------------------------------------------ mbarrier

RDNA_DEV void mbar_init(uint32_t bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}

RDNA_DEV void fence_barrier_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

RDNA_DEV void mbar_arrive(uint32_t bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}

RDNA_DEV void mbar_arrive_expect_tx(uint32_t bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
}

RDNA_DEV bool mbar_try_wait(uint32_t bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}\n"
        : "=r"(ok)
        : "r"(bar), "r"(parity)
        : "memory");
    return ok != 0;
}

// Every wait in the kernels is bounded: a wait that has not completed after
// kWaitLimitNs sets the CTA-wide abort flag (shared memory) and a device
// status word, then returns false so the caller can unwind.  Once the abort
// flag is set, every other wait in the CTA returns false immediately.
constexpr uint64_t kWaitLimitNs = 2000000000ull;  // 2 s

struct Abort {
    volatile int* flag;                 // shared, CTA-wide
    uint64_t limit_ns = kWaitLimitNs;   // per-wait limit (a debug launch may shorten it)
};

}  // namespace sm100
}  // namespace rdna

// Device status word of the module: [0] = first error code recorded by an
// expired wait, [1] = number of such events.  This header is included by a
// single translation unit (forward.cu, which holds every kernel), so the
// definition lives here.
__device__ int g_rdna_status[2];

namespace rdna {
namespace sm100 {

RDNA_DEV void record_error(const Abort& ab, int code) {
    *ab.flag = 1;
    atomicCAS(&g_rdna_status[0], 0, code);
    atomicAdd(&g_rdna_status[1], 1);
}

// try_wait with an explicit suspend-time hint: a thread whose phase is not yet
// complete is parked (woken when the phase completes, or after hint_ns) instead
// of returning at once, so waiting warps do not take issue slots from the
// warps that share their scheduler.
RDNA_DEV bool mbar_try_wait_suspend(uint32_t bar, uint32_t parity, uint32_t hint_ns) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}\n"
        : "=r"(ok)
        : "r"(bar), "r"(parity), "r"(hint_ns)
        : "memory");
    return ok != 0;
}

constexpr uint32_t kSuspendHintNs = 20000;  // 20 us per parked try_wait

RDNA_DEV bool mbar_wait(uint32_t bar, uint32_t parity, const Abort& ab, int site) {
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = globaltimer_ns();
    while (true) {
        if (mbar_try_wait_suspend(bar, parity, kSuspendHintNs)) return true;
        if (*ab.flag) return false;
        if (globaltimer_ns() - t0 > ab.limit_ns) {
            record_error(ab, site);
            return false;
        }
    }
}

// Wait used on the unwind path only: ignores the abort flag, still bounded.
RDNA_DEV bool mbar_wait_drain(uint32_t bar, uint32_t parity) {
    const uint64_t t0 = globaltimer_ns();
    while (!mbar_try_wait(bar, parity)) {
        if (globaltimer_ns() - t0 > kWaitLimitNs) return false;
    }
    return true;
}

RDNA_DEV void named_bar_sync(int id, int nthreads) {
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}

// Programmatic dependent launch: waits until the grids this one was launched to
// overlap (cudaLaunchAttributeProgrammaticStreamSerialization) have completed and
// their memory is visible.  Returns at once for an ordinary launch.
RDNA_DEV void grid_dependency_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

// ----------------------------------------------------------------------- TMA

RDNA_DEV void prefetch_tmap(const CUtensorMap* m) {
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(m)) : "memory");
}

RDNA_DEV uint64_t policy_evict_last() {
    uint64_t p;
    asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(p));
    return p;
}

RDNA_DEV uint64_t policy_evict_first() {
    uint64_t p;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
    return p;
}

// 4-D tiled load into this CTA's shared memory, completion counted on `bar`.
// c0 (innermost, head_dim) must be a multiple of 16 bytes: callers pass box
// origins that are multiples of the 32- or 64-element box width.
RDNA_DEV void tma_load_4d(uint32_t dst, const CUtensorMap* m, uint32_t bar, int c0, int c1, int c2, int c3,
                          uint64_t policy) {
    asm volatile(
        "cp.async.bulk.tensor.4d.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
        " [%0], [%1, {%3, %4, %5, %6}], [%2], %7;"
        ::"r"(dst), "l"(reinterpret_cast<uint64_t>(m)), "r"(bar), "r"(c0), "r"(c1), "r"(c2), "r"(c3),
          "l"(policy)
        : "memory");
}

// 4-D tiled store from shared memory; rows beyond the tensor extent are clipped.
RDNA_DEV void tma_store_4d(const CUtensorMap* m, uint32_t src, int c0, int c1, int c2, int c3) {
    asm volatile("cp.async.bulk.tensor.4d.global.shared::cta.bulk_group [%0, {%2, %3, %4, %5}], [%1];"
                 ::"l"(reinterpret_cast<uint64_t>(m)), "r"(src), "r"(c0), "r"(c1), "r"(c2), "r"(c3)
                 : "memory");
}

RDNA_DEV void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
RDNA_DEV void bulk_wait_read_all() { asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory"); }
RDNA_DEV void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }
RDNA_DEV void fence_proxy_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

// ------------------------------------------------------------------- tcgen05

RDNA_DEV void tmem_alloc(uint32_t dst_smem, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(dst_smem), "r"(ncols)
                 : "memory");
}
RDNA_DEV void tmem_relinquish() {
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
RDNA_DEV void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
RDNA_DEV void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
RDNA_DEV void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
RDNA_DEV void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// Arrives once on `bar` when every tcgen05 async operation issued so far by
// this thread has completed.
RDNA_DEV void tc_commit(uint32_t bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar)
                 : "memory");
}

// D(tmem) (+)= A(smem desc) * B(smem desc)
RDNA_DEV void mma_f16_ss(uint32_t d, uint64_t a, uint64_t b, uint32_t idesc, uint32_t accum) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}\n"
        ::"r"(d), "l"(a), "l"(b), "r"(idesc), "r"(accum)
        : "memory");
}
// D(tmem) (+)= A(tmem) * B(smem desc)
RDNA_DEV void mma_f16_ts(uint32_t d, uint32_t a_tmem, uint64_t b, uint32_t idesc, uint32_t accum) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}\n"
        ::"r"(d), "r"(a_tmem), "l"(b), "r"(idesc), "r"(accum)
        : "memory");
}
RDNA_DEV void mma_i8_ss(uint32_t d, uint64_t a, uint64_t b, uint32_t idesc, uint32_t accum) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}\n"
        ::"r"(d), "l"(a), "l"(b), "r"(idesc), "r"(accum)
        : "memory");
}
RDNA_DEV void mma_i8_ts(uint32_t d, uint32_t a_tmem, uint64_t b, uint32_t idesc, uint32_t accum) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::i8 [%0], [%1], %2, %3, p;\n\t}\n"
        ::"r"(d), "r"(a_tmem), "l"(b), "r"(idesc), "r"(accum)
        : "memory");
}

// Shared-memory matrix descriptor.  layout: 2 = 128B swizzle, 4 = 64B swizzle.
RDNA_DEV uint64_t smem_desc(uint32_t saddr, uint32_t lbo_bytes, uint32_t sbo_bytes, uint32_t layout) {
    uint64_t d = 0;
    d |= static_cast<uint64_t>((saddr >> 4) & 0x3FFFu);
    d |= static_cast<uint64_t>((lbo_bytes >> 4) & 0x3FFFu) << 16;
    d |= static_cast<uint64_t>((sbo_bytes >> 4) & 0x3FFFu) << 32;
    d |= static_cast<uint64_t>(1) << 46;
    d |= static_cast<uint64_t>(layout & 7u) << 61;
    return d;
}

// Instruction descriptor.  c_fmt: 1 = f32, 2 = s32.  ab_fmt: 0 = f16, 1 = s8
// (for kind::i8).  b_mn_major: B operand stored MN-major (N contiguous).
__host__ __device__ constexpr uint32_t instr_desc(uint32_t c_fmt, uint32_t ab_fmt, uint32_t b_mn_major, uint32_t M,
                                                  uint32_t N) {
    return (c_fmt << 4) | (ab_fmt << 7) | (ab_fmt << 10) | (0u << 15) | (b_mn_major << 16) | ((N >> 3) << 17) |
           ((M >> 4) << 24);
}

// Register re-split between warpgroups.  Must be executed by all four warps
// of a warpgroup; the sum over the CTA may not exceed the registers it was
// launched with (threads x registers per thread at launch).
template <int N>
RDNA_DEV void regs_increase() {
    asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(N));
}
template <int N>
RDNA_DEV void regs_decrease() {
    asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(N));
}

// --------------------------------------------------------------- math utils

RDNA_DEV float ex2(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

// Three-input max (sm_100).
RDNA_DEV float fmax3(float a, float b, float c) {
    float r;
    asm("max.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(a), "f"(b), "f"(c));
    return r;
}

// Two fp32 values in one 64-bit register: operands of sm_100's paired
// fp32 instructions (fma/add/mul .f32x2, one issue for both lanes).
RDNA_DEV uint64_t f2(float lo, float hi) {
    uint64_t r;
    asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
    return r;
}
RDNA_DEV void f2_split(uint64_t v, float& lo, float& hi) {
    asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(v));
}
RDNA_DEV uint64_t ffma2(uint64_t a, uint64_t b, uint64_t c) {
    uint64_t d;
    asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
    return d;
}
RDNA_DEV uint64_t fadd2(uint64_t a, uint64_t b) {
    uint64_t d;
    asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
    return d;
}
RDNA_DEV uint64_t fmul2(uint64_t a, uint64_t b) {
    uint64_t d;
    asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
    return d;
}

// int32 (a TMEM word) -> float, cvt.rn: exact for |v| <= 2^24.  The INT8 score
// conversion uses it (measured faster on sm_100 than the biased form below).
RDNA_DEV float s32_to_f32(uint32_t v) { return __int2float_rn(static_cast<int>(v)); }

// Exact int32 -> float for |v| < 2^22 on the ALU/FMA pipes: returns
// float(v) + 12582912 (the accumulator fold subtracts the bias in the same
// paired instruction that scales it).
RDNA_DEV float i2f_biased(uint32_t v) { return __int_as_float(static_cast<int>(v + 0x4B400000u)); }

// Bytes 0 of four words packed into one word (b0 lowest).
RDNA_DEV uint32_t pack_low_bytes(uint32_t b0, uint32_t b1, uint32_t b2, uint32_t b3) {
    uint32_t lo, hi, r;
    asm("prmt.b32 %0, %1, %2, 0x0040;" : "=r"(lo) : "r"(b0), "r"(b1));
    asm("prmt.b32 %0, %1, %2, 0x0040;" : "=r"(hi) : "r"(b2), "r"(b3));
    asm("prmt.b32 %0, %1, %2, 0x5410;" : "=r"(r) : "r"(lo), "r"(hi));
    return r;
}

// Packed half-precision helpers.
RDNA_DEV uint32_t ex2_h2(uint32_t x) {
    uint32_t y;
    asm("ex2.approx.f16x2 %0, %1;" : "=r"(y) : "r"(x));
    return y;
}
RDNA_DEV uint32_t hfma2(uint32_t a, uint32_t b, uint32_t c) {
    uint32_t d;
    asm("fma.rn.f16x2 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}
RDNA_DEV uint32_t hadd2(uint32_t a, uint32_t b) {
    uint32_t d;
    asm("add.rn.f16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
    return d;
}
// Byte 0 and byte 2 of a, then of b: the low bytes of the four halves.
RDNA_DEV uint32_t pack_half_low_bytes(uint32_t a, uint32_t b) {
    uint32_t r;
    asm("prmt.b32 %0, %1, %2, 0x6420;" : "=r"(r) : "r"(a), "r"(b));
    return r;
}

RDNA_DEV uint32_t pack_half2(float lo, float hi) {
    uint32_t r;
    // cvt.rn.f16x2.f32 d, a, b puts a in the upper half and b in the lower half.
    asm("cvt.rn.f16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
    return r;
}

}  // namespace sm100
}  // namespace rdna
