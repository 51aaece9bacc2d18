// Host side of librdnattention.so: argument validation, TMA tensor-map
// construction, kernel selection and launch.  Mirrors the reference's
// dispatch layer (src/rdna/fa2_forward_f16.hip:879-1077,
// src/rdna/fa2_forward_int8qk.hip:497-593): rdna::forwardF16 /
// rdna::forwardInt8QK take the same parameter structs, enqueue on the
// caller's stream without synchronising, and report failures through a
// thread-local message.  Every kernel of the library lives in this
// translation unit.
#include <cuda.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>

#include <cstdint>
#include <cstdio>
#include <cstring>
#include <mutex>

#include "rdna/forward.hpp"

#include "fa_decode.cuh"
#include "fa_prefill.cuh"
#include "peer.cuh"
#include "rope.cuh"
#include "quant.cuh"

namespace rdna {
namespace {

thread_local char g_err_f16[512] = {0};
thread_local char g_err_i8[512] = {0};

int fail(char* buf, const char* fmt, const char* arg) {
    std::snprintf(buf, 512, fmt, arg);
    return -1;
}

int fail(char* buf, const char* msg) { return fail(buf, "%s", msg); }

// ------------------------------------------------------------ tensor maps
PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q{};
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    });
    return fn;
}

struct View4 {
    const void* base;
    uint64_t dim[4];     // {head_dim, seq, heads, batch}
    int64_t stride[3];   // elements, for seq / heads / batch
};

// Builds a 4-D tiled map over a [batch, heads, seq, head_dim] view with
// element strides.  Axes of extent 1 get a synthetic (valid) stride, since
// their stride is never applied.
const char* make_map(CUtensorMap* m, const View4& v, CUtensorMapDataType dt, int esz, uint32_t box_inner,
                     uint32_t box_rows, CUtensorMapSwizzle sw) {
    auto enc = encode_fn();
    if (enc == nullptr) return "cuTensorMapEncodeTiled is unavailable (driver too old?)";
    cuuint64_t dims[4] = {v.dim[0], v.dim[1], v.dim[2], v.dim[3]};
    cuuint64_t strides[3];
    uint64_t fallback = v.dim[0] * static_cast<uint64_t>(esz);
    for (int i = 0; i < 3; ++i) {
        uint64_t s = static_cast<uint64_t>(v.stride[i]) * static_cast<uint64_t>(esz);
        if (v.dim[i + 1] <= 1) s = ((fallback + 15) / 16) * 16;
        strides[i] = s;
        fallback = s * v.dim[i + 1];
    }
    cuuint32_t box[4] = {box_inner, box_rows, 1, 1};
    cuuint32_t estr[4] = {1, 1, 1, 1};
    CUresult r = enc(m, dt, 4, const_cast<void*>(v.base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, sw,
                     CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return "cuTensorMapEncodeTiled rejected a tensor (pointer/stride alignment)";
    return nullptr;
}

// --------------------------------------------------------------- checks
struct Common {
    const void *q, *k, *v;
    void* o;
    int64_t qs[3], ks[3], vs[3], os[3];  // b, h, s
    uint32_t B, H, Hkv, S, KS, D;
    int esz;  // input element size
};

bool fits_i32(int64_t s) { return s >= INT32_MIN && s <= INT32_MAX; }

// K/V axes broadcast with element stride 0 (prefill::KV_BCAST_* bits).  Their
// tensor maps get extent 1 on that axis and the kernels load coordinate 0.
int kv_bcast_bits(const Common& c) {
    int m = 0;
    if (c.KS == 0) return 0;
    if (c.B > 1 && c.ks[0] == 0) m |= prefill::KV_BCAST_KB;
    if (c.Hkv > 1 && c.ks[1] == 0) m |= prefill::KV_BCAST_KH;
    if (c.B > 1 && c.vs[0] == 0) m |= prefill::KV_BCAST_VB;
    if (c.Hkv > 1 && c.vs[1] == 0) m |= prefill::KV_BCAST_VH;
    return m;
}

// A [batch, heads, seq, head_dim] K or V view for a tensor map: broadcast axes shrink to extent 1.
uint64_t bc_extent(uint64_t n, bool bcast) { return bcast ? 1u : n; }

// Debug settings of the calling thread for the expired-wait test
// (rdna_debug_set_wait_test): withheld K tile and shortened wait limit.
thread_local int g_dbg_withhold = -1;
thread_local unsigned long long g_dbg_wait_limit_ns = 0;

// Debug timing hook of the calling thread (rdna_debug_set_kernel_events): events
// recorded right before and right after the launch of each call's attention
// kernel (prefill or decode), not around the RoPE pre-pass.
thread_local cudaEvent_t g_dbg_ev[2] = {nullptr, nullptr};

template <class F>
cudaError_t launch_timed(cudaStream_t st, const F& launch) {
    if (g_dbg_ev[0] != nullptr) cudaEventRecord(g_dbg_ev[0], st);
    cudaError_t e = launch();
    if (g_dbg_ev[1] != nullptr) cudaEventRecord(g_dbg_ev[1], st);
    return e;
}

// Output replicas of the call in progress on this thread (the *Peers entry
// points set them for the duration of one call): other GPUs' counterparts of
// the output pointer, which every kernel writes with the same values as O.
struct OutputPeers {
    int n = 0;
    void* o[prefill::kMaxPeers] = {};
};
thread_local OutputPeers g_peers;

// Sets g_peers for one call and clears it when the call returns.
struct PeerScope {
    PeerScope(int n, void* const* o) {
        g_peers.n = n;
        for (int i = 0; i < n; ++i) g_peers.o[i] = o[i];
    }
    ~PeerScope() { g_peers = OutputPeers{}; }
};

const char* check_peers(int n, void* const* o) {
    if (n < 0 || n > prefill::kMaxPeers) return "peer output count must be between 0 and 7";
    if (n > 0 && o == nullptr) return "null peer output array";
    for (int i = 0; i < n; ++i)
        if (o[i] == nullptr || (reinterpret_cast<uintptr_t>(o[i]) & 15u) != 0)
            return "peer outputs must be non-null and 16-byte aligned";
    return nullptr;
}

const char* check_common(const Common& c) {
    // with key_seq_len == 0 K and V are never read (an empty tensor may have a null pointer)
    if (c.q == nullptr || c.o == nullptr || (c.KS > 0 && (c.k == nullptr || c.v == nullptr)))
        return "null tensor pointer";
    if (c.B == 0 || c.H == 0 || c.S == 0) return "empty problem (batch_size, num_heads and seq_len must be > 0)";
    if (c.Hkv == 0 || c.H % c.Hkv != 0) return "numHeads must be a positive multiple of numKvHeads";
    if (!fits_i32(c.qs[2]) || !fits_i32(c.ks[2]) || !fits_i32(c.vs[2]) || !fits_i32(c.os[2]))
        return "sequence-axis stride exceeds int32 range - not a realistic tensor size for this kernel";
    const int64_t align_in = 16 / c.esz;  // elements per 16 bytes
    auto aligned = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; };
    if (!aligned(c.q) || !aligned(c.o) || (c.KS > 0 && (!aligned(c.k) || !aligned(c.v))))
        return "tensor base pointers must be 16-byte aligned";
    const int64_t* in[3] = {c.qs, c.ks, c.vs};
    const uint64_t ext_q[3] = {c.B, c.H, c.S};
    const uint64_t ext_kv[3] = {c.B, c.Hkv, c.KS};
    for (int t = 0; t < 3; ++t) {
        if (t > 0 && c.KS == 0) continue;  // K/V are never read
        const uint64_t* ext = t == 0 ? ext_q : ext_kv;
        for (int a = 0; a < 3; ++a) {
            if (ext[a] <= 1) continue;
            // K/V may broadcast one tensor over the batch or head axis (stride 0, e.g. one
            // KV head shared by every query head); everything else needs positive strides
            if (in[t][a] == 0 && t > 0 && a < 2) continue;
            if (in[t][a] <= 0)
                return "strides must be positive (stride 0 only on the K/V batch and head axes; reversed axes are "
                       "not supported)";
            if (in[t][a] % align_in != 0) return "batch/head/seq strides must be multiples of 16 bytes";
        }
    }
    for (int a = 0; a < 3; ++a) {
        if (ext_q[a] <= 1) continue;
        if (c.os[a] <= 0) return "output strides must be positive";
        if (c.os[a] % 8 != 0) return "output batch/head/seq strides must be multiples of 16 bytes";
    }
    return nullptr;
}

// ---------------------------------------------------------------- launch
// pdl: the launch may overlap the preceding kernel on the stream (the RoPE
// pre-pass), whose output the kernel's producers wait for (griddepcontrol).
template <class T>
int launch_prefill(char* err, const Common& c, prefill::Params p, cudaStream_t stream, CUtensorMapDataType dt,
                   bool pdl = false) {
    using namespace prefill;
    if (p.rope_q && !T::ROPE_Q) return fail(err, "internal: Q rotation requested from a kernel without it");
    CUtensorMap tmQ, tmK, tmV, tmO;
    const CUtensorMapSwizzle sw = T::SW == 128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B;
    const CUtensorMapSwizzle osw = T::O_SW == 128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B;
    const View4 vq{c.q, {c.D, c.S, c.H, c.B}, {c.qs[2], c.qs[1], c.qs[0]}};
    // key_seq_len == 0: K/V are never read; give them a valid 1-row map
    const bool nokv = c.KS == 0;
    p.kv_bcast = kv_bcast_bits(c);
    const int bc = p.kv_bcast;
    const View4 vk{nokv ? c.q : c.k,
                   {c.D, nokv ? 1u : c.KS, nokv ? 1u : bc_extent(c.Hkv, bc & KV_BCAST_KH),
                    nokv ? 1u : bc_extent(c.B, bc & KV_BCAST_KB)},
                   {c.ks[2], c.ks[1], c.ks[0]}};
    const View4 vv{nokv ? c.q : c.v,
                   {c.D, nokv ? 1u : c.KS, nokv ? 1u : bc_extent(c.Hkv, bc & KV_BCAST_VH),
                    nokv ? 1u : bc_extent(c.B, bc & KV_BCAST_VB)},
                   {c.vs[2], c.vs[1], c.vs[0]}};
    p.dbg_withhold = g_dbg_withhold;
    p.dbg_wait_limit_ns = g_dbg_wait_limit_ns;
    p.n_peer = g_peers.n;
    const View4 vo{c.o, {c.D, c.S, c.H, c.B}, {c.os[2], c.os[1], c.os[0]}};
    // the peers' outputs: the same view at each peer's counterpart of c.o
    PeerMaps pm{};
    for (int i = 0; i < g_peers.n; ++i) {
        const View4 vp{g_peers.o[i], {c.D, c.S, c.H, c.B}, {c.os[2], c.os[1], c.os[0]}};
        if (const char* pe = make_map(&pm.m[i], vp, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, T::O_BOX, BM, osw))
            return fail(err, "%s", pe);
    }
    const char* e = nullptr;
    if ((e = make_map(&tmQ, vq, dt, T::ESZ, T::BOX, BM, sw)) ||
        (e = make_map(&tmK, vk, dt, T::ESZ, T::BOX, T::BC, sw)) ||
        (e = make_map(&tmV, vv, dt, T::ESZ, T::BOX, T::BC, sw)) ||
        (e = make_map(&tmO, vo, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, T::O_BOX, BM, osw)))
        return fail(err, "%s", e);

    p.B = c.B;
    p.H = c.H;
    p.Hkv = c.Hkv;
    p.S = c.S;
    p.KS = c.KS;
    p.G = c.H / c.Hkv;
    p.delta = static_cast<int>(c.KS) - static_cast<int>(c.S);
    p.n_rb = (c.S + BM - 1) / BM;
    p.n_rp = (p.n_rb + 1) / 2;
    p.pair_heads = (T::NT == 2 && p.G % 2 == 0) ? 1 : 0;
    if (T::D > T::DVMAX) {
        p.n_split = 2;
        const int half = (T::D / 2 + T::BOX - 1) / T::BOX * T::BOX;
        p.dv_split = half;
    } else {
        p.n_split = 1;
        p.dv_split = T::D;
    }
    int64_t items;
    if (T::NT == 1)
        items = static_cast<int64_t>(p.n_rb) * c.B * c.H;
    else if (p.pair_heads)
        items = static_cast<int64_t>(p.n_rb) * c.B * c.Hkv * (p.G / 2);
    else
        items = static_cast<int64_t>(p.n_rp) * c.B * c.H;
    items *= p.n_split;
    if (items > INT32_MAX) return fail(err, "problem too large for one launch");
    p.n_items = static_cast<int>(items);

    // one CTA per work item
    const int64_t grid = items;
    const int smem_bytes = T::SMEM_BYTES;

    auto kern = fa_prefill_kernel<T>;
    cudaError_t ce = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem_bytes);
    if (ce != cudaSuccess) return fail(err, "%s", cudaGetErrorString(ce));
    if constexpr (T::MIN_BLOCKS > 1) {
        ce = cudaFuncSetAttribute(kern, cudaFuncAttributePreferredSharedMemoryCarveout, 100);
        if (ce != cudaSuccess) return fail(err, "%s", cudaGetErrorString(ce));
    }
    if constexpr (T::RESPLIT) {
        // setmaxnreg.inc waits for registers the CTA was launched with: refuse to
        // launch unless the binary really allocates LAUNCH_REGS per thread.
        cudaFuncAttributes fa{};
        ce = cudaFuncGetAttributes(&fa, kern);
        if (ce != cudaSuccess) return fail(err, "%s", cudaGetErrorString(ce));
        if (fa.numRegs != T::LAUNCH_REGS)
            return fail(err, "internal: kernel register count does not match its register split");
    }

    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(static_cast<unsigned>(grid), 1, 1);
    cfg.blockDim = dim3(T::THREADS, 1, 1);
    cfg.dynamicSmemBytes = static_cast<size_t>(smem_bytes);
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    ce = launch_timed(stream, [&] { return cudaLaunchKernelEx(&cfg, kern, tmQ, tmK, tmV, tmO, pm, p); });
    if (ce == cudaSuccess) ce = cudaGetLastError();
    if (ce != cudaSuccess) return fail(err, "%s", cudaGetErrorString(ce));
    return 0;
}


template <int D>
int dispatch_f16_dim(char* err, const Common& c, const prefill::Params& p, cudaStream_t st, bool pdl) {
    using namespace prefill;
    constexpr CUtensorMapDataType dt = CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
    if constexpr (D <= 96) {
        // one 128-row tile per CTA, S double-buffered (256 TMEM columns), two
        // CTAs per SM: one CTA's prologue and epilogue overlap the other's main
        // loop.  Measured 6-9 % faster than the two-tile CTA for D <= 64 and
        // 5 % at D = 96 (three K/V stages); at D = 128 only two stages fit
        // beside a second CTA and it is 25 % slower.
        constexpr int st1 = D <= 64 ? 4 : 3;
        return launch_prefill<Traits<D, D, 64, 1, st1, st1, false, true>>(err, c, p, st, dt, pdl);
    } else if constexpr (D <= 128) {
        // two 128-row tiles per CTA, 64-key blocks, S double-buffered in TMEM
        // (2 tiles x 2 buffers x 64 columns + 2 x D columns of O <= 512)
        constexpr int stages = D <= 64 ? 6 : D <= 96 ? 5 : 4;
        return launch_prefill<Traits<D, D, 64, 2, stages, stages, false, true>>(err, c, p, st, dt, pdl);
    } else if constexpr (D <= 256) {
        // one tile per CTA (TMEM holds one O of up to 256 columns), 64-key blocks
        constexpr int stages = D <= 192 ? 3 : 2;
        return launch_prefill<Traits<D, D, 64, 1, stages, stages, false>>(err, c, p, st, dt, pdl);
    } else {
        // head_dim > 256: two CTAs per tile, each owning half of the output columns
        constexpr int qk = 128 * D * 2, kt = 64 * D * 2, vt = 64 * 256 * 2;
        constexpr int stages = (2048 + qk + 2 * (kt + vt) <= 232448) ? 2 : 1;
        return launch_prefill<Traits<D, 256, 64, 1, stages, stages, false>>(err, c, p, st, dt, pdl);
    }
}

}  // namespace

namespace {

constexpr size_t kWsAlign = 256;

size_t align_up(size_t x) { return (x + kWsAlign - 1) / kWsAlign * kWsAlign; }

// Whether the prefill kernel of this call rotates Q itself (the head_dim <= 128
// kernels, prefill::Traits::ROPE_Q); otherwise the pre-pass rotates Q too.
bool q_rope_in_kernel(const ForwardParams& a) {
    return a.hasRope && a.headDim <= 128 && prefill::Traits<128, 128, 64, 2, 4, 4, false, true>::ROPE_Q;
}

// Workspace of an FP16 call: rotated K (and Q, see q_rope_in_kernel), contiguous
// fp16, when RoPE is on and the call takes the prefill path (the decode kernel
// rotates in place).
size_t f16_workspace_bytes(const ForwardParams& a) {
    if (!a.hasRope) return 0;
    if (a.numKvHeads != 0 && decode::eligible(a.seqLen, a.numHeads / a.numKvHeads, a.headDim)) return 0;
    const size_t q = static_cast<size_t>(a.batchSize) * a.numHeads * a.seqLen * a.headDim * 2;
    const size_t k = static_cast<size_t>(a.batchSize) * a.numKvHeads * a.keySeqLen * a.headDim * 2;
    return (q_rope_in_kernel(a) ? 0 : align_up(q)) + align_up(k);
}

int f16_validate(const Common& c, const ForwardParams& a) {
    if (const char* e = check_common(c)) return fail(g_err_f16, "%s", e);
    if (a.headDim < 32 || a.headDim > 512 || a.headDim % 32 != 0)
        return fail(g_err_f16, "unsupported head_dim (multiples of 32 from 32 to 512)");
    if (a.hasRope) {
        if (a.rot_cos == nullptr || a.rot_sin == nullptr)
            return fail(g_err_f16, "has_rope set but rot_cos/rot_sin is null");
        if ((reinterpret_cast<uintptr_t>(a.rot_cos) & 15u) || (reinterpret_cast<uintptr_t>(a.rot_sin) & 15u))
            return fail(g_err_f16, "rot_cos/rot_sin must be 16-byte aligned");
    }
    if (a.seqLen > (1u << 30) || a.keySeqLen > (1u << 30)) return fail(g_err_f16, "sequence too long");
    return 0;
}

Common f16_common(const ForwardParams& a) {
    return Common{a.q, a.k, a.v, a.o,
                  {a.qStrideB, a.qStrideH, a.qStrideS}, {a.kStrideB, a.kStrideH, a.kStrideS},
                  {a.vStrideB, a.vStrideH, a.vStrideS}, {a.oStrideB, a.oStrideH, a.oStrideS},
                  a.batchSize, a.numHeads, a.numKvHeads, a.seqLen, a.keySeqLen, a.headDim, 2};
}

// Enqueues the rotation of K (and of Q unless the kernel rotates it) into `ws`;
// rewrites `c` to read the rotated copies.
int launch_rope(const ForwardParams& a, Common& c, void* ws, cudaStream_t st) {
    rope::Params rp{};
    const bool with_q = !q_rope_in_kernel(a);
    __half* qr = static_cast<__half*>(ws);
    const size_t qbytes = with_q ? static_cast<size_t>(a.batchSize) * a.numHeads * a.seqLen * a.headDim * 2 : 0;
    __half* kr = reinterpret_cast<__half*>(static_cast<char*>(ws) + align_up(qbytes));
    rp.t[0] = rope::Tensor4{static_cast<const __half*>(a.q), qr, a.qStrideB, a.qStrideH, a.qStrideS,
                            static_cast<int>(a.batchSize), static_cast<int>(a.numHeads), static_cast<int>(a.seqLen)};
    rp.t[1] = rope::Tensor4{static_cast<const __half*>(a.k), kr, a.kStrideB, a.kStrideH, a.kStrideS,
                            static_cast<int>(a.batchSize), static_cast<int>(a.numKvHeads),
                            static_cast<int>(a.keySeqLen)};
    const int64_t qrows = with_q ? static_cast<int64_t>(a.batchSize) * a.numHeads * a.seqLen : 0;
    const int64_t krows = static_cast<int64_t>(a.batchSize) * a.numKvHeads * a.keySeqLen;
    if (qrows + krows > INT32_MAX) return fail(g_err_f16, "RoPE pre-pass: too many rows for one launch");
    rp.rows[0] = static_cast<int>(qrows);
    rp.rows[1] = static_cast<int>(krows);
    rp.cos_t = static_cast<const float*>(a.rot_cos);
    rp.sin_t = static_cast<const float*>(a.rot_sin);
    rp.D = static_cast<int>(a.headDim);
    rp.cpr = rp.D / 8;
    rp.rpb = 256 / rp.cpr;
    const int64_t total = qrows + krows;
    int dev = 0, sms = 148;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    const int64_t want = (total + rp.rpb - 1) / rp.rpb;
    const int grid = static_cast<int>(want < static_cast<int64_t>(sms) * 8 ? want : static_cast<int64_t>(sms) * 8);
    if (grid > 0) rope::rope_rotate_kernel<<<grid, rp.rpb * rp.cpr, 0, st>>>(rp);
    cudaError_t ce = cudaGetLastError();
    if (ce != cudaSuccess) return fail(g_err_f16, "%s", cudaGetErrorString(ce));
    const int64_t D = a.headDim;
    if (with_q) {
        c.q = qr;
        c.qs[0] = static_cast<int64_t>(a.numHeads) * a.seqLen * D;
        c.qs[1] = static_cast<int64_t>(a.seqLen) * D;
        c.qs[2] = D;
    }
    c.k = kr;
    c.ks[0] = static_cast<int64_t>(a.numKvHeads) * a.keySeqLen * D;
    c.ks[1] = static_cast<int64_t>(a.keySeqLen) * D;
    c.ks[2] = D;
    return 0;
}

int f16_attention(const ForwardParams& a, const Common& c, cudaStream_t st, bool pdl) {
    prefill::Params p{};
    p.causal = a.causal ? 1 : 0;
    p.window = a.windowSize > 0 ? a.windowSize : 0;
    p.scale_log2 = a.scale * 1.4426950408889634f;
    p.rope_q = q_rope_in_kernel(a) ? 1 : 0;
    p.rope_cos = static_cast<const float*>(a.rot_cos);
    p.rope_sin = static_cast<const float*>(a.rot_sin);
    switch (a.headDim) {
#define RDNA_D(Dv) \
    case Dv: return dispatch_f16_dim<Dv>(g_err_f16, c, p, st, pdl);
        RDNA_D(32) RDNA_D(64) RDNA_D(96) RDNA_D(128) RDNA_D(160) RDNA_D(192) RDNA_D(224) RDNA_D(256)
        RDNA_D(288) RDNA_D(320) RDNA_D(352) RDNA_D(384) RDNA_D(416) RDNA_D(448) RDNA_D(480) RDNA_D(512)
#undef RDNA_D
        default:
            break;
    }
    return fail(g_err_f16, "unsupported head_dim (multiples of 32 from 32 to 512)");
}

}  // namespace

namespace decode {

// Cluster-split decode launch: one cluster of CS CTAs per (batch, kv head).
int launch_f16(char* err, const ForwardParams& a, cudaStream_t stream) {
    const int D = static_cast<int>(a.headDim);
    Params p{};
    p.q = static_cast<const __half*>(a.q);
    p.o = static_cast<__half*>(a.o);
    p.qsb = a.qStrideB;
    p.qsh = a.qStrideH;
    p.qss = a.qStrideS;
    p.osb = a.oStrideB;
    p.osh = a.oStrideH;
    p.oss = a.oStrideS;
    p.B = static_cast<int>(a.batchSize);
    p.H = static_cast<int>(a.numHeads);
    p.Hkv = static_cast<int>(a.numKvHeads);
    p.S = static_cast<int>(a.seqLen);
    p.KS = static_cast<int>(a.keySeqLen);
    p.G = p.H / p.Hkv;
    p.R = p.G * p.S;
    p.delta = p.KS - p.S;
    p.causal = a.causal ? 1 : 0;
    p.window = a.windowSize > 0 ? a.windowSize : 0;
    p.scale_log2 = a.scale * 1.4426950408889634f;
    p.rope = a.hasRope ? 1 : 0;
    p.rope_cos = static_cast<const float*>(a.rot_cos);
    p.rope_sin = static_cast<const float*>(a.rot_sin);
    p.n_peer = g_peers.n;
    for (int i = 0; i < g_peers.n; ++i) p.o_peer[i] = static_cast<__half*>(g_peers.o[i]);

    CUtensorMap tmK, tmV;
    const bool nokv = a.keySeqLen == 0;
    p.kv_bcast = kv_bcast_bits(f16_common(a));
    const int bc = p.kv_bcast;
    const uint64_t e1 = nokv ? 1 : a.keySeqLen, e2 = nokv ? 1 : a.numKvHeads, e3 = nokv ? 1 : a.batchSize;
    const View4 vk{nokv ? a.q : a.k,
                   {a.headDim, e1, bc_extent(e2, bc & prefill::KV_BCAST_KH), bc_extent(e3, bc & prefill::KV_BCAST_KB)},
                   {a.kStrideS, a.kStrideH, a.kStrideB}};
    const View4 vv{nokv ? a.q : a.v,
                   {a.headDim, e1, bc_extent(e2, bc & prefill::KV_BCAST_VH), bc_extent(e3, bc & prefill::KV_BCAST_VB)},
                   {a.vStrideS, a.vStrideH, a.vStrideB}};
    const char* e = nullptr;
    if ((e = make_map(&tmK, vk, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, 64, KT, CU_TENSOR_MAP_SWIZZLE_128B)) ||
        (e = make_map(&tmV, vv, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, 64, KT, CU_TENSOR_MAP_SWIZZLE_128B)))
        return fail(err, "%s", e);

    // row groups of 16 rows inside the CTA; their count divides the consumer warps
    p.NRG = p.R <= MAX_ROWS ? 1 : p.R <= 2 * MAX_ROWS ? 2 : 4;
    const int64_t units = static_cast<int64_t>(p.B) * p.Hkv;
    if (units > 65535) return fail(err, "too many (batch, kv head) units for one decode launch");
    const int64_t tiles = (static_cast<int64_t>(p.KS) + KT - 1) / KT;
    // Cluster size: the split with the least modelled time, waves over the SMs (one CTA
    // each) x (tiles per CTA + a fixed cost per CTA that grows with the cluster: ring fill,
    // DSMEM combine, and the SMs a wide cluster leaves idle while it waits for enough
    // free SMs in one GPC).  The fixed costs are in tile times, fitted on B200 (32-key
    // tiles, head_dim 128, KS 8192-32768, batch 8-64): clusters of 1 / 2 / 4 / 8 cost
    // about 2 / 15 / 24 / 78 tiles.  Each CTA keeps >= 8 tiles.
    int dev = 0, sms = 148;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    auto cost = [&](int c) {
        const int64_t waves = (units * c + sms - 1) / sms;
        const int64_t fixed = c == 1 ? 2 : c == 2 ? 15 : c == 4 ? 24 : 78;
        return waves * ((tiles + c - 1) / c + fixed);
    };
    int cs = 1;
    for (int c = 2; c <= MAX_CLUSTER && tiles / c >= 8; c *= 2)
        if (cost(c) < cost(cs)) cs = c;

    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(cs, static_cast<unsigned>(units), 1);
    cfg.blockDim = dim3(p.rope ? THREADS_ROPE : THREADS, 1, 1);
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = cs;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    auto launch = [&](auto kern, int smem) {
        cfg.dynamicSmemBytes = smem;
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
        return e == cudaSuccess ? cudaLaunchKernelEx(&cfg, kern, tmK, tmV, p) : e;
    };
    cudaError_t ce = launch_timed(stream, [&] {
        if (D == 64)
            return p.rope ? launch(fa_decode_kernel<64, true>, Layout<64>::SMEM_BYTES)
                          : launch(fa_decode_kernel<64, false>, Layout<64>::SMEM_BYTES);
        return p.rope ? launch(fa_decode_kernel<128, true>, Layout<128>::SMEM_BYTES)
                      : launch(fa_decode_kernel<128, false>, Layout<128>::SMEM_BYTES);
    });
    if (ce == cudaSuccess) ce = cudaGetLastError();
    if (ce != cudaSuccess) return fail(err, "%s", cudaGetErrorString(ce));
    return 0;
}

}  // namespace decode

namespace {
}  // namespace

size_t workspaceBytesF16(const ForwardParams& a) { return f16_workspace_bytes(a); }

int forwardF16Ws(const ForwardParams& a, void* workspace, size_t workspace_bytes, void* stream) {
    Common c = f16_common(a);
    if (int rc = f16_validate(c, a)) return rc;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    // small seq_len x group: the split-KV decode kernel (RoPE applied in place)
    if (decode::eligible(a.seqLen, a.numHeads / a.numKvHeads, a.headDim)) return decode::launch_f16(g_err_f16, a, st);
    const size_t need = f16_workspace_bytes(a);
    if (need > 0) {
        if (workspace == nullptr || workspace_bytes < need)
            return fail(g_err_f16, "workspace missing or smaller than rdna_attention_forward_workspace_size()");
        if (reinterpret_cast<uintptr_t>(workspace) & (kWsAlign - 1))
            return fail(g_err_f16, "workspace must be 256-byte aligned");
        if (int rc = launch_rope(a, c, workspace, st)) return rc;
    }
    // after a RoPE pre-pass the attention kernel is launched to overlap its tail
    return f16_attention(a, c, st, need > 0);
}

int forwardF16(const ForwardParams& a, void* stream) {
    const size_t need = f16_workspace_bytes(a);
    if (need == 0) return forwardF16Ws(a, nullptr, 0, stream);
    {
        Common c = f16_common(a);
        if (int rc = f16_validate(c, a)) return rc;
    }
    // Stream-ordered workspace for the rotated Q/K: allocated and released on
    // the caller's stream, so the call still never blocks the host.
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    void* ws = nullptr;
    cudaError_t ce = cudaMallocAsync(&ws, need, st);
    if (ce != cudaSuccess) return fail(g_err_f16, "workspace allocation failed: %s", cudaGetErrorString(ce));
    const int rc = forwardF16Ws(a, ws, need, stream);
    ce = cudaFreeAsync(ws, st);
    if (rc != 0) return rc;
    if (ce != cudaSuccess) return fail(g_err_f16, "%s", cudaGetErrorString(ce));
    return 0;
}

// ------------------------------------------------- fixed-workspace variant
//
// For callers that cannot allocate device memory (see
// rdna_attention_forward_noalloc in rdnattention.h): the RoPE workspace is this
// file-scope array, reserved on every device that loads the library's module
// until the process exits.  In host code the name below is only a host-side
// stand-in; its device address comes from cudaGetSymbolAddress, taken once
// per device with that device current, on the first call there (so calls
// after cudaDeviceReset on that device, which reloads the module, are not
// supported: the cached address may no longer be the array's).  Every call
// shares the array: the RoPE pre-pass overwrites every byte the attention
// kernel reads before it is read, so nothing needs clearing, but calls that
// overlap on the GPU (other streams, other threads) race on it.
constexpr size_t kNoAllocWorkspaceBytes = size_t(32) << 20;  // 32 MiB
static __device__ __align__(256) unsigned char g_noalloc_workspace[kNoAllocWorkspaceBytes];

namespace {
std::mutex g_noalloc_mu;
constexpr int kMaxDevices = 256;
void* g_noalloc_ptr[kMaxDevices] = {};
}  // namespace

size_t noAllocWorkspaceLimit() { return kNoAllocWorkspaceBytes; }

int forwardF16NoAlloc(const ForwardParams& a, void* stream) {
    {
        // argument errors first, so a malformed call gets its own message
        Common c = f16_common(a);
        if (int rc = f16_validate(c, a)) return rc;
    }
    const size_t need = f16_workspace_bytes(a);
    if (need > kNoAllocWorkspaceBytes) {
        char msg[160];
        std::snprintf(msg, sizeof(msg), "RoPE workspace of %zu bytes exceeds the fixed %zu-byte no-alloc workspace",
                      need, kNoAllocWorkspaceBytes);
        return fail(g_err_f16, "%s", msg);
    }
    if (need == 0) return forwardF16Ws(a, nullptr, 0, stream);
    int dev = -1;
    cudaError_t ce = cudaGetDevice(&dev);
    if (ce != cudaSuccess) return fail(g_err_f16, "%s", cudaGetErrorString(ce));
    if (dev < 0 || dev >= kMaxDevices) return fail(g_err_f16, "device ordinal out of range");
    void* ws = nullptr;
    {
        std::lock_guard<std::mutex> lock(g_noalloc_mu);
        if (g_noalloc_ptr[dev] == nullptr) {
            void* p = nullptr;
            ce = cudaGetSymbolAddress(&p, g_noalloc_workspace);
            if (ce != cudaSuccess) return fail(g_err_f16, "cudaGetSymbolAddress: %s", cudaGetErrorString(ce));
            g_noalloc_ptr[dev] = p;
        }
        ws = g_noalloc_ptr[dev];
    }
    return forwardF16Ws(a, ws, kNoAllocWorkspaceBytes, stream);
}

namespace {
int int8_forward(const ForwardParamsInt8QK& a, int32_t* s_dump, void* stream) {
    Common c{a.q, a.k, a.v, a.o,
             {a.qStrideB, a.qStrideH, a.qStrideS}, {a.kStrideB, a.kStrideH, a.kStrideS},
             {a.vStrideB, a.vStrideH, a.vStrideS}, {a.oStrideB, a.oStrideH, a.oStrideS},
             a.batchSize, a.numHeads, a.numKvHeads, a.seqLen, a.keySeqLen, a.headDim, 1};
    if (a.numKvHeads == 0 || a.numHeads % a.numKvHeads != 0)
        return fail(g_err_i8, "numHeads must be a positive multiple of numKvHeads");
    if (const char* e = check_common(c)) return fail(g_err_i8, "%s", e);
    if (a.headDim != 64 && a.headDim != 128)
        return fail(g_err_i8, "unsupported head_dim (only 64 and 128 are compiled in for the int8 kernel)");
    if (a.seqLen > (1u << 30) || a.keySeqLen > (1u << 30)) return fail(g_err_i8, "sequence too long");

    prefill::Params p{};
    p.causal = a.causal ? 1 : 0;
    p.window = a.windowSize > 0 ? a.windowSize : 0;
    p.scale_log2 = a.scale * 1.4426950408889634f;
    p.q_scale = a.qScale;
    p.k_scale = a.kScale;
    p.pv_scale = a.vScale / 127.0f;
    p.q_vec = static_cast<const float*>(a.qScaleVec);
    p.k_vec = static_cast<const float*>(a.kScaleVec);
    p.v_chan = static_cast<const float*>(a.vChannel);
    p.s_dump = s_dump;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    constexpr CUtensorMapDataType dt = CU_TENSOR_MAP_DATA_TYPE_UINT8;
    // head_dim 64: one pass over 128-key blocks, two query tiles per CTA (S 2 x 128 + ACC
    // 2 x 64 + O 2 x 64 = 512 TMEM columns), the s32 accumulator folded into the fp32 O
    // when a row max moves.  head_dim 128, up to kTwoPassMaxKeys keys: two passes (row
    // maxima, then P against the final max), so the accumulator is never rescaled and
    // needs no O in TMEM, which leaves room for two tiles (S 2 x 128 + ACC 2 x 128); longer
    // key ranges take the one-pass kernel with one tile (S + ACC + O = 384 columns).
    constexpr uint32_t kTwoPassMaxKeys = 131072;  // 127 * 128 * keys < 2^31: no s32 overflow
    const bool two = a.keySeqLen <= kTwoPassMaxKeys;
    using namespace prefill;
    if (s_dump != nullptr) {
        // debug instantiations: the same kernels plus the score dump
        if (a.headDim == 64)
            return launch_prefill<Traits<64, 64, 128, 2, 4, 4, true, false, true>>(g_err_i8, c, p, st, dt);
        return two ? launch_prefill<Traits<128, 128, 128, 2, 3, 3, true, false, true, true>>(g_err_i8, c, p, st, dt)
                   : launch_prefill<Traits<128, 128, 128, 1, 3, 3, true, false, true>>(g_err_i8, c, p, st, dt);
    }
    if (a.headDim == 64) return launch_prefill<Traits<64, 64, 128, 2, 4, 4, true>>(g_err_i8, c, p, st, dt);
    return two ? launch_prefill<Traits<128, 128, 128, 2, 3, 3, true, false, false, true>>(g_err_i8, c, p, st, dt)
               : launch_prefill<Traits<128, 128, 128, 1, 3, 3, true>>(g_err_i8, c, p, st, dt);
}
}  // namespace

int forwardInt8QK(const ForwardParamsInt8QK& a, void* stream) { return int8_forward(a, nullptr, stream); }

int forwardF16WsPeers(const ForwardParams& a, void* workspace, size_t workspace_bytes, int n_peers,
                      void* const* peers, void* stream) {
    if (const char* e = check_peers(n_peers, peers)) return fail(g_err_f16, "%s", e);
    PeerScope scope(n_peers, peers);
    return forwardF16Ws(a, workspace, workspace_bytes, stream);
}

int forwardInt8QKPeers(const ForwardParamsInt8QK& a, int n_peers, void* const* peers, void* stream) {
    if (const char* e = check_peers(n_peers, peers)) return fail(g_err_i8, "%s", e);
    PeerScope scope(n_peers, peers);
    return int8_forward(a, nullptr, stream);
}

// ------------------------------------------------ device memory shared across processes
int ipcAlloc(size_t bytes, void** ptr, void* handle) {
    if (ptr == nullptr || handle == nullptr) return fail(g_err_f16, "null argument");
    if (bytes == 0) return fail(g_err_f16, "empty allocation");
    *ptr = nullptr;
    cudaError_t ce = cudaMalloc(ptr, bytes);
    if (ce != cudaSuccess) return fail(g_err_f16, "%s", cudaGetErrorString(ce));
    cudaIpcMemHandle_t h{};
    ce = cudaIpcGetMemHandle(&h, *ptr);
    if (ce != cudaSuccess) {
        cudaFree(*ptr);
        *ptr = nullptr;
        return fail(g_err_f16, "%s", cudaGetErrorString(ce));
    }
    std::memcpy(handle, &h, sizeof(h));
    return 0;
}

int ipcOpen(const void* handle, void** ptr) {
    if (ptr == nullptr || handle == nullptr) return fail(g_err_f16, "null argument");
    cudaIpcMemHandle_t h{};
    std::memcpy(&h, handle, sizeof(h));
    cudaError_t ce = cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess);
    if (ce != cudaSuccess) return fail(g_err_f16, "%s", cudaGetErrorString(ce));
    return 0;
}

int ipcClose(void* ptr) {
    cudaError_t ce = cudaIpcCloseMemHandle(ptr);
    if (ce != cudaSuccess) return fail(g_err_f16, "%s", cudaGetErrorString(ce));
    return 0;
}

int peerBarrier(int world, int rank, void* const* peer_flags, void* my_flags, unsigned int epoch, void* stream) {
    if (world < 2 || world > peer::kMaxPeers + 1 || rank < 0 || rank >= world)
        return fail(g_err_f16, "barrier: world must be 2 to 8 ranks and 0 <= rank < world");
    auto bad = [](const void* q) { return q == nullptr || (reinterpret_cast<uintptr_t>(q) & 3u) != 0; };
    if (peer_flags == nullptr || bad(my_flags)) return fail(g_err_f16, "barrier: null or misaligned flag array");
    peer::BarrierParams p{};
    for (int i = 0; i < world - 1; ++i) {
        if (bad(peer_flags[i])) return fail(g_err_f16, "barrier: null or misaligned flag array");
        p.peer_flags[i] = static_cast<unsigned int*>(peer_flags[i]);
    }
    p.world = world;
    p.rank = rank;
    p.my_flags = static_cast<unsigned int*>(my_flags);
    p.epoch = epoch;
    // (the expired-wait test hook shortens the barrier's waits too)
    p.limit_ns = g_dbg_wait_limit_ns > 0 ? g_dbg_wait_limit_ns : peer::kBarrierLimitNs;
    peer::barrier_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(p);
    cudaError_t ce = cudaGetLastError();
    if (ce != cudaSuccess) return fail(g_err_f16, "%s", cudaGetErrorString(ce));
    return 0;
}

int ipcFree(void* ptr) {
    cudaError_t ce = cudaFree(ptr);
    if (ce != cudaSuccess) return fail(g_err_f16, "%s", cudaGetErrorString(ce));
    return 0;
}

int debugInt8QKScores(const ForwardParamsInt8QK& a, void* scores, void* stream) {
    if (scores == nullptr || (reinterpret_cast<uintptr_t>(scores) & 3u) != 0)
        return fail(g_err_i8, "scores must be a 4-byte aligned int32 buffer");
    return int8_forward(a, static_cast<int32_t*>(scores), stream);
}

int quantizeInt8QKV(const QuantizeInt8Params& a, void* stream) {
    if (a.q == nullptr || a.k == nullptr || a.v == nullptr || a.qInt8 == nullptr || a.kInt8 == nullptr ||
        a.vInt8 == nullptr || a.qScale == nullptr || a.kScale == nullptr || a.vChannel == nullptr)
        return fail(g_err_i8, "null tensor pointer");
    if (a.batchSize == 0 || a.numHeads == 0 || a.seqLen == 0 || a.keySeqLen == 0) return fail(g_err_i8, "empty problem");
    if (a.numKvHeads == 0 || a.numHeads % a.numKvHeads != 0)
        return fail(g_err_i8, "numHeads must be a positive multiple of numKvHeads");
    if (a.headDim != 64 && a.headDim != 128)
        return fail(g_err_i8, "unsupported head_dim (only 64 and 128 are compiled in for the int8 kernel)");
    auto aligned = [](const void* p, uintptr_t n) { return (reinterpret_cast<uintptr_t>(p) & (n - 1)) == 0; };
    if (!aligned(a.q, 16) || !aligned(a.k, 16) || !aligned(a.v, 16) || !aligned(a.qInt8, 8) || !aligned(a.kInt8, 8) ||
        !aligned(a.vInt8, 8) || !aligned(a.qScale, 4) || !aligned(a.kScale, 4) || !aligned(a.vChannel, 4))
        return fail(g_err_i8, "tensor base pointers must be 16-byte aligned (int8 outputs 8, scales 4)");
    const int64_t st[9] = {a.qStrideB, a.qStrideH, a.qStrideS, a.kStrideB, a.kStrideH, a.kStrideS,
                           a.vStrideB, a.vStrideH, a.vStrideS};
    for (int64_t x : st)
        if (x <= 0 || x % 8 != 0) return fail(g_err_i8, "strides must be positive multiples of 16 bytes");
    const int64_t qrows = static_cast<int64_t>(a.batchSize) * a.numHeads * a.seqLen;
    const int64_t krows = static_cast<int64_t>(a.batchSize) * a.numKvHeads * a.keySeqLen;
    const int64_t units = static_cast<int64_t>(a.batchSize) * a.numKvHeads;
    quant::Params p{};
    p.t[0] = quant::Rows{static_cast<const __half*>(a.q), static_cast<int8_t*>(a.qInt8), static_cast<float*>(a.qScale),
                         a.qStrideB, a.qStrideH, a.qStrideS, static_cast<int>(a.numHeads), static_cast<int>(a.seqLen),
                         qrows};
    p.t[1] = quant::Rows{static_cast<const __half*>(a.k), static_cast<int8_t*>(a.kInt8), static_cast<float*>(a.kScale),
                         a.kStrideB, a.kStrideH, a.kStrideS, static_cast<int>(a.numKvHeads),
                         static_cast<int>(a.keySeqLen), krows};
    p.v = static_cast<const __half*>(a.v);
    p.vi = static_cast<int8_t*>(a.vInt8);
    p.vch = static_cast<float*>(a.vChannel);
    p.vsb = a.vStrideB;
    p.vsh = a.vStrideH;
    p.vss = a.vStrideS;
    p.Hkv = static_cast<int>(a.numKvHeads);
    p.KS = static_cast<int>(a.keySeqLen);
    p.D = static_cast<int>(a.headDim);
    // per-token part: enough warps to cover every row a few times over the SMs
    const int rows_per_block = (quant::kThreads / 32) * (32 / (p.D / 8));
    auto blocks_for = [&](int64_t rows) {
        const int64_t want = (rows + rows_per_block - 1) / rows_per_block;
        return static_cast<int>(want < 148 * 8 ? want : 148 * 8);
    };
    p.blocks_q = blocks_for(qrows);
    p.blocks_k = blocks_for(krows);
    const int64_t grid = static_cast<int64_t>(p.blocks_q) + p.blocks_k + units;
    if (grid > INT32_MAX) return fail(g_err_i8, "problem too large for one launch");
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    quant::quantize_qkv_kernel<<<static_cast<unsigned>(grid), quant::kThreads, 0, s>>>(p);
    const cudaError_t ce = cudaGetLastError();
    if (ce != cudaSuccess) return fail(g_err_i8, "%s", cudaGetErrorString(ce));
    return 0;
}

void debugSetKernelEvents(void* start, void* stop) {
    g_dbg_ev[0] = static_cast<cudaEvent_t>(start);
    g_dbg_ev[1] = static_cast<cudaEvent_t>(stop);
}

void debugSetWaitTest(int32_t withhold_block, uint64_t wait_limit_ns) {
    g_dbg_withhold = withhold_block;
    g_dbg_wait_limit_ns = withhold_block >= 0 ? wait_limit_ns : 0;
}

const char* lastError() { return g_err_f16[0] ? g_err_f16 : nullptr; }
const char* lastErrorInt8QK() { return g_err_i8[0] ? g_err_i8 : nullptr; }

bool hasDevice() {
    int n = 0;
    return cudaGetDeviceCount(&n) == cudaSuccess && n > 0;
}

int debugReadStatus(int32_t* out2, const char** why) {
    int host[2] = {0, 0};
    cudaError_t e = cudaDeviceSynchronize();
    if (e == cudaSuccess) e = cudaMemcpyFromSymbol(host, g_rdna_status, sizeof(host));
    if (e == cudaSuccess) {
        const int zero[2] = {0, 0};
        e = cudaMemcpyToSymbol(g_rdna_status, zero, sizeof(zero));
    }
    if (e != cudaSuccess) {
        *why = cudaGetErrorString(e);
        return -1;
    }
    out2[0] = host[0];
    out2[1] = host[1];
    return 0;
}

}  // namespace rdna
