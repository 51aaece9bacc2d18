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

const char* check_common(const Common& c) {
    if (c.q == nullptr || c.k == nullptr || c.v == nullptr || c.o == nullptr) return "null tensor pointer";
    if (c.B == 0 || c.H == 0 || c.S == 0) return "empty problem (batch_size, num_heads and seq_len must be > 0)";
    if (c.Hkv == 0 || c.H % c.Hkv != 0) return "numHeads must be a positive multiple of numKvHeads";
    if (!fits_i32(c.qs[2]) || !fits_i32(c.ks[2]) || !fits_i32(c.vs[2]) || !fits_i32(c.os[2]))
        return "sequence-axis stride exceeds int32 range - not a realistic tensor size for this kernel";
    const int64_t align_in = 16 / c.esz;  // elements per 16 bytes
    auto aligned = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; };
    if (!aligned(c.q) || !aligned(c.k) || !aligned(c.v) || !aligned(c.o))
        return "tensor base pointers must be 16-byte aligned";
    const int64_t* in[3] = {c.qs, c.ks, c.vs};
    const uint64_t ext_q[3] = {c.B, c.H, c.S};
    const uint64_t ext_kv[3] = {c.B, c.Hkv, c.KS};
    for (int t = 0; t < 3; ++t) {
        const uint64_t* ext = t == 0 ? ext_q : ext_kv;
        for (int a = 0; a < 3; ++a) {
            if (ext[a] <= 1) continue;
            if (in[t][a] <= 0) return "strides must be positive (broadcast or reversed axes are not supported)";
            if (in[t][a] % align_in != 0) return "batch/head/seq strides must be multiples of 16 bytes";
        }
    }
    for (int a = 0; a < 3; ++a) {
        if (ext_q[a] <= 1) continue;
        if (c.os[a] <= 0) return "strides must be positive (broadcast or reversed axes are not supported)";
        if (c.os[a] % 8 != 0) return "output batch/head/seq strides must be multiples of 16 bytes";
    }
    return nullptr;
}

// ---------------------------------------------------------------- launch
template <class T>
int launch_prefill(char* err, const Common& c, prefill::Params p, cudaStream_t stream, CUtensorMapDataType dt) {
    using namespace prefill;
    CUtensorMap tmQ, tmK, tmV, tmO;
    const CUtensorMapSwizzle sw = T::SW == 128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B;
    const CUtensorMapSwizzle osw = T::O_SW == 128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B;
    const uint64_t ks_ext = c.KS > 0 ? c.KS : 1;
    const View4 vq{c.q, {c.D, c.S, c.H, c.B}, {c.qs[2], c.qs[1], c.qs[0]}};
    const View4 vk{c.k, {c.D, ks_ext, c.Hkv, c.B}, {c.ks[2], c.ks[1], c.ks[0]}};
    const View4 vv{c.v, {c.D, ks_ext, c.Hkv, c.B}, {c.vs[2], c.vs[1], c.vs[0]}};
    const View4 vo{c.o, {c.D, c.S, c.H, c.B}, {c.os[2], c.os[1], c.os[0]}};
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

    auto kern = fa_prefill_kernel<T>;
    cudaError_t ce = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, T::SMEM_BYTES);
    if (ce != cudaSuccess) return fail(err, "%s", cudaGetErrorString(ce));
    kern<<<static_cast<unsigned>(items), T::THREADS, T::SMEM_BYTES, stream>>>(tmQ, tmK, tmV, tmO, p);
    ce = cudaGetLastError();
    if (ce != cudaSuccess) return fail(err, "%s", cudaGetErrorString(ce));
    return 0;
}

template <int D>
int dispatch_f16_dim(char* err, const Common& c, const prefill::Params& p, cudaStream_t st) {
    using namespace prefill;
    constexpr CUtensorMapDataType dt = CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
    if constexpr (D <= 128) {
        // two 128-row tiles per CTA, 128-key blocks
        constexpr int stages = D <= 32 ? 4 : D <= 64 ? 4 : D <= 96 ? 3 : 2;
        return launch_prefill<Traits<D, D, 128, 2, stages, stages, false>>(err, c, p, st, dt);
    } else if constexpr (D <= 256) {
        // one tile per CTA (TMEM holds one O of up to 256 columns), 64-key blocks
        constexpr int stages = D <= 192 ? 3 : 2;
        return launch_prefill<Traits<D, D, 64, 1, stages, stages, false>>(err, c, p, st, dt);
    } else {
        // head_dim > 256: two CTAs per tile, each owning half of the output columns
        constexpr int qk = 128 * D * 2, kt = 64 * D * 2, vt = 64 * 256 * 2;
        constexpr int stages = (2048 + qk + 2 * (kt + vt) <= 232448) ? 2 : 1;
        return launch_prefill<Traits<D, 256, 64, 1, stages, stages, false>>(err, c, p, st, dt);
    }
}

}  // namespace

int forwardF16(const ForwardParams& a, void* stream) {
    Common c{a.q, a.k, a.v, a.o,
             {a.qStrideB, a.qStrideH, a.qStrideS}, {a.kStrideB, a.kStrideH, a.kStrideS},
             {a.vStrideB, a.vStrideH, a.vStrideS}, {a.oStrideB, a.oStrideH, a.oStrideS},
             a.batchSize, a.numHeads, a.numKvHeads, a.seqLen, a.keySeqLen, a.headDim, 2};
    if (const char* e = check_common(c)) return fail(g_err_f16, "%s", e);
    if (a.headDim < 32 || a.headDim > 512 || a.headDim % 32 != 0)
        return fail(g_err_f16, "unsupported head_dim (multiples of 32 from 32 to 512)");
    if (a.hasRope) {
        if (a.rot_cos == nullptr || a.rot_sin == nullptr) return fail(g_err_f16, "has_rope set but rot_cos/rot_sin is null");
        if ((reinterpret_cast<uintptr_t>(a.rot_cos) & 15u) || (reinterpret_cast<uintptr_t>(a.rot_sin) & 15u))
            return fail(g_err_f16, "rot_cos/rot_sin must be 16-byte aligned");
    }
    if (a.seqLen > (1u << 30) || a.keySeqLen > (1u << 30)) return fail(g_err_f16, "sequence too long");

    prefill::Params p{};
    p.causal = a.causal ? 1 : 0;
    p.window = a.windowSize > 0 ? a.windowSize : 0;
    p.has_rope = a.hasRope ? 1 : 0;
    p.scale_log2 = a.scale * 1.4426950408889634f;
    p.rot_cos = static_cast<const float*>(a.rot_cos);
    p.rot_sin = static_cast<const float*>(a.rot_sin);
    cudaStream_t st = static_cast<cudaStream_t>(stream);

    if (!a.hasRope && decode::eligible(a.seqLen, a.numHeads / a.numKvHeads, a.headDim))
        return decode::launch_f16(g_err_f16, a, st);

    switch (a.headDim) {
#define RDNA_D(Dv) \
    case Dv: return dispatch_f16_dim<Dv>(g_err_f16, c, p, st);
        RDNA_D(32) RDNA_D(64) RDNA_D(96) RDNA_D(128) RDNA_D(160) RDNA_D(192) RDNA_D(224) RDNA_D(256)
        RDNA_D(288) RDNA_D(320) RDNA_D(352) RDNA_D(384) RDNA_D(416) RDNA_D(448) RDNA_D(480) RDNA_D(512)
#undef RDNA_D
        default:
            break;
    }
    return fail(g_err_f16, "unsupported head_dim (multiples of 32 from 32 to 512)");
}

int forwardInt8QK(const ForwardParamsInt8QK& a, void* stream) {
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
    p.has_rope = 0;
    p.scale_log2 = a.scale * 1.4426950408889634f;
    p.q_scale = a.qScale;
    p.k_scale = a.kScale;
    p.pv_scale = a.vScale / 127.0f;
    p.q_vec = static_cast<const float*>(a.qScaleVec);
    p.k_vec = static_cast<const float*>(a.kScaleVec);
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    constexpr CUtensorMapDataType dt = CU_TENSOR_MAP_DATA_TYPE_UINT8;
    if (a.headDim == 64)
        return launch_prefill<prefill::Traits<64, 64, 128, 2, 4, 4, true>>(g_err_i8, c, p, st, dt);
    return launch_prefill<prefill::Traits<128, 128, 128, 1, 3, 3, true>>(g_err_i8, c, p, st, dt);
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
