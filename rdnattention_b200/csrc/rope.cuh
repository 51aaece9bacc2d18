// RoPE pre-pass: rotates K (and, for the kernels that do not rotate Q
// themselves, Q) once per launch into a contiguous fp16 workspace, so the
// attention kernel's K tiles are already rotated when TMA brings them into
// shared memory.
//
// Interleaved pairs, as the reference kernel applies them
// (src/rdna/fa2_forward_f16.hip:63-77): (x[2i], x[2i+1]) ->
// (a*c - b*s, a*s + b*c) with c/s = table[pos][i] (fp32), computed in fp32 and
// rounded to fp16; pos = row index within the tensor.
//
// One thread moves one 16-byte chunk (8 halves = 4 pairs) per iteration:
// a coalesced 16 B load of x, two 16 B loads of the tables (L2-resident,
// shared by every head and batch), one 16 B store.  HBM-bound.
#pragma once

#include <cuda_fp16.h>

#include <cstdint>

namespace rdna {
namespace rope {

// One interleaved pair (x[2i], x[2i+1]) packed as half2 -> (a*c - b*s, a*s + b*c),
// fp32 math rounded to fp16.  Shared by the pre-pass, the prefill kernel's Q
// rotation and the decode kernel, so every path rotates identically.
__device__ __forceinline__ uint32_t rotate_pair(uint32_t v, float c, float s) {
    const __half2 h2 = *reinterpret_cast<const __half2*>(&v);
    const float a = __low2float(h2), b = __high2float(h2);
    // explicit roundings, so every kernel that inlines this computes the same bits
    const __half2 r = __floats2half2_rn(__fmaf_rn(a, c, -__fmul_rn(b, s)), __fmaf_rn(a, s, __fmul_rn(b, c)));
    return *reinterpret_cast<const uint32_t*>(&r);
}

// One 16-byte chunk (4 pairs) in place; c/s hold the pairs' table entries.
__device__ __forceinline__ void rotate_chunk(uint8_t* ptr, const float4& c, const float4& s) {
    uint4 x = *reinterpret_cast<const uint4*>(ptr);
    x.x = rotate_pair(x.x, c.x, s.x);
    x.y = rotate_pair(x.y, c.y, s.y);
    x.z = rotate_pair(x.z, c.z, s.z);
    x.w = rotate_pair(x.w, c.w, s.w);
    *reinterpret_cast<uint4*>(ptr) = x;
}

struct Tensor4 {
    const __half* src;
    __half* dst;  // contiguous [B, H, S, D]
    int64_t sb, sh, ss;
    int B, H, S;
};

struct Params {
    Tensor4 t[2];    // Q, K
    int rows[2];     // B * H * S rows per tensor
    const float* cos_t;
    const float* sin_t;
    int D;
    int cpr;         // 16-byte chunks per row (D / 8)
    int rpb;         // rows per block iteration (blockDim.x / cpr)
};

// blockDim.x = rpb * cpr: thread -> (row within the block's slab, chunk).
// Index math is per row and 32-bit (rows < 2^31).  Each thread handles two rows
// per iteration with both loads issued before either store, so twice the bytes
// are in flight per thread.  The first statement lets a dependent attention
// kernel (launched with programmatic stream serialization) start its prologue
// while this grid drains; that kernel waits for this grid's stores before it
// reads the rotated rows.
__device__ __forceinline__ const __half* rope_src(const Params& p, int row, int ch, int& which, unsigned& r,
                                                 unsigned& s) {
    which = row < p.rows[0] ? 0 : 1;
    const Tensor4& T = p.t[which];
    r = static_cast<unsigned>(which == 0 ? row : row - p.rows[0]);
    s = r % static_cast<unsigned>(T.S);
    const unsigned bh = r / static_cast<unsigned>(T.S);
    const unsigned h = bh % static_cast<unsigned>(T.H);
    const unsigned b = bh / static_cast<unsigned>(T.H);
    return T.src + b * T.sb + h * T.sh + s * T.ss + ch * 8;
}

__device__ __forceinline__ void rope_store(const Params& p, int which, unsigned r, unsigned s, int ch,
                                           const uint4& x) {
    const int64_t toff = static_cast<int64_t>(s) * (p.D / 2) + ch * 4;
    const float4 cv = __ldg(reinterpret_cast<const float4*>(p.cos_t + toff));
    const float4 sv = __ldg(reinterpret_cast<const float4*>(p.sin_t + toff));
    const uint4 y{rotate_pair(x.x, cv.x, sv.x), rotate_pair(x.y, cv.y, sv.y), rotate_pair(x.z, cv.z, sv.z),
                  rotate_pair(x.w, cv.w, sv.w)};
    *reinterpret_cast<uint4*>(p.t[which].dst + static_cast<int64_t>(r) * p.D + ch * 8) = y;
}

__global__ void __launch_bounds__(256) rope_rotate_kernel(const __grid_constant__ Params p) {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    const int ch = threadIdx.x % p.cpr;
    const int rsub = threadIdx.x / p.cpr;
    if (rsub >= p.rpb) return;
    const int64_t total = static_cast<int64_t>(p.rows[0]) + p.rows[1];
    const int64_t stride = static_cast<int64_t>(gridDim.x) * p.rpb;
    for (int64_t row = static_cast<int64_t>(blockIdx.x) * p.rpb + rsub; row < total; row += 2 * stride) {
        int w0, w1 = 0;
        unsigned r0, s0, r1 = 0, s1 = 0;
        const uint4 x0 = *reinterpret_cast<const uint4*>(rope_src(p, static_cast<int>(row), ch, w0, r0, s0));
        const bool two = row + stride < total;
        uint4 x1{0u, 0u, 0u, 0u};
        if (two) x1 = *reinterpret_cast<const uint4*>(rope_src(p, static_cast<int>(row + stride), ch, w1, r1, s1));
        rope_store(p, w0, r0, s0, ch, x0);
        if (two) rope_store(p, w1, r1, s1, ch, x1);
    }
}

}  // namespace rope
}  // namespace rdna
