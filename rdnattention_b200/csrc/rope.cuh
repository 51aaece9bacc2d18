// RoPE pre-pass: rotates Q and K once per launch into a contiguous fp16
// workspace, so the attention kernel's tiles are already rotated when TMA
// brings them into shared memory.
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
// Index math is per row and 32-bit (rows < 2^31).
__global__ void __launch_bounds__(256) rope_rotate_kernel(const __grid_constant__ Params p) {
    const int ch = threadIdx.x % p.cpr;
    const int rsub = threadIdx.x / p.cpr;
    if (rsub >= p.rpb) return;
    const int total = p.rows[0] + p.rows[1];
    for (int row = blockIdx.x * p.rpb + rsub; row < total; row += gridDim.x * p.rpb) {
        const int which = row < p.rows[0] ? 0 : 1;
        const Tensor4& T = p.t[which];
        const unsigned r = static_cast<unsigned>(which == 0 ? row : row - p.rows[0]);
        const unsigned s = r % static_cast<unsigned>(T.S);
        const unsigned bh = r / static_cast<unsigned>(T.S);
        const unsigned h = bh % static_cast<unsigned>(T.H);
        const unsigned b = bh / static_cast<unsigned>(T.H);
        const uint4 x = *reinterpret_cast<const uint4*>(T.src + b * T.sb + h * T.sh + s * T.ss + ch * 8);
        const int64_t toff = static_cast<int64_t>(s) * (p.D / 2) + ch * 4;
        const float4 cv = __ldg(reinterpret_cast<const float4*>(p.cos_t + toff));
        const float4 sv = __ldg(reinterpret_cast<const float4*>(p.sin_t + toff));
        const float cc[4] = {cv.x, cv.y, cv.z, cv.w};
        const float ss[4] = {sv.x, sv.y, sv.z, sv.w};
        const uint32_t* u = reinterpret_cast<const uint32_t*>(&x);
        uint4 y;
        uint32_t* w = reinterpret_cast<uint32_t*>(&y);
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            const __half2 h2 = *reinterpret_cast<const __half2*>(&u[k]);
            const float a = __low2float(h2), bb = __high2float(h2);
            const __half2 rr = __floats2half2_rn(a * cc[k] - bb * ss[k], a * ss[k] + bb * cc[k]);
            w[k] = *reinterpret_cast<const uint32_t*>(&rr);
        }
        *reinterpret_cast<uint4*>(T.dst + static_cast<int64_t>(r) * p.D + ch * 8) = y;
    }
}

}  // namespace rope
}  // namespace rdna
