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
    Tensor4 t[2];        // Q, K
    int64_t chunks[2];   // 16-byte chunks per tensor
    const float* cos_t;
    const float* sin_t;
    int D;
};

__global__ void __launch_bounds__(256) rope_rotate_kernel(const __grid_constant__ Params p) {
    const int cpr = p.D / 8;  // chunks per row
    const int64_t total = p.chunks[0] + p.chunks[1];
    for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const int which = i < p.chunks[0] ? 0 : 1;
        const Tensor4& T = p.t[which];
        const int64_t c = which == 0 ? i : i - p.chunks[0];
        const int ch = static_cast<int>(c % cpr);
        const int64_t row = c / cpr;  // (b * H + h) * S + s
        const int s = static_cast<int>(row % T.S);
        const int64_t bh = row / T.S;
        const int h = static_cast<int>(bh % T.H);
        const int b = static_cast<int>(bh / T.H);
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
            const __half2 r = __floats2half2_rn(a * cc[k] - bb * ss[k], a * ss[k] + bb * cc[k]);
            w[k] = *reinterpret_cast<const uint32_t*>(&r);
        }
        *reinterpret_cast<uint4*>(T.dst + row * p.D + ch * 8) = y;
    }
}

}  // namespace rope
}  // namespace rdna
