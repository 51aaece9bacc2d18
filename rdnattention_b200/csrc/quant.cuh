// Device-side INT8 quantisation for the INT8 attention path: one launch turns
// fp16 Q/K/V into the operands of the fused per-channel-V kernel.
//
//   Q, K: one scale per (batch, head, row) = max|x| / 127 (0 -> 1), the row
//         quantised to round-half-even(x / scale) clamped to [-127, 127];
//   V:    one scale per (batch, kv head, head_dim column) = max over the
//         sequence of |v| / 127 (0 -> 1), quantised the same way; the
//         attention epilogue multiplies O by it (attention is linear in V).
//
// Same arithmetic as the reference helpers (rdnattention/__init__.py:303-343)
// run on CUDA tensors: fp32 max; `max / 127.0`, which torch evaluates on the
// GPU as a multiplication by the fp32 reciprocal of the scalar; fp32 x / scale
// (a tensor divisor: true division); torch.round = half-even; clamp — so the
// outputs are bit-identical.  HBM-bound streaming kernel: Q and K are read
// once, V twice (its scales need the whole sequence first).
#pragma once

#include <cuda_fp16.h>

#include <cstdint>

namespace rdna {
namespace quant {

struct Rows {
    const __half* src;  // strided [B, H, S, D]
    int8_t* dst;        // contiguous [B, H, S, D]
    float* scale;       // contiguous [B, H, S]
    int64_t sb, sh, ss;
    int H, S;
    int64_t rows;       // B * H * S
};

struct Params {
    Rows t[2];          // Q, K
    // V: per (batch, kv head) block
    const __half* v;
    int8_t* vi;         // contiguous [B, Hkv, KS, D]
    float* vch;         // contiguous [B, Hkv, D]
    int64_t vsb, vsh, vss;
    int Hkv, KS;
    int D;
    int blocks_q, blocks_k;  // CTAs of the per-token part (then one CTA per (b, kv head) of V)
};

constexpr int kThreads = 256;

// max|x| / 127 as torch computes it for a CUDA tensor and a Python-scalar
// divisor (x * (1 / 127) in fp32); 0 -> 1
__device__ __forceinline__ float scale_of(float m) {
    const float s = __fmul_rn(m, 1.0f / 127.0f);
    return s == 0.f ? 1.f : s;
}

__device__ __forceinline__ int8_t q8(float x, float s) {
    float r = rintf(__fdiv_rn(x, s));  // round half to even, as torch.round
    r = fminf(fmaxf(r, -127.f), 127.f);
    return static_cast<int8_t>(r);
}

// 8 halves (one 16-byte chunk) -> 8 floats
__device__ __forceinline__ void unpack8(const uint4& u, float* f) {
    const __half2* h = reinterpret_cast<const __half2*>(&u);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const float2 v = __half22float2(h[i]);
        f[2 * i] = v.x;
        f[2 * i + 1] = v.y;
    }
}

__device__ __forceinline__ uint2 pack8(const int8_t* b) {
    uint2 r;
    r.x = (uint32_t)(uint8_t)b[0] | ((uint32_t)(uint8_t)b[1] << 8) | ((uint32_t)(uint8_t)b[2] << 16) |
          ((uint32_t)(uint8_t)b[3] << 24);
    r.y = (uint32_t)(uint8_t)b[4] | ((uint32_t)(uint8_t)b[5] << 8) | ((uint32_t)(uint8_t)b[6] << 16) |
          ((uint32_t)(uint8_t)b[7] << 24);
    return r;
}

// Per-token rows: a group of D/8 lanes per row (D in {64, 128}: 8 or 16 lanes),
// each lane one 16-byte chunk; the row max is a shuffle reduction inside the group.
__device__ void token_rows(const Rows& R, int D, int64_t block, int64_t nblocks) {
    const int cpr = D / 8;                  // chunks (lanes) per row
    const int rpw = 32 / cpr;               // rows per warp
    const int lane = threadIdx.x % 32;
    const int sub = lane / cpr, ch = lane % cpr;
    const int64_t warps_total = nblocks * (kThreads / 32);
    const int64_t wid = block * (kThreads / 32) + threadIdx.x / 32;
    for (int64_t r0 = wid * rpw; r0 < R.rows; r0 += warps_total * rpw) {
        const int64_t row = r0 + sub;
        const bool live = row < R.rows;
        float f[8];
        float m = 0.f;
        if (live) {
            const int64_t s = row % R.S, bh = row / R.S;
            const int64_t h = bh % R.H, b = bh / R.H;
            const uint4 u = *reinterpret_cast<const uint4*>(R.src + b * R.sb + h * R.sh + s * R.ss + ch * 8);
            unpack8(u, f);
#pragma unroll
            for (int i = 0; i < 8; ++i) m = fmaxf(m, fabsf(f[i]));
        }
        for (int off = cpr / 2; off > 0; off >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, off));
        if (live) {
            const float sc = scale_of(m);
            int8_t b8[8];
#pragma unroll
            for (int i = 0; i < 8; ++i) b8[i] = q8(f[i], sc);
            *reinterpret_cast<uint2*>(R.dst + row * D + ch * 8) = pack8(b8);
            if (ch == 0) R.scale[row] = sc;
        }
    }
}

// V of one (batch, kv head): column maxima over the sequence (thread = one
// 16-byte column chunk of every G-th row, then a shared-memory reduction over
// the row groups), scales, then a second pass that quantises.
__device__ void v_unit(const Params& p, int unit, float* red, float* scl) {
    const int D = p.D, cpr = D / 8, groups = kThreads / cpr;
    const int ch = threadIdx.x % cpr, grp = threadIdx.x / cpr;
    const int b = unit / p.Hkv, h = unit % p.Hkv;
    const __half* base = p.v + b * p.vsb + h * p.vsh + ch * 8;
    float m[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    for (int s = grp; s < p.KS; s += groups) {
        const uint4 u = *reinterpret_cast<const uint4*>(base + s * p.vss);
        float f[8];
        unpack8(u, f);
#pragma unroll
        for (int i = 0; i < 8; ++i) m[i] = fmaxf(m[i], fabsf(f[i]));
    }
#pragma unroll
    for (int i = 0; i < 8; ++i) red[grp * D + ch * 8 + i] = m[i];
    __syncthreads();
    for (int c = threadIdx.x; c < D; c += kThreads) {
        float mx = 0.f;
        for (int g = 0; g < groups; ++g) mx = fmaxf(mx, red[g * D + c]);
        const float sc = scale_of(mx);
        scl[c] = sc;
        p.vch[static_cast<int64_t>(unit) * D + c] = sc;
    }
    __syncthreads();
    int8_t* out = p.vi + static_cast<int64_t>(unit) * p.KS * D + ch * 8;
    for (int s = grp; s < p.KS; s += groups) {
        const uint4 u = *reinterpret_cast<const uint4*>(base + s * p.vss);
        float f[8];
        unpack8(u, f);
        int8_t b8[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) b8[i] = q8(f[i], scl[ch * 8 + i]);
        *reinterpret_cast<uint2*>(out + static_cast<int64_t>(s) * D) = pack8(b8);
    }
}

// blocks [0, blocks_q): Q rows; [blocks_q, blocks_q + blocks_k): K rows;
// then one block per (batch, kv head) of V.
__global__ void __launch_bounds__(kThreads) quantize_qkv_kernel(const __grid_constant__ Params p) {
    __shared__ float red[kThreads / 8 * 128];  // row groups x columns (D <= 128)
    __shared__ float scl[128];
    const int bx = blockIdx.x;
    if (bx < p.blocks_q) {
        token_rows(p.t[0], p.D, bx, p.blocks_q);
    } else if (bx < p.blocks_q + p.blocks_k) {
        token_rows(p.t[1], p.D, bx - p.blocks_q, p.blocks_k);
    } else {
        v_unit(p, bx - p.blocks_q - p.blocks_k, red, scl);
    }
}

}  // namespace quant
}  // namespace rdna
