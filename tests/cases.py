"""Case lists of the reference's own correctness gates, and input builders.

The shapes below restate the case tables of the reference's gates (data, not
code): tests/hip_forward_gate.hip:259-316 (FP16, 50 cases, LCG seed 12345,
rel_rms < 5e-3) and tests/hip_forward_int8qk_gate.hip:264-317 (INT8, 38
cases, LCG seed 424242, rel_rms < 5e-2), plus the head_dim sweep variants of
tests/head_dim.py:10-20 and the RoPE cases of tests/rope.py:66-73.
"""
import numpy as np
import torch

from oracle import c_oracle

# (name, batch, heads, kv_heads, seq, key_seq, head_dim, causal, window, rope)
F16_GATE = [
    ("d64_dense_small", 1, 4, 4, 96, 96, 64, False, 0, False),
    ("d64_dense_tail", 2, 4, 4, 200, 200, 64, False, 0, False),
    ("d64_causal", 1, 4, 4, 257, 257, 64, True, 0, False),
    ("d64_gqa_causal", 1, 8, 2, 300, 300, 64, True, 0, False),
    ("d64_gqa_ratio2_exact", 1, 8, 4, 300, 300, 64, True, 0, False),
    ("d64_gqa_ratio8", 1, 16, 2, 300, 300, 64, True, 0, False),
    ("d64_gqa_ratio3_pad", 2, 6, 2, 257, 257, 64, True, 0, False),
    ("d64_gqa_ratio6_even", 1, 12, 2, 300, 300, 64, False, 0, False),
    ("d64_gqa_ratio5_pad", 2, 10, 2, 199, 199, 64, True, 64, True),
    ("d64_gqa_batch4", 4, 8, 2, 96, 96, 64, False, 0, False),
    ("d64_mqa", 2, 8, 1, 199, 199, 64, True, 0, False),
    ("d64_gqa_decode_1tok", 1, 8, 2, 1, 300, 64, False, 0, False),
    ("d64_gqa_decode_few", 2, 16, 4, 4, 300, 64, False, 0, False),
    ("d64_gqa_window", 1, 8, 2, 300, 300, 64, False, 64, False),
    ("d64_gqa_numkv8", 1, 32, 8, 256, 256, 64, True, 0, True),
    ("d64_window", 1, 4, 4, 300, 300, 64, False, 64, False),
    ("d64_causal_window", 1, 4, 4, 300, 300, 64, True, 32, False),
    ("d64_rope_causal", 2, 4, 4, 271, 271, 64, True, 0, True),
    ("d64_kv_longer", 1, 4, 4, 64, 300, 64, False, 0, False),
    ("d128_dense", 1, 4, 4, 130, 130, 128, False, 0, False),
    ("d128_causal", 1, 4, 4, 150, 150, 128, True, 0, False),
    ("d128_rope_gqa_causal", 1, 8, 4, 199, 199, 128, True, 0, True),
    ("d32_dense", 1, 2, 2, 100, 100, 32, False, 0, False),
    ("d96_dense", 1, 2, 2, 100, 100, 96, False, 0, False),
    ("d160_dense", 1, 2, 2, 100, 100, 160, False, 0, False),
    ("d192_dense", 1, 2, 2, 100, 100, 192, False, 0, False),
    ("d224_dense", 1, 2, 2, 100, 100, 224, False, 0, False),
    ("d256_dense", 1, 2, 2, 100, 100, 256, False, 0, False),
    ("d288_dense", 1, 2, 2, 100, 100, 288, False, 0, False),
    ("d320_dense", 1, 2, 2, 100, 100, 320, False, 0, False),
    ("d352_dense", 1, 2, 2, 100, 100, 352, False, 0, False),
    ("d384_dense", 1, 2, 2, 100, 100, 384, False, 0, False),
    ("d416_dense", 1, 2, 2, 100, 100, 416, False, 0, False),
    ("d448_dense", 1, 2, 2, 100, 100, 448, False, 0, False),
    ("d480_dense", 1, 2, 2, 100, 100, 480, False, 0, False),
    ("d512_dense", 1, 2, 2, 100, 100, 512, False, 0, False),
    ("d384_causal", 1, 2, 2, 100, 100, 384, True, 0, False),
    ("d384_gqa_causal", 1, 8, 2, 100, 100, 384, True, 0, False),
    ("d384_window", 1, 2, 2, 100, 100, 384, False, 32, False),
    ("d384_causal_window", 1, 2, 2, 100, 100, 384, True, 32, False),
    ("d384_rope_causal", 1, 2, 2, 100, 100, 384, True, 0, True),
    ("d384_kv_longer", 1, 2, 2, 40, 100, 384, False, 0, False),
    ("d384_decode_1tok", 1, 4, 2, 1, 100, 384, False, 0, False),
    ("d512_causal", 1, 2, 2, 100, 100, 512, True, 0, False),
    ("d512_gqa_rope_causal", 1, 4, 2, 100, 100, 512, True, 0, True),
    ("d512_window", 1, 2, 2, 100, 100, 512, False, 32, False),
    ("d512_kv_longer", 1, 2, 2, 40, 100, 512, False, 0, False),
    ("d256_rope_causal", 1, 2, 2, 100, 100, 256, True, 0, True),
    ("d256_gqa_window", 1, 8, 2, 100, 100, 256, False, 32, False),
    ("d352_causal_aligned", 1, 2, 2, 96, 96, 352, True, 0, False),
]

# (name, batch, heads, seq, key_seq, head_dim, kv_heads (0 = heads), causal, window, per_token)
I8_GATE = [
    ("d64_small", 1, 4, 96, 96, 64, 0, False, -1, False),
    ("d64_tail", 2, 4, 200, 200, 64, 0, False, -1, False),
    ("d64_batch4", 4, 8, 128, 128, 64, 0, False, -1, False),
    ("d64_kv_longer", 1, 4, 64, 300, 64, 0, False, -1, False),
    ("d64_single_head", 1, 1, 257, 257, 64, 0, False, -1, False),
    ("d64_large", 2, 16, 512, 512, 64, 0, False, -1, False),
    ("d64_br128_clean", 1, 8, 1024, 1024, 64, 0, False, -1, False),
    ("d64_br128_tail", 2, 4, 1300, 1300, 64, 0, False, -1, False),
    ("d64_causal", 1, 4, 256, 256, 64, 0, True, -1, False),
    ("d64_causal_tail", 2, 4, 200, 200, 64, 0, True, -1, False),
    ("d64_causal_br128", 1, 4, 1024, 1024, 64, 0, True, -1, False),
    ("d64_causal_kv_longer", 1, 4, 64, 300, 64, 0, True, -1, False),
    ("d64_causal_decode", 1, 4, 1, 256, 64, 0, True, -1, False),
    ("d64_window", 1, 4, 256, 256, 64, 0, False, 64, False),
    ("d64_causal_window", 1, 4, 256, 256, 64, 0, True, 64, False),
    ("d64_gqa_r2", 1, 8, 256, 256, 64, 4, False, -1, False),
    ("d64_gqa_r8", 1, 8, 256, 256, 64, 1, False, -1, False),
    ("d64_mqa_causal", 2, 8, 300, 300, 64, 1, True, -1, False),
    ("d64_gqa_r4_br128", 1, 8, 1024, 1024, 64, 2, False, -1, False),
    ("d128_small", 1, 4, 96, 96, 128, 0, False, -1, False),
    ("d128_tail", 2, 4, 200, 200, 128, 0, False, -1, False),
    ("d128_causal", 1, 4, 256, 256, 128, 0, True, -1, False),
    ("d128_gqa_causal", 1, 8, 300, 300, 128, 2, True, -1, False),
    ("d128_kv_longer", 1, 4, 64, 300, 128, 0, False, -1, False),
    ("d128_large", 1, 8, 1024, 1024, 128, 0, False, -1, False),
    ("d128_br128", 1, 2, 2048, 2048, 128, 0, False, -1, False),
    ("d128_br128_tail", 1, 2, 2100, 2100, 128, 0, False, -1, False),
    ("d128_br128_bh", 8, 16, 1024, 64, 128, 0, False, -1, False),
    ("d128_br128_causal", 1, 2, 2048, 2048, 128, 0, True, -1, False),
    ("ptok_d64", 1, 4, 256, 256, 64, 0, False, -1, True),
    ("ptok_d64_tail", 2, 4, 200, 200, 64, 0, False, -1, True),
    ("ptok_d64_causal", 1, 4, 256, 256, 64, 0, True, -1, True),
    ("ptok_d64_window", 1, 4, 256, 256, 64, 0, True, 64, True),
    ("ptok_d64_gqa", 1, 8, 256, 256, 64, 2, False, -1, True),
    ("ptok_d64_kvlonger", 1, 4, 64, 300, 64, 0, False, -1, True),
    ("ptok_d64_br128", 1, 4, 1024, 1024, 64, 0, True, -1, True),
    ("ptok_d128", 1, 4, 256, 256, 128, 0, False, -1, True),
    ("ptok_d128_gqa_c", 1, 8, 300, 300, 128, 2, True, -1, True),
]

# tests/head_dim.py:10-20 (name, kv divisor, seq, key_seq, causal, window)
HEAD_DIM_VARIANTS = [
    ("dense", 1, 300, 300, False, -1), ("causal", 1, 300, 300, True, -1), ("gqa", 4, 300, 300, False, -1),
    ("gqa_causal", 4, 300, 300, True, -1), ("window", 1, 300, 300, False, 64),
    ("causal_window", 1, 300, 300, True, 32), ("cross", 1, 200, 300, False, -1),
    ("decode", 1, 1, 300, False, -1), ("aligned", 1, 256, 256, True, -1),
]

# tests/rope.py:66-73 (name, B, H, KH, S, KS, D, causal)
ROPE_CASES = [
    ("MHA d64 rope", 1, 8, 8, 256, 256, 64, False), ("MHA d128 rope", 2, 8, 8, 512, 512, 128, False),
    ("causal d64 rope", 1, 8, 8, 256, 256, 64, True), ("causal d128 rope", 1, 8, 8, 384, 384, 128, True),
    ("GQA d64 rope", 1, 8, 2, 256, 256, 64, False), ("cross-attn d64 rope", 1, 8, 8, 128, 512, 64, False),
    ("tail 300 rope", 1, 8, 8, 300, 300, 64, False),
]


def gate_f16_inputs(B, H, Hkv, S, KS, D, rope):
    """LCG seed 12345 stream q, k, v rounded to fp16; the gate's theta=10000 tables over KS rows."""
    qf, s2 = c_oracle.lcg_uniform(12345, B * H * S * D)
    kf, s3 = c_oracle.lcg_uniform(0, B * Hkv * KS * D, state=s2)
    vf, _ = c_oracle.lcg_uniform(0, B * Hkv * KS * D, state=s3)
    q = torch.from_numpy(qf.astype(np.float16)).reshape(B, H, S, D)
    k = torch.from_numpy(kf.astype(np.float16)).reshape(B, Hkv, KS, D)
    v = torch.from_numpy(vf.astype(np.float16)).reshape(B, Hkv, KS, D)
    cos = sin = None
    if rope:
        rows = max(S, KS)
        half = D // 2
        s = np.arange(rows, dtype=np.float32)[:, None]
        p = np.arange(half, dtype=np.float32)[None, :]
        theta = (s / np.power(np.float32(10000.0), (2.0 * p / np.float32(D)).astype(np.float32))).astype(np.float32)
        cos = torch.from_numpy(np.cos(theta).astype(np.float32))
        sin = torch.from_numpy(np.sin(theta).astype(np.float32))
    return q, k, v, cos, sin


def gate_i8_inputs(B, H, Hkv, S, KS, D, per_token):
    """tests/hip_forward_int8qk_gate.hip:131-176: LCG seed 424242 gaussian-ish values,
    per-tensor (absmax/127) or per-token scales, the gate's quantiser."""
    qf, s2 = c_oracle.lcg_gaussianish(424242, B * H * S * D)
    kf, s3 = c_oracle.lcg_gaussianish(0, B * Hkv * KS * D, state=s2)
    vf, _ = c_oracle.lcg_gaussianish(0, B * Hkv * KS * D, state=s3)
    qsc = np.float32(np.abs(qf).max() / np.float32(127.0))
    ksc = np.float32(np.abs(kf).max() / np.float32(127.0))
    vsc = np.float32(np.abs(vf).max() / np.float32(127.0))
    qvec = np.full(B * H * S, qsc, dtype=np.float32)
    kvec = np.full(B * Hkv * KS, ksc, dtype=np.float32)
    if per_token:
        qm = np.abs(qf.reshape(-1, D)).max(axis=1)
        km = np.abs(kf.reshape(-1, D)).max(axis=1)
        qvec = np.where(qm > 0, qm / np.float32(127.0), np.float32(1.0)).astype(np.float32)
        kvec = np.where(km > 0, km / np.float32(127.0), np.float32(1.0)).astype(np.float32)
    qi = c_oracle.quantize(qf, qvec, D).reshape(B, H, S, D)
    ki = c_oracle.quantize(kf, kvec, D).reshape(B, Hkv, KS, D)
    vi = c_oracle.quantize(vf, np.array([vsc], dtype=np.float32), vf.size).reshape(B, Hkv, KS, D)
    return (torch.from_numpy(qi), torch.from_numpy(ki), torch.from_numpy(vi), float(qsc), float(ksc), float(vsc),
            torch.from_numpy(qvec.reshape(B, H, S)), torch.from_numpy(kvec.reshape(B, Hkv, KS)))


def rope_tables(rows, D, theta=10000.0, device="cpu"):
    """tests/rope.py:78-82 / docs/api.md:84-87: ang = pos * theta^(-2i/D)."""
    pos = torch.arange(rows, device=device).unsqueeze(1).float()
    inv = theta ** (-torch.arange(0, D, 2, device=device).float() / D)
    ang = pos * inv
    return ang.cos().contiguous(), ang.sin().contiguous()


def rel_rms(got, ref):
    got = got.double().cpu()
    ref = ref.double().cpu()
    den = ref.pow(2).sum().sqrt()
    num = (got - ref).pow(2).sum().sqrt()
    return (num / den).item() if den > 0 else num.item()
