"""Split-KV decode path (seq_len * GQA group <= 64 rows in row groups of 16,
head_dim 64/128, with or without RoPE) vs the fp64 oracle.  Tolerance: max-abs <= 2e-3 and mean-abs
<= 2e-4 (the north-star FP16 gate), rel_rms < 3e-3 (tests/head_dim.py:49).
With RoPE the oracle rounds the rotated Q/K to fp16 as the reference kernel
does (src/rdna/fa2_forward_f16.hip:74-75)."""
import numpy as np
import pytest
import torch

from cases import rel_rms, rope_tables
from oracle import c_oracle

pytestmark = pytest.mark.gpu

R = pytest.importorskip("rdnattention_b200")


@pytest.fixture(scope="module", autouse=True)
def _device():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    yield
    assert R.debug_read_status() == (0, 0), "a kernel recorded an expired wait"


def _cache(B, Hkv, KS, D, g):
    """KV cache stored [B, KS, Hkv, D], viewed [B, Hkv, KS, D] through strides."""
    kb = torch.randn(B, KS, Hkv, D, generator=g).half()
    vb = torch.randn(B, KS, Hkv, D, generator=g).half()
    return kb, vb


def _check(got, ref):
    err = (got.double() - ref).abs()
    assert err.max().item() <= 2e-3, err.max().item()
    assert err.mean().item() <= 2e-4, err.mean().item()
    assert rel_rms(got, ref) < 3e-3


@pytest.mark.parametrize("B,H,Hkv,S,KS,D,causal,window", [
    (4, 64, 8, 1, 32768, 128, False, -1),   # decode B64 Hq64 Hkv8 KS32768 shape at B=4
    (2, 8, 2, 1, 300, 64, False, -1),        # key tail, D=64
    (3, 16, 4, 4, 1000, 128, True, -1),      # few-token decode, causal
    (2, 8, 8, 1, 777, 128, False, -1),       # MHA decode
    (1, 16, 1, 1, 5000, 128, False, -1),     # MQA, G=16 rows
    (2, 8, 2, 2, 4096, 128, True, 256),      # causal sliding window
    (2, 8, 2, 1, 4096, 64, False, 512),      # two-sided window
    (1, 4, 4, 1, 33, 128, False, -1),        # tiny: one CTA, two tiles
    (1, 4, 2, 1, 1, 128, False, -1),         # single key
    (2, 32, 4, 4, 2000, 128, True, -1),      # 32 rows per KV head: two row groups
    (1, 16, 1, 4, 3000, 64, False, 512),     # 64 rows: four row groups, window
    (2, 24, 4, 3, 777, 128, True, 100),      # 18 rows: a full and a 2-row group
])
def test_decode_vs_oracle(B, H, Hkv, S, KS, D, causal, window):
    g = torch.Generator().manual_seed(B * 1000 + KS)
    q = torch.randn(B, H, S, D, generator=g).half()
    kb, vb = _cache(B, Hkv, KS, D, g)
    got = R.flash_attn_strided(q.cuda(), kb.cuda().transpose(1, 2), vb.cuda().transpose(1, 2), is_causal=causal,
                               window_size=window).cpu()
    ref = c_oracle.attention_f16(q, kb.transpose(1, 2), vb.transpose(1, 2), causal=causal, window=window)
    _check(got, ref)


def test_decode_contiguous_cache_matches_strided():
    g = torch.Generator().manual_seed(3)
    q = torch.randn(2, 32, 1, 128, generator=g).half().cuda()
    kb, vb = _cache(2, 8, 3000, 128, g)
    a = R.flash_attn_strided(q, kb.cuda().transpose(1, 2), vb.cuda().transpose(1, 2))
    b = R.flash_attn(q, kb.transpose(1, 2).contiguous().cuda(), vb.transpose(1, 2).contiguous().cuda())
    assert torch.equal(a, b)


def test_decode_full_config5_sampled():
    """Decode at B=64, Hq=64, Hkv=8, KS=32768, D=128 (8.6 GB cache), sampled query heads vs the oracle."""
    B, H, Hkv, KS, D = 64, 64, 8, 32768, 128
    g = torch.Generator(device="cuda").manual_seed(5)
    q = torch.randn(B, H, 1, D, generator=g, device="cuda", dtype=torch.float16)
    kb = torch.randn(B, KS, Hkv, D, generator=g, device="cuda", dtype=torch.float16)
    vb = torch.randn(B, KS, Hkv, D, generator=g, device="cuda", dtype=torch.float16)
    out = R.flash_attn_strided(q, kb.transpose(1, 2), vb.transpose(1, 2))
    for b in (0, 37, 63):
        for h in (0, 13, 63):
            kvh = h // (H // Hkv)
            qq = q[b:b + 1, h:h + 1].cpu()
            kk = kb[b:b + 1, :, kvh:kvh + 1].cpu().transpose(1, 2)
            vv = vb[b:b + 1, :, kvh:kvh + 1].cpu().transpose(1, 2)
            ref = c_oracle.attention_f16(qq, kk, vv)
            _check(out[b:b + 1, h:h + 1].cpu(), ref)
    del kb, vb
    torch.cuda.empty_cache()


@pytest.mark.parametrize("B,H,Hkv,S,KS,D,causal,window,theta", [
    (2, 32, 8, 1, 4096, 128, False, -1, 500000.0),  # GQA decode step, theta 5e5
    (2, 8, 2, 4, 1000, 64, True, -1, 10000.0),      # few tokens, causal, D=64
    (1, 16, 1, 1, 3000, 128, False, 512, 1e6),      # MQA, two-sided window
    (1, 4, 4, 1, 33, 128, False, -1, 10000.0),      # key tail (zero-filled rows past KS)
    (2, 16, 2, 3, 1500, 128, True, -1, 500000.0),   # 24 rows per KV head: two row groups
    (1, 16, 2, 8, 777, 64, False, -1, 10000.0),      # 64 rows per KV head: four row groups, D=64, key tail
    (1, 8, 1, 5, 1300, 128, True, 256, 1e6),         # 40 rows: four row groups, causal + window
])
def test_decode_rope_vs_oracle(B, H, Hkv, S, KS, D, causal, window, theta):
    """RoPE inside the decode kernel: Q at its row position, each K row at its
    key position (reference semantics, no delta shift), cache read once."""
    g = torch.Generator().manual_seed(B * 77 + KS)
    q = torch.randn(B, H, S, D, generator=g).half()
    kb, vb = _cache(B, Hkv, KS, D, g)
    cos, sin = rope_tables(max(S, KS), D, theta)
    got = R.flash_attn_strided(q.cuda(), kb.cuda().transpose(1, 2), vb.cuda().transpose(1, 2), is_causal=causal,
                               window_size=window, rot_cos=cos.cuda(), rot_sin=sin.cuda()).cpu()
    ref = c_oracle.attention_f16(q, kb.transpose(1, 2), vb.transpose(1, 2), causal=causal, window=window,
                                 rot_cos=cos, rot_sin=sin, rope_round=True)
    _check(got, ref)
