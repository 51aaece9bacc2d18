"""fp32 torch-on-CPU oracle — TEST INFRASTRUCTURE / CPU BASELINE ONLY.

Restates tests/accuracy.py:39-47 (dense_attention_reference: per (batch,
head) ``softmax((q @ k^T) * scale) @ v``) in fp32, extended with:

* the masks of tests/head_dim.py:23-44 (causal aligned to the end of the key
  sequence, one-sided causal window, two-sided ``|q+delta-k| <= w//2``
  window), with rows that see no key returning 0 as the reference kernel does
  (src/rdna/fa2_forward_f16.hip:733);
* GQA head mapping h -> h // (H / Hkv) (tests/head_dim.py:32);
* interleaved-pair RoPE of tests/rope.py:29-37 (table row = position);
* INT8 operands dequantised per tests/hip_forward_int8qk_gate.hip:158-176.

Loops per (batch, kv-head) group and per query-row chunk to bound memory; each
chunk multiplies only the key columns some of its rows can see.
"""
import math
from typing import Optional

import torch


def rope_interleaved(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
    """(x[2i], x[2i+1]) -> (a*c - b*s, a*s + b*c), c/s = table[pos, i]; x is [..., S, D]."""
    S = x.shape[-2]
    c = cos[:S].to(x.dtype)
    s = sin[:S].to(x.dtype)
    a, b = x[..., 0::2], x[..., 1::2]
    out = torch.empty_like(x)
    out[..., 0::2] = a * c - b * s
    out[..., 1::2] = a * s + b * c
    return out


def _key_span(S: int, KS: int, causal: bool, window: int, q0: int, q1: int):
    """[lo, hi) of the keys any row in [q0, q1) can see (the whole range without masks)."""
    if not causal and window <= 0:
        return 0, KS
    delta = KS - S
    hi = KS
    lo = 0
    if causal:
        hi = min(KS, q1 - 1 + delta + 1)
    if window > 0:
        if causal:
            lo = max(0, q0 + delta - window + 1)
        else:
            lo = max(0, q0 + delta - window // 2)
            hi = min(hi, q1 - 1 + delta + window // 2 + 1)
    return lo, max(lo, hi)


def _mask(S: int, KS: int, causal: bool, window: int, q0: int, q1: int, k0: int = 0,
          k1: Optional[int] = None) -> Optional[torch.Tensor]:
    if not causal and window <= 0:
        return None
    k1 = KS if k1 is None else k1
    delta = KS - S
    qi = torch.arange(q0, q1).unsqueeze(1)
    ki = torch.arange(k0, k1).unsqueeze(0)
    keep = torch.ones(q1 - q0, k1 - k0, dtype=torch.bool)
    if causal:
        keep &= ki <= qi + delta
    if window > 0:
        if causal:
            keep &= (qi + delta - ki) < window
        else:
            keep &= (qi + delta - ki).abs() <= window // 2
    return keep


def attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, causal: bool = False, window: int = -1,
              rot_cos=None, rot_sin=None, scale=None, dtype=torch.float32, row_chunk: int = 4096,
              heads: Optional[range] = None) -> torch.Tensor:
    """Attention in `dtype` on CPU.  q [B,H,S,D], k/v [B,Hkv,KS,D] (any float dtype).

    ``heads`` restricts the computation to a range of query heads (the
    result then has len(heads) heads); used to time bounded samples.
    """
    B, H, S, D = q.shape
    Hkv, KS = k.shape[1], k.shape[2]
    G = H // Hkv
    if scale is None:
        scale = 1.0 / math.sqrt(D)
    heads = heads if heads is not None else range(H)
    out = torch.zeros(B, len(heads), S, v.shape[-1], dtype=dtype)
    cos = rot_cos.to(dtype) if rot_cos is not None else None
    sin = rot_sin.to(dtype) if rot_sin is not None else None
    for b in range(B):
        kv_cache = {}
        for oh, h in enumerate(heads):
            g = h // G
            if g not in kv_cache:
                kk = k[b, g].to(dtype)
                if cos is not None:
                    kk = rope_interleaved(kk, cos, sin)
                kv_cache = {g: (kk, v[b, g].to(dtype))}
            kk, vv = kv_cache[g]
            qq = q[b, h].to(dtype)
            if cos is not None:
                qq = rope_interleaved(qq, cos, sin)
            for q0 in range(0, S, row_chunk):
                q1 = min(S, q0 + row_chunk)
                # only the keys some row of the chunk can see (masked scores are -inf,
                # so dropping whole masked columns changes nothing)
                k0, k1 = _key_span(S, KS, causal, window, q0, q1)
                if k1 <= k0:
                    continue  # no row of the chunk sees a key: output 0
                s = (qq[q0:q1] @ kk[k0:k1].transpose(0, 1)) * scale
                keep = _mask(S, KS, causal, window, q0, q1, k0, k1)
                if keep is not None:
                    s = s.masked_fill(~keep, float("-inf"))
                    empty = ~keep.any(dim=1)
                    p = torch.softmax(s, dim=-1)
                    p = torch.nan_to_num(p, nan=0.0)
                    p[empty] = 0.0
                else:
                    p = torch.softmax(s, dim=-1)
                out[b, oh, q0:q1] = p @ vv[k0:k1]
    return out


def attention_int8_dequant(qi, ki, vi, q_scale, k_scale, v_scale, causal=False, window=-1, scale=None,
                           dtype=torch.float32) -> torch.Tensor:
    """Dequantise (per-tensor or per-token Q/K scales, scalar V) then attend, unquantised P."""
    qf = qi.to(dtype)
    kf = ki.to(dtype)
    qf = qf * (q_scale.to(dtype).unsqueeze(-1) if isinstance(q_scale, torch.Tensor) else float(q_scale))
    kf = kf * (k_scale.to(dtype).unsqueeze(-1) if isinstance(k_scale, torch.Tensor) else float(k_scale))
    vf = vi.to(dtype) * float(v_scale)
    return attention(qf, kf, vf, causal=causal, window=window, scale=scale, dtype=dtype)


def valid_pairs(S: int, KS: int, causal: bool, window: int) -> int:
    """Exact number of visible (query, key) pairs per head (extends tests/benchmark.py:77-88 to windows)."""
    total = 0
    delta = KS - S
    if not causal and window <= 0:
        return S * KS
    for qq in range(S):
        lo, hi = 0, KS - 1
        if causal:
            hi = min(hi, qq + delta)
        if window > 0:
            if causal:
                lo = max(lo, qq + delta - window + 1)
            else:
                lo = max(lo, qq + delta - window // 2)
                hi = min(hi, qq + delta + window // 2)
        if hi >= lo:
            total += hi - lo + 1
    return total


def flops(B: int, H: int, S: int, KS: int, D: int, causal: bool, window: int) -> int:
    """Both GEMMs at 2 FLOP/MAC over exactly the visible pairs (tests/benchmark.py:77-88)."""
    return 4 * B * H * D * valid_pairs(S, KS, causal, window)
