"""ctypes wrapper over oracle/attn_oracle.c — TEST INFRASTRUCTURE ONLY.

Takes CPU torch tensors (any strides, head_dim contiguous) and returns
float64 results.  See attn_oracle.c for the reference lines each function
restates.
"""
import ctypes
from typing import Optional, Sequence

import numpy as np
import torch

from . import build as _build

_lib = None


def lib():
    global _lib
    if _lib is None:
        path = _build.LIB if _build.LIB.exists() else _build.build()
        L = ctypes.CDLL(str(path))
        i64, i32, f32, f64, vp = ctypes.c_int64, ctypes.c_int32, ctypes.c_float, ctypes.c_double, ctypes.c_void_p
        L.oracle_attention_f16.argtypes = [vp] * 5 + [i64] * 9 + [i64] * 6 + [f64] + [i32] * 4 + [vp, i64, vp]
        L.oracle_attention_f16.restype = ctypes.c_int
        L.oracle_attention_int8.argtypes = [vp] * 3 + [i64] * 9 + [i64] * 6 + [f64, f32, f32, f32, vp, vp, i32, i32,
                                                                              vp, i64, vp]
        L.oracle_attention_int8.restype = ctypes.c_int
        L.oracle_lcg_uniform.argtypes = [ctypes.POINTER(ctypes.c_uint32), vp, i64]
        L.oracle_lcg_gaussianish.argtypes = [ctypes.POINTER(ctypes.c_uint32), vp, i64]
        L.oracle_quantize.argtypes = [vp, i64, vp, i64, vp]
        L.oracle_key_range.argtypes = [i64, i64, i64, i32, i32, ctypes.POINTER(i64), ctypes.POINTER(i64)]
        L.oracle_num_threads.restype = i32
        _lib = L
    return _lib


def _cpu(t):
    if t is None:
        return None
    if t.device.type != "cpu":
        t = t.cpu()
    return t


def _rows_arg(rows):
    if rows is None:
        return None, 0, None
    arr = np.ascontiguousarray(np.asarray(rows, dtype=np.int64))
    return arr, arr.size, arr.ctypes.data


def attention_f16(q, k, v, causal=False, window=-1, rot_cos=None, rot_sin=None, scale=None,
                  rows: Optional[Sequence[int]] = None, rope_round: bool = False) -> torch.Tensor:
    """fp64 attention of fp16 q/k/v ([B,H,S,D], [B,Hkv,KS,D]) with the gate's semantics.

    Returns float64 [B,H,S,D], or [len(rows), D] when rows (flat (b*H+h)*S+q) is given.
    """
    q, k, v = _cpu(q), _cpu(k), _cpu(v)
    assert q.dtype == torch.float16 and k.dtype == torch.float16 and v.dtype == torch.float16
    for t in (q, k, v):
        assert t.stride(-1) == 1, "head_dim must be contiguous"
    B, H, S, D = q.shape
    Hkv, KS = k.shape[1], k.shape[2]
    if scale is None:
        scale = D ** -0.5
    has_rope = rot_cos is not None
    cos_p = sin_p = None
    if has_rope:
        rot_cos = _cpu(rot_cos).float().contiguous()
        rot_sin = _cpu(rot_sin).float().contiguous()
        cos_p, sin_p = rot_cos.data_ptr(), rot_sin.data_ptr()
    rows_arr, nrows, rows_p = _rows_arg(rows)
    out = torch.empty((nrows, D) if rows is not None else (B, H, S, D), dtype=torch.float64)
    qs, ks, vs = q.stride(), k.stride(), v.stride()
    rc = lib().oracle_attention_f16(q.data_ptr(), k.data_ptr(), v.data_ptr(), cos_p, sin_p,
                                    qs[0], qs[1], qs[2], ks[0], ks[1], ks[2], vs[0], vs[1], vs[2],
                                    B, H, Hkv, S, KS, D, float(scale), int(bool(causal)), int(has_rope),
                                    int(window), int(bool(rope_round)), rows_p, nrows, out.data_ptr())
    if rc != 0:
        raise ValueError(f"oracle_attention_f16 rejected its arguments (rc={rc})")
    return out


def attention_int8(qi, ki, vi, q_scale, k_scale, v_scale, causal=False, window=-1, scale=None,
                   rows: Optional[Sequence[int]] = None) -> torch.Tensor:
    """fp64 INT8 attention with the semantics of tests/hip_forward_int8qk_gate.hip:69-120.

    q_scale / k_scale: float, or float32 tensors (B,H,S) / (B,Hkv,KS) of per-token scales.
    """
    qi, ki, vi = _cpu(qi), _cpu(ki), _cpu(vi)
    for t in (qi, ki, vi):
        assert t.dtype == torch.int8 and t.stride(-1) == 1
    B, H, S, D = qi.shape
    Hkv, KS = ki.shape[1], ki.shape[2]
    if scale is None:
        scale = D ** -0.5
    q_vec = k_vec = None
    qsc, ksc = 1.0, 1.0
    if isinstance(q_scale, torch.Tensor):
        q_vec = _cpu(q_scale).float().contiguous()
    else:
        qsc = float(q_scale)
    if isinstance(k_scale, torch.Tensor):
        k_vec = _cpu(k_scale).float().contiguous()
    else:
        ksc = float(k_scale)
    rows_arr, nrows, rows_p = _rows_arg(rows)
    out = torch.empty((nrows, D) if rows is not None else (B, H, S, D), dtype=torch.float64)
    qs, ks, vs = qi.stride(), ki.stride(), vi.stride()
    rc = lib().oracle_attention_int8(qi.data_ptr(), ki.data_ptr(), vi.data_ptr(),
                                     qs[0], qs[1], qs[2], ks[0], ks[1], ks[2], vs[0], vs[1], vs[2],
                                     B, H, Hkv, S, KS, D, float(scale), qsc, ksc, float(v_scale),
                                     q_vec.data_ptr() if q_vec is not None else None,
                                     k_vec.data_ptr() if k_vec is not None else None,
                                     int(bool(causal)), int(window), rows_p, nrows, out.data_ptr())
    if rc != 0:
        raise ValueError(f"oracle_attention_int8 rejected its arguments (rc={rc})")
    return out


def lcg_uniform(seed: int, n: int, state=None):
    """Values of tests/hip_forward_gate.hip:35-37 frand(); returns (float32 array, new seed)."""
    s = ctypes.c_uint32(seed if state is None else state)
    out = np.empty(n, dtype=np.float32)
    lib().oracle_lcg_uniform(ctypes.byref(s), out.ctypes.data, n)
    return out, s.value


def lcg_gaussianish(seed: int, n: int, state=None):
    """Values of tests/hip_forward_int8qk_gate.hip:45-50; returns (float32 array, new seed)."""
    s = ctypes.c_uint32(seed if state is None else state)
    out = np.empty(n, dtype=np.float32)
    lib().oracle_lcg_gaussianish(ctypes.byref(s), out.ctypes.data, n)
    return out, s.value


def quantize(x: np.ndarray, scales: np.ndarray, group: int) -> np.ndarray:
    """tests/hip_forward_int8qk_gate.hip:61-65 with one scale per `group` consecutive values."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    scales = np.ascontiguousarray(scales, dtype=np.float32)
    out = np.empty(x.shape, dtype=np.int8)
    lib().oracle_quantize(x.ctypes.data, x.size, scales.ctypes.data, group, out.ctypes.data)
    return out


def key_range(q, S, KS, causal, window):
    lo, hi = ctypes.c_int64(), ctypes.c_int64()
    lib().oracle_key_range(q, S, KS, int(bool(causal)), int(window), ctypes.byref(lo), ctypes.byref(hi))
    return lo.value, hi.value


def num_threads() -> int:
    return int(lib().oracle_num_threads())
