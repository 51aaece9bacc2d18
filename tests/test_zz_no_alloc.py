"""rdna_attention_forward_noalloc: the FP16 entry point for callers that cannot
allocate device memory (a plugin whose host framework owns the allocator, a
process under a hard memory budget, a device without stream-ordered memory
pools).  Its RoPE workspace is a fixed 32 MiB array inside the library instead
of a cudaMallocAsync buffer.

Called through the C ABI and compared with rdna_attention_forward on the same
inputs, twice in a row with different inputs (the shared array keeps the
previous call's contents), at the tolerance the FP16 tests use (max-abs
<= 2e-3).  This file is named so pytest collects it last, and it builds all
of its own state, so it also runs alone in a fresh process.
"""
import ctypes
import os
import sys
from pathlib import Path

import pytest
import torch

ROOT = Path(__file__).resolve().parent.parent
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))

pytestmark = pytest.mark.gpu

_ARGS = ([ctypes.c_void_p] * 6 + [ctypes.c_int64] * 12 + [ctypes.c_uint32] * 6 + [ctypes.c_float]
         + [ctypes.c_int32] * 3 + [ctypes.c_void_p])


def _lib():
    path = os.environ.get("RDNATTENTION_LIB") or str(ROOT / "rdnattention_b200" / "lib" / "librdnattention.so")
    lib = ctypes.CDLL(path)
    for name in ("rdna_attention_forward", "rdna_attention_forward_noalloc"):
        f = getattr(lib, name)
        f.argtypes = _ARGS
        f.restype = ctypes.c_int32
    lib.rdna_get_error.restype = ctypes.c_char_p
    return lib


def _call(fn, q, k, v, o, cos, sin, causal, scale):
    B, H, S, D = q.shape
    Hkv, KS = k.shape[1], k.shape[2]
    return fn(q.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr(), cos.data_ptr(), sin.data_ptr(),
              *q.stride()[:3], *k.stride()[:3], *v.stride()[:3], *o.stride()[:3],
              B, H, Hkv, S, KS, D, scale, int(causal), 1, -1, torch.cuda.current_stream().cuda_stream)


def _tables(rows, D, theta):
    pos = torch.arange(rows, device="cuda").unsqueeze(1).float()
    ang = pos * (theta ** (-torch.arange(0, D, 2, device="cuda").float() / D))
    return ang.cos().contiguous(), ang.sin().contiguous()


@pytest.fixture(scope="module")
def lib():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return _lib()


def _pool_bytes():
    """(used, reserved) bytes of the current device's default stream-ordered memory pool,
    through the CUDA runtime (cudaMemPoolAttrUsedMemCurrent / ReservedMemCurrent)."""
    rt = ctypes.CDLL("libcudart.so.12")
    pool = ctypes.c_void_p()
    assert rt.cudaDeviceGetDefaultMemPool(ctypes.byref(pool), torch.cuda.current_device()) == 0
    used, reserved = ctypes.c_uint64(), ctypes.c_uint64()
    assert rt.cudaMemPoolGetAttribute(pool, 7, ctypes.byref(used)) == 0
    assert rt.cudaMemPoolGetAttribute(pool, 5, ctypes.byref(reserved)) == 0
    return used.value, reserved.value


def test_noalloc_matches_allocating_entry_point_twice(lib):
    shapes = [(1, 8, 2, 512, 512, 128, True, 500000.0), (2, 4, 4, 300, 700, 64, False, 10000.0),
              (1, 4, 2, 200, 300, 256, True, 10000.0)]  # head_dim 256: rotated Q in the array too
    for seed, (B, H, Hkv, S, KS, D, causal, theta) in enumerate(shapes):
        g = torch.Generator(device="cuda").manual_seed(100 + seed)
        q = torch.randn(B, H, S, D, generator=g, device="cuda", dtype=torch.float16)
        k = torch.randn(B, Hkv, KS, D, generator=g, device="cuda", dtype=torch.float16)
        v = torch.randn(B, Hkv, KS, D, generator=g, device="cuda", dtype=torch.float16)
        cos, sin = _tables(max(S, KS), D, theta)
        ref = torch.empty_like(q)
        out = torch.full_like(q, float("nan"))
        scale = D ** -0.5
        assert _call(lib.rdna_attention_forward, q, k, v, ref, cos, sin, causal, scale) == 0, lib.rdna_get_error()
        torch.cuda.synchronize()
        pool_before, torch_before = _pool_bytes(), torch.cuda.memory_allocated()
        assert _call(lib.rdna_attention_forward_noalloc, q, k, v, out, cos, sin, causal, scale) == 0, \
            lib.rdna_get_error()
        torch.cuda.synchronize()
        # nothing was taken from the stream-ordered pool or from torch's allocator
        assert _pool_bytes() == pool_before
        assert torch.cuda.memory_allocated() == torch_before
        assert torch.isfinite(out).all()
        assert (out.double() - ref.double()).abs().max().item() <= 2e-3


def test_noalloc_workspace_limit_is_exact(lib):
    """8 KV heads, head_dim 128, 16384 keys: exactly the 32 MiB of rotated K the array
    holds (head_dim <= 128 rotates Q inside the kernel) -- accepted and correct; one key
    more is rejected with -3."""
    B, H, Hkv, S, D = 1, 8, 8, 128, 128
    for KS, ok in ((16384, True), (16385, False)):
        g = torch.Generator(device="cuda").manual_seed(KS)
        q = torch.randn(B, H, S, D, generator=g, device="cuda", dtype=torch.float16)
        k = torch.randn(B, Hkv, KS, D, generator=g, device="cuda", dtype=torch.float16)
        v = torch.randn(B, Hkv, KS, D, generator=g, device="cuda", dtype=torch.float16)
        cos, sin = _tables(KS, D, 500000.0)
        out = torch.empty_like(q)
        rc = _call(lib.rdna_attention_forward_noalloc, q, k, v, out, cos, sin, False, D ** -0.5)
        if not ok:
            assert rc == -3 and "exceeds the fixed" in lib.rdna_get_error().decode()
            continue
        assert rc == 0, lib.rdna_get_error()
        ref = torch.empty_like(q)
        assert _call(lib.rdna_attention_forward, q, k, v, ref, cos, sin, False, D ** -0.5) == 0
        torch.cuda.synchronize()
        assert (out.double() - ref.double()).abs().max().item() <= 2e-3


def test_noalloc_rejects_workspace_beyond_limit(lib):
    # 8 heads, 128 query rows, 20480 keys, head_dim 128: 40 MiB of rotated K > 32 MiB
    B, H, Hkv, S, KS, D = 1, 8, 8, 128, 20480, 128
    q = torch.zeros(B, H, S, D, device="cuda", dtype=torch.float16)
    k = torch.zeros(B, Hkv, KS, D, device="cuda", dtype=torch.float16)
    cos, sin = _tables(KS, D, 10000.0)
    out = torch.empty_like(q)
    rc = _call(lib.rdna_attention_forward_noalloc, q, k, k, out, cos, sin, True, D ** -0.5)
    assert rc == -3
    msg = lib.rdna_get_error().decode()
    assert "exceeds the fixed" in msg and str(32 << 20) in msg, msg
