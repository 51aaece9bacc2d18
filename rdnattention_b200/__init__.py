"""rdnattention for B200 — FlashAttention-2 forward on sm_100a tensor cores.

Drop-in for the reference package ``rdnattention`` (rdnattention/__init__.py
of dmonkman/RDNAttention): same public names, argument meaning, validation
errors and C-ABI calls.  The kernels behind it are hand-written sm_100a CUDA
(TMA + tcgen05.mma + TMEM) in ``librdnattention.so``; there is no CPU or
library fallback — without the shared library every compute entry point
raises :class:`RDNAttentionError`.

    >>> import torch
    >>> from rdnattention_b200 import flash_attn
    >>> q = torch.randn(1, 8, 512, 64, dtype=torch.float16, device="cuda")
    >>> out = flash_attn(q, q, q, is_causal=True)
"""
import ctypes
import logging
import os
import platform
from pathlib import Path

logger = logging.getLogger(__name__)

__version__ = "0.1.0"

SUPPORTED_HEAD_DIMS = tuple(range(32, 513, 32))
SUPPORTED_HEAD_DIMS_INT8 = (64, 128)

_lib = None
_PKG = Path(__file__).resolve().parent


class RDNAttentionError(Exception):
    """Raised for any rdnattention library error."""


def _candidate_paths():
    """Search order of the reference loader (rdnattention/__init__.py:46-67):
    $RDNATTENTION_LIB, else <source tree>/build/ (a CMake build, which wins in a
    source checkout), else the package's own lib/ (python -m rdnattention_b200.build)."""
    name = "librdnattention.so"
    return [_PKG.parent / "build" / name, _PKG / "lib" / name]


def library_path() -> Path:
    """Where librdnattention.so is loaded from: $RDNATTENTION_LIB, else build/, else lib/."""
    if platform.system() != "Linux":
        raise RDNAttentionError(f"Unsupported platform: {platform.system()} (CUDA build is Linux-only)")
    override = os.environ.get("RDNATTENTION_LIB")
    if override:
        path = Path(override)
        if not path.exists():
            raise RDNAttentionError(f"RDNATTENTION_LIB points at a missing file: {path}")
        return path
    for path in _candidate_paths():
        if path.exists():
            return path
    raise RDNAttentionError(
        "Could not find librdnattention.so in " + ", ".join(str(p.parent) for p in _candidate_paths())
        + ". Build it first: python -m rdnattention_b200.build (or cmake -B build && cmake --build build)")


def _lib_handle():
    global _lib
    if _lib is None:
        lib = ctypes.CDLL(str(library_path()))
        i64, u32, i32, f32, vp = ctypes.c_int64, ctypes.c_uint32, ctypes.c_int32, ctypes.c_float, ctypes.c_void_p
        lib.rdna_has_device.argtypes = []
        lib.rdna_has_device.restype = i32
        lib.rdna_get_error.argtypes = []
        lib.rdna_get_error.restype = ctypes.c_char_p
        lib.rdna_attention_forward.argtypes = [vp] * 6 + [i64] * 12 + [u32] * 6 + [f32, i32, i32, i32, vp]
        lib.rdna_attention_forward.restype = i32
        lib.rdna_attention_forward_ws.argtypes = ([vp] * 6 + [i64] * 12 + [u32] * 6 + [f32, i32, i32, i32]
                                                  + [vp, ctypes.c_uint64, vp])
        lib.rdna_attention_forward_ws.restype = i32
        lib.rdna_attention_forward_workspace_size.argtypes = [u32] * 6 + [i32]
        lib.rdna_attention_forward_workspace_size.restype = ctypes.c_uint64
        lib.rdna_attention_forward_int8qk.argtypes = ([vp] * 4 + [i64] * 12 + [u32] * 6 + [f32] * 4 + [vp, vp]
                                                      + [i32, i32, vp])
        lib.rdna_attention_forward_int8qk.restype = i32
        lib.rdna_attention_forward_int8qk_vch.argtypes = ([vp] * 4 + [i64] * 12 + [u32] * 6 + [f32] * 4
                                                          + [vp, vp, vp] + [i32, i32, vp])
        lib.rdna_attention_forward_int8qk_vch.restype = i32
        lib.rdna_int8_quantize_qkv.argtypes = [vp] * 3 + [i64] * 9 + [u32] * 6 + [vp] * 7
        lib.rdna_int8_quantize_qkv.restype = i32
        lib.rdna_debug_int8qk_scores.argtypes = ([vp] * 4 + [i64] * 12 + [u32] * 6 + [f32] * 4 + [vp, vp]
                                                 + [i32, i32, vp, vp])
        lib.rdna_debug_int8qk_scores.restype = i32
        lib.rdna_debug_read_status.argtypes = [ctypes.POINTER(i32)]
        lib.rdna_debug_read_status.restype = i32
        lib.rdna_debug_set_wait_test.argtypes = [i32, ctypes.c_uint64]
        lib.rdna_debug_set_wait_test.restype = i32
        pp = ctypes.POINTER(vp)
        lib.rdna_attention_forward_ws_peers.argtypes = ([vp] * 6 + [i64] * 12 + [u32] * 6 + [f32, i32, i32, i32]
                                                        + [vp, ctypes.c_uint64, i32, pp, vp])
        lib.rdna_attention_forward_ws_peers.restype = i32
        lib.rdna_attention_forward_int8qk_vch_peers.argtypes = ([vp] * 4 + [i64] * 12 + [u32] * 6 + [f32] * 4
                                                                + [vp, vp, vp] + [i32, i32, i32, pp, vp])
        lib.rdna_attention_forward_int8qk_vch_peers.restype = i32
        lib.rdna_ipc_alloc.argtypes = [ctypes.c_uint64, pp, vp]
        lib.rdna_ipc_alloc.restype = i32
        lib.rdna_ipc_open.argtypes = [vp, pp]
        lib.rdna_ipc_open.restype = i32
        lib.rdna_ipc_close.argtypes = [vp]
        lib.rdna_ipc_close.restype = i32
        lib.rdna_ipc_free.argtypes = [vp]
        lib.rdna_ipc_free.restype = i32
        lib.rdna_peer_barrier.argtypes = [i32, i32, pp, vp, u32, vp]
        lib.rdna_peer_barrier.restype = i32
        lib.rdna_debug_set_kernel_events.argtypes = [vp, vp]
        lib.rdna_debug_set_kernel_events.restype = i32
        _lib = lib
    return _lib


def _last_error() -> str:
    return _lib_handle().rdna_get_error().decode(errors="replace")


def has_device() -> bool:
    """Whether a usable CUDA device is present."""
    return _lib_handle().rdna_has_device() == 1


def _validate_inputs(query, key, value, expected_dtype, require_contiguous=True) -> None:
    import torch

    if not all(isinstance(t, torch.Tensor) for t in (query, key, value)):
        raise TypeError("requires torch.Tensor inputs (GPU tensors already on this device)")
    for name, t in (("query", query), ("key", key), ("value", value)):
        if not t.is_cuda:
            raise ValueError(f"{name} must be on a CUDA device")
        if t.dtype != expected_dtype:
            raise ValueError(f"{name} must be {expected_dtype}, got {t.dtype}")
        if t.dim() != 4:
            raise ValueError(f"{name} must be 4D [batch, heads, seq, head_dim], got shape {tuple(t.shape)}")
        if require_contiguous and not t.is_contiguous():
            raise ValueError(f"{name} must be contiguous - call .contiguous() first")
        if not require_contiguous and t.stride(-1) != 1:
            raise ValueError(f"{name} must have a contiguous head_dim axis")
    if query.shape[0] != key.shape[0] or query.shape[0] != value.shape[0]:
        raise ValueError(f"Batch size must match: Q={tuple(query.shape)}, K={tuple(key.shape)}, V={tuple(value.shape)}")
    if key.shape[1] == 0 or query.shape[1] % key.shape[1] != 0:
        raise ValueError(f"Q heads ({query.shape[1]}) must be a multiple of K heads ({key.shape[1]})")
    if key.shape != value.shape:
        raise ValueError(f"key and value shapes must match: K={tuple(key.shape)}, V={tuple(value.shape)}")
    if query.shape[-1] != key.shape[-1]:
        raise ValueError(f"head_dim must match: Q={query.shape[-1]}, K={key.shape[-1]}")
    if not (query.device == key.device == value.device):
        raise ValueError("query, key and value must be on the same device")


def _check_head_dim(head_dim: int, who: str, allowed=SUPPORTED_HEAD_DIMS):
    if head_dim not in allowed:
        raise RDNAttentionError(f"{who}: head_dim {head_dim} not supported (allowed: {list(allowed)})")


def _rope_args(rot_cos, rot_sin, query, seq_len, key_seq_len, head_dim):
    """Validates the angle tables; returns (cos_ptr, sin_ptr, has_rope)."""
    import torch

    if rot_cos is None and rot_sin is None:
        return None, None, 0
    if rot_cos is None or rot_sin is None:
        raise ValueError("pass both rot_cos and rot_sin, or neither")
    rows = max(seq_len, key_seq_len)
    for name, t in (("rot_cos", rot_cos), ("rot_sin", rot_sin)):
        if not isinstance(t, torch.Tensor):
            raise TypeError(f"{name} must be a torch.Tensor")
        if t.device != query.device:
            raise ValueError(f"{name} must be on the same device as query")
        if t.dtype != torch.float32:
            raise ValueError(f"{name} must be float32, got {t.dtype}")
        if not t.is_contiguous():
            raise ValueError(f"{name} must be contiguous - call .contiguous() first")
        if t.dim() != 2:
            raise ValueError(f"{name} must be 2D [positions, head_dim // 2], got {tuple(t.shape)}")
        if t.shape[1] != head_dim // 2:
            raise ValueError(f"{name} must have head_dim // 2 = {head_dim // 2} columns, got {t.shape[1]}")
        if t.shape[0] < rows:
            raise ValueError(f"{name} needs at least max(seq_len, key_seq_len) = {rows} rows, got {t.shape[0]}")
    return rot_cos.data_ptr(), rot_sin.data_ptr(), 1


def _stream_handle(device):
    import torch

    return torch.cuda.current_stream(device).cuda_stream


def _on_device(device):
    """Makes `device` current around a library call: the C side reads the current
    device for its per-device state (SM count, kernel attributes, the no-alloc
    workspace address)."""
    import torch

    return torch.cuda.device(device)


MAX_PEER_OUTPUTS = 7
IPC_HANDLE_BYTES = 64


def _peer_array(peer_outputs):
    """(count, ctypes array) of peer output addresses, or (0, None)."""
    if not peer_outputs:
        return 0, None
    addrs = [int(a) for a in peer_outputs]
    if len(addrs) > MAX_PEER_OUTPUTS:
        raise ValueError(f"at most {MAX_PEER_OUTPUTS} peer outputs, got {len(addrs)}")
    return len(addrs), (ctypes.c_void_p * len(addrs))(*addrs)


def _ipc_alloc(nbytes: int):
    """Device memory on the current device that other processes can map:
    (address, 64-byte CUDA IPC handle)."""
    ptr = ctypes.c_void_p()
    handle = ctypes.create_string_buffer(IPC_HANDLE_BYTES)
    if _lib_handle().rdna_ipc_alloc(int(nbytes), ctypes.byref(ptr), handle) != 0:
        raise RDNAttentionError(_last_error())
    return ptr.value, handle.raw


def _ipc_open(handle: bytes) -> int:
    """Maps another process's _ipc_alloc memory (by its handle); returns its address here."""
    if len(handle) != IPC_HANDLE_BYTES:
        raise ValueError(f"an IPC handle has {IPC_HANDLE_BYTES} bytes, got {len(handle)}")
    ptr = ctypes.c_void_p()
    buf = ctypes.create_string_buffer(handle, IPC_HANDLE_BYTES)
    if _lib_handle().rdna_ipc_open(buf, ctypes.byref(ptr)) != 0:
        raise RDNAttentionError(_last_error())
    return ptr.value


def _ipc_close(ptr: int) -> None:
    if _lib_handle().rdna_ipc_close(ptr) != 0:
        raise RDNAttentionError(_last_error())


def _ipc_free(ptr: int) -> None:
    if _lib_handle().rdna_ipc_free(ptr) != 0:
        raise RDNAttentionError(_last_error())


def _peer_barrier(world: int, rank: int, peer_flags, my_flags: int, epoch: int, device) -> None:
    """Enqueues the cross-GPU barrier kernel (rdna_peer_barrier) on the current stream of `device`."""
    arr = (ctypes.c_void_p * len(peer_flags))(*[int(a) for a in peer_flags])
    with _on_device(device):
        rc = _lib_handle().rdna_peer_barrier(world, rank, arr, my_flags, epoch & 0xFFFFFFFF,
                                             _stream_handle(device))
    if rc != 0:
        raise RDNAttentionError(_last_error())


def _fp16_forward(query, key, value, is_causal, window_size, rot_cos, rot_sin, out, scale, require_contiguous,
                  peer_outputs=None):
    import torch

    _validate_inputs(query, key, value, torch.float16, require_contiguous)
    _check_head_dim(query.shape[-1], "flash_attn")
    if not has_device():
        raise RDNAttentionError("no usable CUDA device found")
    batch, heads, seq_len, head_dim = query.shape
    _, kv_heads, key_seq_len, _ = key.shape
    cos_p, sin_p, has_rope = _rope_args(rot_cos, rot_sin, query, seq_len, key_seq_len, head_dim)
    if out is None:
        out = torch.empty(query.shape, dtype=torch.float16, device=query.device)
    if scale is None:
        scale = head_dim ** -0.5
    qs, ks, vs, os_ = query.stride(), key.stride(), value.stride(), out.stride()
    lib = _lib_handle()
    # RoPE runs as a pre-pass into a workspace; take it from torch's caching allocator
    ws_bytes = lib.rdna_attention_forward_workspace_size(batch, heads, kv_heads, seq_len, key_seq_len, head_dim,
                                                         has_rope)
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device=query.device) if ws_bytes else None
    n_peers, peers = _peer_array(peer_outputs)
    args = (query.data_ptr(), key.data_ptr(), value.data_ptr(), out.data_ptr(), cos_p, sin_p,
            qs[0], qs[1], qs[2], ks[0], ks[1], ks[2], vs[0], vs[1], vs[2], os_[0], os_[1], os_[2],
            batch, heads, kv_heads, seq_len, key_seq_len, head_dim,
            float(scale), 1 if is_causal else 0, has_rope, int(window_size),
            ws.data_ptr() if ws is not None else None, ws_bytes)
    with _on_device(query.device):
        if n_peers:
            rc = lib.rdna_attention_forward_ws_peers(*args, n_peers, peers, _stream_handle(query.device))
        else:
            rc = lib.rdna_attention_forward_ws(*args, _stream_handle(query.device))
    if rc != 0:
        raise RDNAttentionError(f"flash_attn failed: {_last_error()}")
    return out


def flash_attn(query, key, value, is_causal: bool = False, window_size: int = -1, rot_cos=None, rot_sin=None):
    """FlashAttention-2 forward in fp16.  query/key/value: contiguous float16
    [batch, heads, seq, head_dim] on a CUDA device, head_dim in
    SUPPORTED_HEAD_DIMS; key/value may have fewer heads (GQA, exact divisor)
    and a different sequence length (cross-attention / decode; causal aligns
    to the end of the key sequence).  window_size > 0 limits each query to a
    band (one-sided when causal, +-window_size//2 otherwise).  rot_cos /
    rot_sin: float32 [max(seq_len, key_seq_len), head_dim // 2] angle tables
    applied in-kernel as interleaved-pair RoPE to Q and K.  Softmax scale is
    1/sqrt(head_dim).  Returns a new tensor shaped like query.

    Mirrors rdnattention/__init__.py:195-238 of the reference.
    """
    return _fp16_forward(query, key, value, is_causal, window_size, rot_cos, rot_sin, None, None, True)


def flash_attn_strided(query, key, value, is_causal: bool = False, window_size: int = -1, rot_cos=None,
                       rot_sin=None, out=None, scale=None, peer_outputs=None):
    """flash_attn over arbitrary batch/head/seq strides (head_dim contiguous),
    e.g. a KV cache stored [batch, seq, kv_heads, head_dim] and viewed with
    ``.transpose(1, 2)``.  Optional preallocated ``out`` (any strides) and
    softmax ``scale``.  Extension: the reference reaches this only through
    its raw C ABI (tests/rope.py:9-27, tests/benchmark.py:232-263).

    ``peer_outputs`` (multi-GPU extension): addresses of up to 7 other GPUs'
    counterparts of ``out`` (same strides, mapped into this process, e.g. by
    multigpu.SymmetricOutput); the kernels store every output tile there too,
    over NVLink.  They hold the result once this call's kernels have completed.
    """
    return _fp16_forward(query, key, value, is_causal, window_size, rot_cos, rot_sin, out, scale, False,
                         peer_outputs)


def flash_attn_int8qk(query, key, value, q_scale, k_scale, v_scale: float, is_causal: bool = False,
                      window_size: int = -1, *, out=None, peer_outputs=None):
    """INT8 attention, both GEMMs on the int8 tensor cores.  query/key/value:
    contiguous int8 [batch, heads, seq, head_dim], head_dim in
    SUPPORTED_HEAD_DIMS_INT8; output float16.  Symmetric dequant scales:
    q_scale / k_scale are floats or float32 per-token tensors shaped
    (batch, heads, seq_len) / (batch, kv_heads, key_seq_len); v_scale is a
    float.  Causal, window, GQA and cross-attention supported; no RoPE.

    Mirrors rdnattention/__init__.py:241-300 of the reference.  Extensions
    (keyword only): a preallocated float16 ``out`` (any strides), and
    ``peer_outputs`` as in flash_attn_strided (other GPUs' counterparts of
    ``out`` that the kernel also writes).
    """
    return _int8_forward(query, key, value, q_scale, k_scale, v_scale, is_causal, window_size, out, peer_outputs,
                         True)


def flash_attn_int8qk_strided(query, key, value, q_scale, k_scale, v_scale: float, is_causal: bool = False,
                              window_size: int = -1, out=None, peer_outputs=None):
    """flash_attn_int8qk over arbitrary batch/head/seq strides (head_dim
    contiguous), e.g. the views of one rank's units in a multi-GPU split;
    per-token scale tensors may be strided views too (they are made contiguous).
    Extension: the reference reaches strided INT8 only through its raw C ABI."""
    return _int8_forward(query, key, value, q_scale, k_scale, v_scale, is_causal, window_size, out, peer_outputs,
                         False)


def _int8_forward(query, key, value, q_scale, k_scale, v_scale, is_causal, window_size, out, peer_outputs,
                  require_contiguous):
    import torch

    _validate_inputs(query, key, value, torch.int8, require_contiguous)
    batch, heads, seq_len, head_dim = query.shape
    _, kv_heads, key_seq_len, _ = key.shape
    _check_head_dim(head_dim, "flash_attn_int8qk", allowed=SUPPORTED_HEAD_DIMS_INT8)
    if not has_device():
        raise RDNAttentionError("no usable CUDA device found")

    def scale_arg(x, name, want):
        if not isinstance(x, torch.Tensor):
            return float(x), None
        t = x.to(dtype=torch.float32, device=query.device).contiguous()
        if tuple(t.shape) != want:
            raise RDNAttentionError(f"flash_attn_int8qk: {name} tensor must be {want}, got {tuple(t.shape)}")
        return 1.0, t

    q_scalar, q_vec = scale_arg(q_scale, "q_scale", (batch, heads, seq_len))
    k_scalar, k_vec = scale_arg(k_scale, "k_scale", (batch, kv_heads, key_seq_len))
    if out is None:
        out = torch.empty(query.shape, dtype=torch.float16, device=query.device)
    elif out.dtype != torch.float16 or tuple(out.shape) != tuple(query.shape) or out.device != query.device:
        raise RDNAttentionError("flash_attn_int8qk: out must be float16, shaped like query, on query's device")
    qs, ks, vs, os_ = query.stride(), key.stride(), value.stride(), out.stride()
    n_peers, peers = _peer_array(peer_outputs)
    args = (query.data_ptr(), key.data_ptr(), value.data_ptr(), out.data_ptr(),
            qs[0], qs[1], qs[2], ks[0], ks[1], ks[2], vs[0], vs[1], vs[2], os_[0], os_[1], os_[2],
            batch, heads, kv_heads, seq_len, key_seq_len, head_dim,
            float(head_dim ** -0.5), q_scalar, k_scalar, float(v_scale),
            q_vec.data_ptr() if q_vec is not None else None, k_vec.data_ptr() if k_vec is not None else None)
    with _on_device(query.device):
        if n_peers:
            rc = _lib_handle().rdna_attention_forward_int8qk_vch_peers(
                *args, None, 1 if is_causal else 0, int(window_size), n_peers, peers, _stream_handle(query.device))
        else:
            rc = _lib_handle().rdna_attention_forward_int8qk(*args, 1 if is_causal else 0, int(window_size),
                                                             _stream_handle(query.device))
    if rc != 0:
        raise RDNAttentionError(f"flash_attn_int8qk failed: {_last_error()}")
    return out


def debug_int8qk_scores(query, key, value, q_scale, k_scale, v_scale: float, is_causal: bool = False,
                        window_size: int = -1):
    """flash_attn_int8qk that also returns the kernel's raw int32 Q K^T:
    (out, scores), scores int32 [batch, heads, seq_len, key_seq_len] with the
    entries of key blocks the masks skip left at INT32_MIN.  Debug extension
    (no counterpart in the reference), for checking the integer GEMM bit for bit."""
    import torch

    _validate_inputs(query, key, value, torch.int8)
    batch, heads, seq_len, head_dim = query.shape
    _, kv_heads, key_seq_len, _ = key.shape
    _check_head_dim(head_dim, "debug_int8qk_scores", allowed=SUPPORTED_HEAD_DIMS_INT8)
    if not has_device():
        raise RDNAttentionError("no usable CUDA device found")

    def scale_arg(x, want):
        if not isinstance(x, torch.Tensor):
            return float(x), None
        t = x.to(dtype=torch.float32, device=query.device).contiguous()
        if tuple(t.shape) != want:
            raise RDNAttentionError(f"debug_int8qk_scores: scale tensor must be {want}, got {tuple(t.shape)}")
        return 1.0, t

    q_scalar, q_vec = scale_arg(q_scale, (batch, heads, seq_len))
    k_scalar, k_vec = scale_arg(k_scale, (batch, kv_heads, key_seq_len))
    out = torch.empty(query.shape, dtype=torch.float16, device=query.device)
    scores = torch.full((batch, heads, seq_len, key_seq_len), -2 ** 31, dtype=torch.int32, device=query.device)
    qs, ks, vs, os_ = query.stride(), key.stride(), value.stride(), out.stride()
    with _on_device(query.device):
        rc = _lib_handle().rdna_debug_int8qk_scores(
            query.data_ptr(), key.data_ptr(), value.data_ptr(), out.data_ptr(),
            qs[0], qs[1], qs[2], ks[0], ks[1], ks[2], vs[0], vs[1], vs[2], os_[0], os_[1], os_[2],
            batch, heads, kv_heads, seq_len, key_seq_len, head_dim,
            float(head_dim ** -0.5), q_scalar, k_scalar, float(v_scale),
            q_vec.data_ptr() if q_vec is not None else None, k_vec.data_ptr() if k_vec is not None else None,
            1 if is_causal else 0, int(window_size), scores.data_ptr(), _stream_handle(query.device))
    if rc != 0:
        raise RDNAttentionError(f"debug_int8qk_scores failed: {_last_error()}")
    return out, scores


def _symmetric_int8(x, scale):
    import torch

    return torch.clamp(torch.round(x / scale), -127, 127).to(torch.int8)


def quantize_int8_perchannel_v(query, key, value):
    """Quantise fp Q/K/V for flash_attn_int8qk with a per-channel V scale.
    Returns (qi, ki, vi, q_scale, k_scale, v_scale, v_channel): Q and K get one
    scale each (absmax/127), V one scale per (batch, head, head_dim column)
    (absmax over the sequence / 127, 0 -> 1.0) returned as v_channel
    (batch, heads, head_dim); attention is linear in V, so multiplying the
    kernel output by v_channel undoes it exactly and v_scale is 1.0.

    Same results as rdnattention/__init__.py:303-324 of the reference.
    """
    import torch

    def tensor_scale(x):
        s = x.abs().max().item() / 127.0
        return s if s != 0.0 else 1.0

    qf, kf, vf = query.float(), key.float(), value.float()
    q_scale, k_scale = tensor_scale(qf), tensor_scale(kf)
    v_channel = vf.abs().amax(dim=-2, keepdim=True) / 127.0
    v_channel = torch.where(v_channel == 0, torch.ones_like(v_channel), v_channel)
    return (_symmetric_int8(qf, q_scale), _symmetric_int8(kf, k_scale), _symmetric_int8(vf, v_channel),
            q_scale, k_scale, 1.0, v_channel.squeeze(-2))


def quantize_int8_qk_pertoken(query, key):
    """Quantise Q and K with one scale per (batch, head, row) = absmax/127
    (0 -> 1.0).  Returns (qi, ki, q_scale, k_scale), the scales float32
    (batch, heads, seq) / (batch, kv_heads, key_seq), ready for
    flash_attn_int8qk.  Same results as rdnattention/__init__.py:327-343.
    """
    import torch

    def per_row(x):
        x = x.float()
        s = x.abs().amax(dim=-1, keepdim=True) / 127.0
        s = torch.where(s == 0, torch.ones_like(s), s)
        return _symmetric_int8(x, s), s.squeeze(-1).contiguous()

    qi, q_scale = per_row(query)
    ki, k_scale = per_row(key)
    return qi, ki, q_scale, k_scale


def quantize_int8_qkv(query, key, value):
    """Device-side quantisation (one kernel) of fp16 Q/K/V for the INT8 path:
    returns (qi, ki, vi, q_scale, k_scale, v_channel) — int8 contiguous
    tensors, per-token float32 Q/K scales (batch, heads, seq) / (batch,
    kv_heads, key_seq) and the per-channel V scale (batch, kv_heads,
    head_dim).  Bit-identical to quantize_int8_qk_pertoken (qi, ki, scales)
    and quantize_int8_perchannel_v (vi, v_channel).  head_dim 64 or 128;
    query/key/value may be strided (head_dim contiguous).  Extension: the
    reference does this with torch ops on the host side.
    """
    import torch

    _validate_inputs(query, key, value, torch.float16, require_contiguous=False)
    batch, heads, seq_len, head_dim = query.shape
    _, kv_heads, key_seq_len, _ = key.shape
    _check_head_dim(head_dim, "quantize_int8_qkv", allowed=SUPPORTED_HEAD_DIMS_INT8)
    dev = query.device
    qi = torch.empty(query.shape, dtype=torch.int8, device=dev)
    ki = torch.empty(key.shape, dtype=torch.int8, device=dev)
    vi = torch.empty(value.shape, dtype=torch.int8, device=dev)
    q_scale = torch.empty(batch, heads, seq_len, dtype=torch.float32, device=dev)
    k_scale = torch.empty(batch, kv_heads, key_seq_len, dtype=torch.float32, device=dev)
    v_channel = torch.empty(batch, kv_heads, head_dim, dtype=torch.float32, device=dev)
    qs, ks, vs = query.stride(), key.stride(), value.stride()
    with _on_device(dev):
        rc = _lib_handle().rdna_int8_quantize_qkv(
            query.data_ptr(), key.data_ptr(), value.data_ptr(), qs[0], qs[1], qs[2], ks[0], ks[1], ks[2],
            vs[0], vs[1], vs[2], batch, heads, kv_heads, seq_len, key_seq_len, head_dim,
            qi.data_ptr(), ki.data_ptr(), vi.data_ptr(), q_scale.data_ptr(), k_scale.data_ptr(),
            v_channel.data_ptr(), _stream_handle(dev))
    if rc != 0:
        raise RDNAttentionError(f"quantize_int8_qkv failed: {_last_error()}")
    return qi, ki, vi, q_scale, k_scale, v_channel


def flash_attn_int8qk_quantized(query, key, value, is_causal: bool = False, window_size: int = -1):
    """INT8 attention from fp16/fp32 Q/K/V — the recommended INT8 entry point:
    per-token Q/K scales in-kernel and an exact per-channel V rescale of the
    output.  Same contract as rdnattention/__init__.py:346-357.

    fp16 inputs with head_dim 64/128 take the device path: one quantisation
    kernel, then the INT8 kernel with the per-channel V scale applied in its
    epilogue before the single fp16 rounding (the reference rescales the
    fp16 output afterwards, a second rounding).  Other dtypes quantise with
    the torch helpers first (exactly the reference's scales).
    """
    import torch

    if (isinstance(query, torch.Tensor) and query.dtype == torch.float16 and query.is_cuda
            and query.dim() == 4 and query.shape[-1] in SUPPORTED_HEAD_DIMS_INT8):
        qi, ki, vi, q_scale, k_scale, v_channel = quantize_int8_qkv(query, key, value)
        v_scale = 1.0
    else:
        _, _, vi, _, _, v_scale, v_channel = quantize_int8_perchannel_v(query, key, value)
        qi, ki, q_scale, k_scale = quantize_int8_qk_pertoken(query, key)
        qi, ki, vi = qi.contiguous(), ki.contiguous(), vi.contiguous()
        v_channel = v_channel.contiguous()
    _validate_inputs(qi, ki, vi, torch.int8)
    batch, heads, seq_len, head_dim = qi.shape
    _, kv_heads, key_seq_len, _ = ki.shape
    _check_head_dim(head_dim, "flash_attn_int8qk", allowed=SUPPORTED_HEAD_DIMS_INT8)
    out = torch.empty(qi.shape, dtype=torch.float16, device=qi.device)
    qs, ks, vs, os_ = qi.stride(), ki.stride(), vi.stride(), out.stride()
    with _on_device(qi.device):
        rc = _lib_handle().rdna_attention_forward_int8qk_vch(
            qi.data_ptr(), ki.data_ptr(), vi.data_ptr(), out.data_ptr(),
            qs[0], qs[1], qs[2], ks[0], ks[1], ks[2], vs[0], vs[1], vs[2], os_[0], os_[1], os_[2],
            batch, heads, kv_heads, seq_len, key_seq_len, head_dim,
            float(head_dim ** -0.5), 1.0, 1.0, float(v_scale), q_scale.data_ptr(), k_scale.data_ptr(),
            v_channel.data_ptr(), 1 if is_causal else 0, int(window_size), _stream_handle(qi.device))
    if rc != 0:
        raise RDNAttentionError(f"flash_attn_int8qk failed: {_last_error()}")
    return out


def debug_time_kernel(call, repeats: int = 10) -> float:
    """Average device time (ms) of the attention kernel that `call()` launches
    (through any of this library's forward entry points, on the current thread),
    timed by CUDA events the library records right around that kernel's launch
    (rdna_debug_set_kernel_events), so a RoPE pre-pass in the same call is not
    counted.  Debug extension; synchronises the device."""
    import torch

    lib = _lib_handle()
    total = 0.0
    for _ in range(repeats):
        start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record()  # creates the CUDA events; the library re-records them
        stop.record()
        lib.rdna_debug_set_kernel_events(start.cuda_event, stop.cuda_event)
        try:
            call()
        finally:
            lib.rdna_debug_set_kernel_events(None, None)
        stop.synchronize()
        total += start.elapsed_time(stop)
    return total / repeats


def debug_read_status():
    """(first error code, count) recorded by expired in-kernel waits on the
    current device, then cleared.  Synchronises the device."""
    out = (ctypes.c_int32 * 2)()
    if _lib_handle().rdna_debug_read_status(out) != 0:
        raise RDNAttentionError(f"debug_read_status failed: {_last_error()}")
    return int(out[0]), int(out[1])


__all__ = ["flash_attn", "flash_attn_int8qk", "flash_attn_int8qk_quantized", "quantize_int8_perchannel_v",
           "quantize_int8_qk_pertoken", "quantize_int8_qkv", "has_device", "RDNAttentionError", "SUPPORTED_HEAD_DIMS",
           "SUPPORTED_HEAD_DIMS_INT8", "__version__"]
