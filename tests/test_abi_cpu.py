"""C-ABI and host-logic checks that need no GPU: the library loads, exports
every symbol include/rdnattention.h declares, and rejects bad arguments with
the reference's return codes and messages (src/c_api.cpp:83-87, 151-154)
before touching a device."""
import ctypes
import re
from pathlib import Path

import pytest
import torch

import rdnattention_b200 as R

ROOT = Path(__file__).resolve().parent.parent


def _declared_symbols():
    text = (ROOT / "include" / "rdnattention.h").read_text()
    return re.findall(r"RDNA_API\s+[\w\s\*]+?\b(rdna_\w+)\s*\(", text)


def test_library_exports_every_declared_symbol():
    lib = R._lib_handle()
    names = _declared_symbols()
    assert {"rdna_has_device", "rdna_get_error", "rdna_attention_forward",
            "rdna_attention_forward_int8qk"} <= set(names)
    for n in names:
        assert hasattr(lib, n), n


def test_reference_ctypes_signature_binds():
    """The reference wrapper's own argtypes (rdnattention/__init__.py:102-127) bind our symbols."""
    lib = ctypes.CDLL(str(R.library_path()))
    f = lib.rdna_attention_forward
    f.argtypes = ([ctypes.c_void_p] * 6 + [ctypes.c_int64] * 12 + [ctypes.c_uint32] * 6 + [ctypes.c_float]
                  + [ctypes.c_int32] * 3 + [ctypes.c_void_p])
    f.restype = ctypes.c_int32
    g = lib.rdna_attention_forward_int8qk
    g.argtypes = ([ctypes.c_void_p] * 4 + [ctypes.c_int64] * 12 + [ctypes.c_uint32] * 6 + [ctypes.c_float] * 4
                  + [ctypes.c_void_p] * 2 + [ctypes.c_int32] * 2 + [ctypes.c_void_p])
    g.restype = ctypes.c_int32
    assert f(None, None, None, None, None, None, *([0] * 12), 1, 1, 1, 1, 1, 64, 0.125, 0, 0, -1, None) == -3


def _fwd(**kw):
    args = dict(q=16, k=16, v=16, o=16, cos=None, sin=None, qs=(64 * 8 * 64, 8 * 64, 64), ks=(64 * 8 * 64, 8 * 64, 64),
                vs=(64 * 8 * 64, 8 * 64, 64), os=(64 * 8 * 64, 8 * 64, 64), B=1, H=8, Hkv=8, S=64, KS=64, D=64,
                scale=0.125, causal=0, rope=0, window=-1)
    args.update(kw)
    lib = R._lib_handle()
    rc = lib.rdna_attention_forward(args["q"], args["k"], args["v"], args["o"], args["cos"], args["sin"],
                                    *args["qs"], *args["ks"], *args["vs"], *args["os"], args["B"], args["H"],
                                    args["Hkv"], args["S"], args["KS"], args["D"], args["scale"], args["causal"],
                                    args["rope"], args["window"], None)
    return rc, lib.rdna_get_error().decode()


@pytest.mark.parametrize("kw,needle", [
    (dict(q=None), "null tensor pointer"),
    (dict(D=48), "unsupported head_dim"),
    (dict(D=544), "unsupported head_dim"),
    (dict(Hkv=0), "positive multiple of numKvHeads"),
    (dict(Hkv=3), "positive multiple of numKvHeads"),
    (dict(S=0), "empty problem"),
    (dict(B=0), "empty problem"),
    (dict(qs=(64 * 8 * 64, 8 * 64, 2 ** 33)), "exceeds int32 range"),
    (dict(q=18), "16-byte aligned"),
    (dict(ks=(64 * 8 * 64, 8 * 64, 68)), "multiples of 16 bytes"),
    (dict(vs=(64 * 8 * 64, -64 * 64, 64)), "strides must be positive"),
    (dict(qs=(64 * 8 * 64, 0, 64)), "strides must be positive"),
    (dict(os=(64 * 8 * 64, 0, 64)), "output strides must be positive"),
    (dict(rope=1), "rot_cos/rot_sin is null"),
    (dict(rope=1, cos=20, sin=32), "16-byte aligned"),
])
def test_fp16_argument_errors(kw, needle):
    rc, msg = _fwd(**kw)
    assert rc == -3
    assert msg.startswith("Attention (fp16) failed: ")
    assert needle in msg, msg


def test_int8_argument_errors():
    lib = R._lib_handle()
    st = (64 * 8 * 64, 8 * 64, 64)
    rc = lib.rdna_attention_forward_int8qk(16, 16, 16, 16, *st, *st, *st, *st, 1, 8, 8, 64, 64, 96, 0.125, 1.0, 1.0,
                                           1.0, None, None, 0, -1, None)
    assert rc == -3
    assert "only 64 and 128" in lib.rdna_get_error().decode()
    rc = lib.rdna_attention_forward_int8qk(16, 16, 16, 16, *st, *st, *st, *st, 1, 8, 3, 64, 64, 64, 0.125, 1.0, 1.0,
                                           1.0, None, None, 0, -1, None)
    assert rc == -3
    assert lib.rdna_get_error().decode() == ("Attention (int8qk) failed: numHeads must be a positive multiple "
                                             "of numKvHeads")


def test_debug_scores_requires_buffer():
    lib = R._lib_handle()
    st = (64 * 8 * 64, 8 * 64, 64)
    rc = lib.rdna_debug_int8qk_scores(16, 16, 16, 16, *st, *st, *st, *st, 1, 8, 8, 64, 64, 64, 0.125, 1.0, 1.0,
                                      1.0, None, None, 0, -1, None, None)
    assert rc == -3
    assert lib.rdna_get_error().decode() == ("Attention (int8qk) failed: scores must be a 4-byte aligned "
                                             "int32 buffer")


def test_error_is_sticky_across_success_and_thread_local():
    rc, msg = _fwd(D=48)
    assert rc == -3
    import threading
    seen = {}

    def other():
        seen["msg"] = R._lib_handle().rdna_get_error().decode()

    t = threading.Thread(target=other)
    t.start()
    t.join()
    assert seen["msg"] == ""  # thread-local
    assert R._lib_handle().rdna_get_error().decode() == msg


def test_has_device_false_without_gpu():
    if torch.cuda.is_available():
        pytest.skip("GPU present")
    assert R.has_device() is False


def test_python_validation_errors():
    q = torch.zeros(1, 2, 8, 64, dtype=torch.float16)
    with pytest.raises(TypeError):
        R.flash_attn(q.numpy(), q, q)
    with pytest.raises(ValueError, match="CUDA device"):
        R.flash_attn(q, q, q)
    with pytest.raises(ValueError):
        R.flash_attn_int8qk(q, q, q, 1.0, 1.0, 1.0)


def test_quant_helpers_match_reference_bit_exactly():
    from golden_io import cases

    for m, a in cases("quant"):
        qi, ki, qs, ks = R.quantize_int8_qk_pertoken(a["q"], a["k"])
        assert torch.equal(qi, a["qi"]) and torch.equal(ki, a["ki"])
        assert torch.equal(qs, a["q_scale"]) and torch.equal(ks, a["k_scale"])
        pqi, pki, pvi, pqs, pks, pvs, vch = R.quantize_int8_perchannel_v(a["q"], a["k"], a["v"])
        assert torch.equal(pqi, a["pqi"]) and torch.equal(pki, a["pki"]) and torch.equal(pvi, a["pvi"])
        assert pqs == m["pq_scale"] and pks == m["pk_scale"] and pvs == m["pv_scale"]
        assert torch.equal(vch, a["v_channel"])


def test_drop_in_import_name():
    import rdnattention

    assert rdnattention.flash_attn is R.flash_attn
    assert rdnattention.SUPPORTED_HEAD_DIMS == tuple(range(32, 513, 32))
    assert rdnattention.SUPPORTED_HEAD_DIMS_INT8 == (64, 128)


def test_workspace_size_is_the_rotated_k_and_wide_q():
    """With RoPE the workspace holds what the pre-pass writes: the rotated K
    (B*Hkv*KS*D*2 bytes) and, for head_dim > 128 only, the rotated Q
    (B*H*S*D*2; the head_dim <= 128 kernels rotate Q in shared memory), each
    rounded up to 256 bytes; none without RoPE."""
    lib = R._lib_handle()
    ws = lib.rdna_attention_forward_workspace_size
    assert ws(4, 32, 8, 4096, 4096, 128, 1) == 4 * 8 * 4096 * 128 * 2
    assert ws(1, 3, 1, 5, 7, 32, 1) == 512  # 448 bytes of K rounded up to a multiple of 256
    assert ws(1, 4, 2, 100, 100, 256, 1) == 4 * 100 * 256 * 2 + 2 * 100 * 256 * 2
    assert ws(1, 3, 1, 5, 7, 160, 1) == 4864 + 2304  # 4800 (Q) and 2240 (K) bytes, each rounded up
    assert ws(4, 32, 8, 4096, 4096, 128, 0) == 0
    # decode-shaped problems (seq_len * group <= 64, head_dim 64/128) rotate in place: no workspace
    assert ws(64, 64, 8, 1, 32768, 128, 1) == 0
    assert ws(64, 64, 8, 8, 32768, 128, 1) == 0  # 64 rows per KV head: four row groups
    assert ws(64, 64, 8, 9, 32768, 128, 1) > 0   # 72 rows per KV head: prefill path


def test_int8_quantize_argument_errors():
    lib = R._lib_handle()
    f = lib.rdna_int8_quantize_qkv
    ok_strides = (8 * 64 * 64, 64 * 64, 64) * 3
    rc = f(None, 16, 16, *ok_strides, 1, 8, 8, 64, 64, 64, 16, 16, 16, 16, 16, 16, None)
    assert rc == -3 and "null tensor pointer" in lib.rdna_get_error().decode()
    rc = f(16, 16, 16, *ok_strides, 1, 8, 8, 64, 64, 96, 16, 16, 16, 16, 16, 16, None)
    assert rc == -3 and "unsupported head_dim" in lib.rdna_get_error().decode()
    rc = f(16, 16, 16, *ok_strides, 1, 8, 3, 64, 64, 64, 16, 16, 16, 16, 16, 16, None)
    assert rc == -3 and "multiple of numKvHeads" in lib.rdna_get_error().decode()
