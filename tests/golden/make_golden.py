"""Generates the golden fixtures in tests/golden/*.npz from the REFERENCE's own
oracle code.  Run in a container where the reference checkout is present:

    python tests/golden/make_golden.py [REFERENCE_ROOT]   (else $RDNA_REFERENCE_ROOT, else ../reference)

Sources of truth, all executed unmodified from the reference checkout:

* dense_fp32.npz   tests/accuracy.py:39-47 dense_attention_reference (fp32 inputs)
* head_dim.npz     tests/head_dim.py:23-44 reference (fp64; causal, both window forms, GQA,
                   cross-attention, decode), variants of tests/head_dim.py:10-20 at reduced sizes
* rope.npz         tests/rope.py:29-58 rope()/reference() (fp64), lifted with ast because
                   rope.py runs its benchmark at import; cases of tests/rope.py:66-73 at
                   reduced sizes, table recipe of tests/rope.py:78-82
* gate_f16.npz     tests/hip_forward_gate.hip:52-129 refAttention/applyRope via
                   oracle/_ref/libgate_ref.so (oracle/build_ref.py), LCG seed 12345 inputs and
                   the gate's theta=10000 table (tests/hip_forward_gate.hip:140-162)
* gate_int8.npz    tests/hip_forward_int8qk_gate.hip:61-120 quantize/refAttention via the same
                   library, LCG seed 424242 gaussian-ish inputs, per-tensor and per-token scales
* quant.npz        rdnattention/__init__.py:303-343 quantize_int8_perchannel_v /
                   quantize_int8_qk_pertoken (the reference package itself)

The fixtures are small (a few hundred KB in total) and committed; the GPU
box, which has no reference checkout, checks against them.
"""
import ast
import ctypes
import importlib.util
import json
import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
REPO = HERE.parent.parent
sys.path.insert(0, str(REPO))

from oracle import build_ref  # noqa: E402
from oracle import c_oracle  # noqa: E402  (LCG generators only)


def _load_module(name, path):
    spec = importlib.util.spec_from_file_location(name, path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def _rope_functions(path: Path):
    """rope.py executes at import; compile only its rope() and reference() definitions."""
    tree = ast.parse(path.read_text())
    keep = [n for n in tree.body if isinstance(n, ast.FunctionDef) and n.name in ("rope", "reference")]
    mod = ast.Module(body=keep, type_ignores=[])
    ns = {"torch": torch}
    exec(compile(mod, str(path), "exec"), ns)
    return ns["rope"], ns["reference"]


class Store:
    def __init__(self):
        self.arrays = {}
        self.meta = []

    def add(self, name, meta, **arrays):
        self.meta.append(dict(name=name, **meta))
        for k, v in arrays.items():
            if isinstance(v, torch.Tensor):
                v = v.detach().cpu().numpy()
            self.arrays[f"{name}__{k}"] = v

    def save(self, path):
        np.savez_compressed(path, meta=np.array(json.dumps(self.meta)), **self.arrays)
        print(f"wrote {path} ({path.stat().st_size / 1024:.0f} KB, {len(self.meta)} cases)")


def fp16_randn(gen, *shape):
    return torch.randn(*shape, generator=gen, dtype=torch.float32).to(torch.float16)


def make_dense_fp32(ref_root):
    acc = _load_module("ref_accuracy", ref_root / "tests" / "accuracy.py")
    st = Store()
    gen = torch.Generator().manual_seed(0)
    for (B, H, S, KS, D) in [(1, 2, 64, 64, 64), (2, 3, 40, 40, 32), (1, 2, 17, 17, 128), (1, 2, 24, 40, 64),
                             (1, 1, 33, 33, 256)]:
        q, k, v = fp16_randn(gen, B, H, S, D), fp16_randn(gen, B, H, KS, D), fp16_randn(gen, B, H, KS, D)
        out = acc.dense_attention_reference(q.float(), k.float(), v.float())
        st.add(f"dense_B{B}H{H}S{S}K{KS}D{D}", dict(B=B, H=H, Hkv=H, S=S, KS=KS, D=D, causal=False, window=-1),
               q=q, k=k, v=v, out=out.float())
    st.save(HERE / "dense_fp32.npz")


def make_head_dim(ref_root):
    hd = _load_module("ref_head_dim", ref_root / "tests" / "head_dim.py")
    st = Store()
    gen = torch.Generator().manual_seed(1234)
    # (name, kv divisor, S, KS, causal, window): tests/head_dim.py:10-20 scaled to S~40 so the
    # windows still cut the band.
    small = [("dense", 1, 30, 30, False, -1), ("causal", 1, 30, 30, True, -1), ("gqa", 4, 30, 30, False, -1),
             ("gqa_causal", 4, 30, 30, True, -1), ("window", 1, 30, 30, False, 12),
             ("causal_window", 1, 30, 30, True, 8), ("cross", 1, 18, 30, False, -1),
             ("decode", 1, 1, 30, False, -1), ("aligned", 1, 32, 32, True, -1),
             ("causal_q_longer", 1, 30, 18, True, -1)]
    for D in (32, 64, 96, 128):
        for name, kvdiv, S, KS, causal, window in small:
            H = 4 if kvdiv > 1 else 2
            Hkv = max(1, H // kvdiv)
            q, k, v = fp16_randn(gen, 1, H, S, D), fp16_randn(gen, 1, Hkv, KS, D), fp16_randn(gen, 1, Hkv, KS, D)
            out = hd.reference(q, k, v, causal, window)
            st.add(f"d{D}_{name}", dict(B=1, H=H, Hkv=Hkv, S=S, KS=KS, D=D, causal=causal, window=window),
                   q=q, k=k, v=v, out=out.float())
    for D in (160, 256, 512):
        for name, kvdiv, S, KS, causal, window in [("dense", 1, 12, 12, False, -1), ("causal", 1, 12, 12, True, -1),
                                                   ("window", 2, 12, 12, False, 6)]:
            H = 2
            Hkv = max(1, H // kvdiv)
            q, k, v = fp16_randn(gen, 1, H, S, D), fp16_randn(gen, 1, Hkv, KS, D), fp16_randn(gen, 1, Hkv, KS, D)
            out = hd.reference(q, k, v, causal, window)
            st.add(f"d{D}_{name}", dict(B=1, H=H, Hkv=Hkv, S=S, KS=KS, D=D, causal=causal, window=window),
                   q=q, k=k, v=v, out=out.float())
    st.save(HERE / "head_dim.npz")


def rope_tables(rows, D, theta=10000.0):
    """tests/rope.py:78-82 recipe on CPU: ang = pos * theta^(-arange(0, D, 2)/D)."""
    pos = torch.arange(rows).unsqueeze(1).float()
    inv = theta ** (-torch.arange(0, D, 2).float() / D)
    ang = pos * inv
    return ang.cos().contiguous(), ang.sin().contiguous()


def make_rope(ref_root):
    rope, reference = _rope_functions(ref_root / "tests" / "rope.py")
    st = Store()
    cases = [("mha_d64", 1, 2, 2, 48, 48, 64, False), ("mha_d128", 1, 2, 2, 40, 40, 128, False),
             ("causal_d64", 1, 2, 2, 48, 48, 64, True), ("causal_d128", 1, 2, 2, 40, 40, 128, True),
             ("gqa_d64", 1, 4, 1, 32, 32, 64, False), ("cross_d64", 1, 2, 2, 16, 48, 64, False),
             ("tail_d64", 1, 2, 2, 37, 37, 64, False)]
    for name, B, H, KH, S, KS, D, causal in cases:
        torch.manual_seed(7)
        q = torch.randn(B, H, S, D).to(torch.float16)
        k = torch.randn(B, KH, KS, D).to(torch.float16)
        v = torch.randn(B, KH, KS, D).to(torch.float16)
        cos, sin = rope_tables(max(S, KS), D)
        out = reference(q, k, v, cos, sin, causal)
        st.add(name, dict(B=B, H=H, Hkv=KH, S=S, KS=KS, D=D, causal=causal, window=-1),
               q=q, k=k, v=v, cos=cos, sin=sin, out=out.float())
    st.save(HERE / "rope.npz")


def _gate_lib():
    L = ctypes.CDLL(str(build_ref.build()))
    vp, i32, f32 = ctypes.c_void_p, ctypes.c_int, ctypes.c_float
    L.gate_f16_ref.argtypes = [vp] * 5 + [i32] * 6 + [f32, i32, i32, vp]
    L.gate_int8_ref.argtypes = [vp] * 3 + [i32] * 6 + [f32, i32, i32, vp]
    L.gate_int8_quantize.argtypes = [f32, f32]
    L.gate_int8_quantize.restype = ctypes.c_int8
    return L


def gate_rope_tables(KS, D):
    """tests/hip_forward_gate.hip:151-162: theta = s / 10000^(2p/D) in float, [KS, D/2]."""
    half = D // 2
    s = np.arange(KS, dtype=np.float32)[:, None]
    p = np.arange(half, dtype=np.float32)[None, :]
    theta = s / np.power(np.float32(10000.0), (2.0 * p / np.float32(D)).astype(np.float32))
    theta = theta.astype(np.float32)
    return np.cos(theta).astype(np.float32), np.sin(theta).astype(np.float32)


def make_gate_f16():
    L = _gate_lib()
    st = Store()
    # Feature mix of tests/hip_forward_gate.hip:259-316 at reduced sizes.
    cases = [("d64_dense_tail", 2, 2, 2, 40, 40, 64, False, 0, False),
             ("d64_causal", 1, 2, 2, 37, 37, 64, True, 0, False),
             ("d64_gqa_ratio3_pad", 1, 6, 2, 33, 33, 64, True, 0, False),
             ("d64_gqa_ratio5_pad_rope_window", 1, 10, 2, 29, 29, 64, True, 8, True),
             ("d64_window", 1, 2, 2, 40, 40, 64, False, 12, False),
             ("d64_causal_window", 1, 2, 2, 40, 40, 64, True, 6, False),
             ("d64_kv_longer", 1, 2, 2, 16, 48, 64, False, 0, False),
             ("d64_decode_1tok", 1, 8, 2, 1, 48, 64, False, 0, False),
             ("d128_rope_gqa_causal", 1, 4, 2, 31, 31, 128, True, 0, True),
             ("d32_dense", 1, 2, 2, 24, 24, 32, False, 0, False),
             ("d96_dense", 1, 2, 2, 24, 24, 96, False, 0, False),
             ("d384_causal", 1, 1, 1, 12, 12, 384, True, 0, False),
             ("d512_kv_longer", 1, 1, 1, 6, 12, 512, False, 0, False)]
    for name, B, H, Hkv, S, KS, D, causal, window, has_rope in cases:
        seed = 12345
        qn, kvn = B * H * S * D, B * Hkv * KS * D
        qf, seed2 = c_oracle.lcg_uniform(seed, qn)
        kf, seed3 = c_oracle.lcg_uniform(0, kvn, state=seed2)
        vf, _ = c_oracle.lcg_uniform(0, kvn, state=seed3)
        qh, kh, vh = qf.astype(np.float16), kf.astype(np.float16), vf.astype(np.float16)
        cos = sin = None
        if has_rope:
            cos, sin = gate_rope_tables(KS, D)
        out = np.empty(qn, dtype=np.float64)
        scale = np.float32(1.0) / np.sqrt(np.float32(D))
        qa, ka, va = (np.ascontiguousarray(x.astype(np.float32)) for x in (qh, kh, vh))
        L.gate_f16_ref(qa.ctypes.data, ka.ctypes.data, va.ctypes.data,
                       cos.ctypes.data if has_rope else None, sin.ctypes.data if has_rope else None,
                       B, H, Hkv, S, KS, D, float(scale), int(causal), window, out.ctypes.data)
        arrays = dict(q=qh.reshape(B, H, S, D), k=kh.reshape(B, Hkv, KS, D), v=vh.reshape(B, Hkv, KS, D),
                      out=out.reshape(B, H, S, D))
        if has_rope:
            arrays.update(cos=cos, sin=sin)
        st.add(name, dict(B=B, H=H, Hkv=Hkv, S=S, KS=KS, D=D, causal=causal, window=window if window else -1,
                          scale=float(scale)), **arrays)
    st.save(HERE / "gate_f16.npz")


def make_gate_int8():
    L = _gate_lib()
    st = Store()
    # (name, B, H, Hkv, S, KS, D, causal, window, per_token): tests/hip_forward_int8qk_gate.hip:264-317.
    cases = [("d64_small", 1, 2, 2, 40, 40, 64, False, -1, False),
             ("d64_kv_longer", 1, 2, 2, 16, 48, 64, False, -1, False),
             ("d64_causal_tail", 1, 2, 2, 37, 37, 64, True, -1, False),
             ("d64_causal_window", 1, 2, 2, 40, 40, 64, True, 8, False),
             ("d64_gqa_r4", 1, 4, 1, 32, 32, 64, False, -1, False),
             ("ptok_d64_window", 1, 2, 2, 40, 40, 64, True, 8, True),
             ("ptok_d64_gqa", 1, 4, 2, 32, 32, 64, False, -1, True),
             ("ptok_d128_gqa_c", 1, 4, 2, 30, 30, 128, True, -1, True),
             ("d128_small", 1, 2, 2, 24, 24, 128, False, -1, False)]
    for name, B, H, Hkv, S, KS, D, causal, window, ptok in cases:
        seed = 424242
        qn, kvn = B * H * S * D, B * Hkv * KS * D
        qf, s2 = c_oracle.lcg_gaussianish(seed, qn)
        kf, s3 = c_oracle.lcg_gaussianish(0, kvn, state=s2)
        vf, _ = c_oracle.lcg_gaussianish(0, kvn, state=s3)
        qsc = np.float32(np.abs(qf).max() / np.float32(127.0))
        ksc = np.float32(np.abs(kf).max() / np.float32(127.0))
        vsc = np.float32(np.abs(vf).max() / np.float32(127.0))
        qvec = np.full(B * H * S, qsc, dtype=np.float32)
        kvec = np.full(B * Hkv * KS, ksc, dtype=np.float32)
        if ptok:
            qm = np.abs(qf.reshape(-1, D)).max(axis=1)
            km = np.abs(kf.reshape(-1, D)).max(axis=1)
            qvec = np.where(qm > 0, qm / np.float32(127.0), np.float32(1.0)).astype(np.float32)
            kvec = np.where(km > 0, km / np.float32(127.0), np.float32(1.0)).astype(np.float32)
        qi = np.array([L.gate_int8_quantize(float(x), float(qvec[i // D])) for i, x in enumerate(qf)], dtype=np.int8)
        ki = np.array([L.gate_int8_quantize(float(x), float(kvec[i // D])) for i, x in enumerate(kf)], dtype=np.int8)
        vi = np.array([L.gate_int8_quantize(float(x), float(vsc)) for x in vf], dtype=np.int8)
        qd = (qi.astype(np.float32) * np.repeat(qvec, D)).astype(np.float32)
        kd = (ki.astype(np.float32) * np.repeat(kvec, D)).astype(np.float32)
        vd = (vi.astype(np.float32) * vsc).astype(np.float32)
        out = np.empty(qn, dtype=np.float64)
        scale = np.float32(1.0) / np.sqrt(np.float32(D))
        L.gate_int8_ref(qd.ctypes.data, kd.ctypes.data, vd.ctypes.data, B, H, Hkv, S, KS, D, float(scale),
                        int(causal), window, out.ctypes.data)
        st.add(name, dict(B=B, H=H, Hkv=Hkv, S=S, KS=KS, D=D, causal=causal, window=window, per_token=ptok,
                          q_scale=float(qsc), k_scale=float(ksc), v_scale=float(vsc), scale=float(scale)),
               qf=qf, kf=kf, qi=qi.reshape(B, H, S, D), ki=ki.reshape(B, Hkv, KS, D),
               vi=vi.reshape(B, Hkv, KS, D), qvec=qvec.reshape(B, H, S), kvec=kvec.reshape(B, Hkv, KS),
               out=out.reshape(B, H, S, D))
    st.save(HERE / "gate_int8.npz")


def make_quant(ref_root):
    spec = importlib.util.spec_from_file_location("ref_rdnattention", ref_root / "rdnattention" / "__init__.py")
    ref = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(ref)
    st = Store()
    gen = torch.Generator().manual_seed(11)
    for name, (B, H, Hkv, S, KS, D) in [("mha", (1, 2, 2, 20, 20, 64)), ("gqa", (2, 4, 2, 9, 13, 128))]:
        q = fp16_randn(gen, B, H, S, D)
        k = fp16_randn(gen, B, Hkv, KS, D)
        v = fp16_randn(gen, B, Hkv, KS, D)
        v[:, :, :, 3] = 0  # an all-zero channel exercises the scale-1.0 fallback
        qi, ki, q_scale, k_scale = ref.quantize_int8_qk_pertoken(q, k)
        pqi, pki, pvi, pqs, pks, pvs, v_channel = ref.quantize_int8_perchannel_v(q, k, v)
        st.add(name, dict(B=B, H=H, Hkv=Hkv, S=S, KS=KS, D=D, pq_scale=pqs, pk_scale=pks, pv_scale=pvs),
               q=q, k=k, v=v, qi=qi, ki=ki, q_scale=q_scale, k_scale=k_scale, pqi=pqi, pki=pki, pvi=pvi,
               v_channel=v_channel)
    st.save(HERE / "quant.npz")


def main():
    from oracle.build_ref import reference_root

    ref_root = reference_root(sys.argv[1] if len(sys.argv) > 1 else None)
    if ref_root is None:
        raise SystemExit("reference checkout not found (pass its root or set RDNA_REFERENCE_ROOT)")
    make_dense_fp32(ref_root)
    make_head_dim(ref_root)
    make_rope(ref_root)
    make_gate_f16()
    make_gate_int8()
    make_quant(ref_root)


if __name__ == "__main__":
    main()
