"""Pins the CPU oracles (oracle/) against fixtures produced by the reference's
own oracle code (tests/golden/make_golden.py).  CPU only."""
import numpy as np
import pytest
import torch

from golden_io import cases
from oracle import c_oracle, torch_oracle


def _max_err(got, ref):
    ref = ref.double()
    # tests/head_dim.py's masked softmax yields NaN for a row that sees no key (causal with
    # seq_len > key_seq_len); the reference kernel and gate define that row as 0
    # (src/rdna/fa2_forward_f16.hip:733, tests/hip_forward_gate.hip:124).
    nan_rows = torch.isnan(ref).all(dim=-1, keepdim=True)
    assert not (torch.isnan(ref) & ~nan_rows).any(), "partial NaN row in reference output"
    ref = torch.where(nan_rows, torch.zeros_like(ref), ref)
    return (got.double() - ref).abs().max().item()


@pytest.mark.parametrize("family", ["dense_fp32", "head_dim", "rope", "gate_f16"])
def test_c_oracle_matches_reference_fp16_oracles(family):
    for m, a in cases(family):
        rope = "cos" in a
        scale = m.get("scale", m["D"] ** -0.5)
        got = c_oracle.attention_f16(a["q"], a["k"], a["v"], causal=m["causal"], window=m["window"],
                                     rot_cos=a.get("cos"), rot_sin=a.get("sin"), scale=scale)
        ref = a["out"]
        # gate_f16 is the same fp64 arithmetic (float RoPE, double dot products): near-exact.
        # The fp32 / fp32-stored references carry their own ~1e-6 rounding; rope.py rotates in fp64.
        tol = 1e-12 if family == "gate_f16" else 2e-5
        err = _max_err(got, ref)
        assert err <= tol, f"{family}/{m['name']}: max abs err {err:.3e} > {tol}"


def test_c_oracle_matches_reference_int8_gate():
    for m, a in cases("gate_int8"):
        qs = a["qvec"] if m["per_token"] else m["q_scale"]
        ks = a["kvec"] if m["per_token"] else m["k_scale"]
        got = c_oracle.attention_int8(a["qi"], a["ki"], a["vi"], qs, ks, m["v_scale"], causal=m["causal"],
                                      window=m["window"], scale=m["scale"])
        err = _max_err(got, a["out"])
        assert err <= 1e-12, f"gate_int8/{m['name']}: max abs err {err:.3e}"


def test_c_oracle_quantize_matches_reference_gate():
    for m, a in cases("gate_int8"):
        D = m["D"]
        qi = c_oracle.quantize(a["qf"].numpy(), a["qvec"].numpy().reshape(-1), D)
        assert np.array_equal(qi, a["qi"].numpy().reshape(-1)), m["name"]
        ki = c_oracle.quantize(a["kf"].numpy(), a["kvec"].numpy().reshape(-1), D)
        assert np.array_equal(ki, a["ki"].numpy().reshape(-1)), m["name"]


@pytest.mark.parametrize("family", ["dense_fp32", "head_dim", "rope"])
def test_torch_oracle_matches_reference(family):
    for m, a in cases(family):
        got = torch_oracle.attention(a["q"], a["k"], a["v"], causal=m["causal"], window=m["window"],
                                     rot_cos=a.get("cos"), rot_sin=a.get("sin"))
        err = _max_err(got, a["out"])
        assert err <= 5e-5, f"{family}/{m['name']}: max abs err {err:.3e}"


def test_c_oracle_row_sampling_matches_full():
    for m, a in cases("head_dim"):
        if m["D"] != 64:
            continue
        full = c_oracle.attention_f16(a["q"], a["k"], a["v"], causal=m["causal"], window=m["window"])
        B, H, S, D = a["q"].shape
        rows = np.arange(0, B * H * S, 3)
        part = c_oracle.attention_f16(a["q"], a["k"], a["v"], causal=m["causal"], window=m["window"], rows=rows)
        assert torch.equal(part, full.reshape(-1, D)[torch.from_numpy(rows)])


def test_c_oracle_reads_strided_inputs():
    """[B,S,Hkv,D] storage viewed as [B,Hkv,S,D] (the decode layout) gives the same result."""
    g = torch.Generator().manual_seed(3)
    B, H, Hkv, S, KS, D = 2, 4, 2, 5, 33, 64
    q = torch.randn(B, H, S, D, generator=g).half()
    kb = torch.randn(B, KS, Hkv, D, generator=g).half()
    vb = torch.randn(B, KS, Hkv, D, generator=g).half()
    k, v = kb.permute(0, 2, 1, 3), vb.permute(0, 2, 1, 3)
    a = c_oracle.attention_f16(q, k, v)
    b = c_oracle.attention_f16(q, k.contiguous(), v.contiguous())
    assert torch.equal(a, b)


def test_flop_count_matches_reference_formula():
    # tests/benchmark.py:77-88 closed form for causal without window.
    for S, KS in [(1, 2048), (128, 2048), (300, 300), (4096, 4096)]:  # delta >= 0, as the formula assumes
        delta = KS - S
        t = max(0, min(KS - delta, S))
        closed = t * (delta + 1) + t * (t - 1) // 2 + (S - t) * KS
        assert torch_oracle.valid_pairs(S, KS, True, -1) == closed
    assert torch_oracle.valid_pairs(4096, 4096, True, -1) == 8390656
    assert torch_oracle.valid_pairs(16384, 16384, True, 4096) == 58722304
    assert torch_oracle.valid_pairs(8192, 8192, False, 2048) == 15735808
