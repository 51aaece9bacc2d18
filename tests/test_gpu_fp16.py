"""FP16 forward on the B200 through the C ABI / Python API vs the CPU oracle.

Tolerances, stated per test: the reference's gate rel_rms < 5e-3
(tests/hip_forward_gate.hip:243-244), head_dim sweep rel_rms < 3e-3
(tests/head_dim.py:49), RoPE rel_rms < 1e-2 (tests/rope.py:92-97), and the
north-star gate max-abs <= 2e-3 / mean-abs <= 2e-4 against the fp32 oracle.
"""
import numpy as np
import pytest
import torch

from cases import F16_GATE, HEAD_DIM_VARIANTS, ROPE_CASES, gate_f16_inputs, rel_rms, rope_tables
from golden_io import cases as golden_cases
from oracle import c_oracle, torch_oracle

pytestmark = pytest.mark.gpu

R = pytest.importorskip("rdnattention_b200")


@pytest.fixture(scope="module", autouse=True)
def _device():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    yield
    assert R.debug_read_status() == (0, 0), "a kernel recorded an expired wait"


def _run(q, k, v, causal=False, window=-1, cos=None, sin=None):
    dev = "cuda"
    out = R.flash_attn(q.to(dev), k.to(dev), v.to(dev), is_causal=causal, window_size=window,
                       rot_cos=None if cos is None else cos.to(dev), rot_sin=None if sin is None else sin.to(dev))
    return out.cpu()


@pytest.mark.parametrize("case", F16_GATE, ids=[c[0] for c in F16_GATE])
def test_reference_fp16_gate_cases(case):
    name, B, H, Hkv, S, KS, D, causal, window, rope = case
    q, k, v, cos, sin = gate_f16_inputs(B, H, Hkv, S, KS, D, rope)
    got = _run(q, k, v, causal, window, cos, sin)
    ref = c_oracle.attention_f16(q, k, v, causal=causal, window=window, rot_cos=cos, rot_sin=sin,
                                 scale=np.float32(1.0) / np.sqrt(np.float32(D)))
    err = rel_rms(got, ref)
    assert err < 5e-3, f"{name}: rel_rms {err:.3e}"


@pytest.mark.parametrize("D", [32, 64, 96, 128, 160, 256, 384, 512])
def test_head_dim_sweep(D):
    """tests/head_dim.py variants at 8 heads, rel_rms < 3e-3 vs fp64."""
    for name, kvdiv, S, KS, causal, window in HEAD_DIM_VARIANTS:
        torch.manual_seed(1234)
        H = 8
        Hkv = max(1, H // kvdiv)
        q = torch.randn(1, H, S, D).half()
        k = torch.randn(1, Hkv, KS, D).half()
        v = torch.randn(1, Hkv, KS, D).half()
        got = _run(q, k, v, causal, window)
        assert torch.isfinite(got).all(), f"D={D} {name}: non-finite output"
        ref = c_oracle.attention_f16(q, k, v, causal=causal, window=window)
        err = rel_rms(got, ref)
        assert err < 3e-3, f"D={D} {name}: rel_rms {err:.3e}"


@pytest.mark.parametrize("case", ROPE_CASES, ids=[c[0] for c in ROPE_CASES])
def test_rope_cases(case):
    name, B, H, KH, S, KS, D, causal = case
    torch.manual_seed(7)
    q = torch.randn(B, H, S, D).half()
    k = torch.randn(B, KH, KS, D).half()
    v = torch.randn(B, KH, KS, D).half()
    cos, sin = rope_tables(max(S, KS), D)
    got = _run(q, k, v, causal, -1, cos, sin)
    ref = c_oracle.attention_f16(q, k, v, causal=causal, rot_cos=cos, rot_sin=sin)
    err = rel_rms(got, ref)
    assert err < 1e-2, f"{name}: rel_rms {err:.3e}"
    assert err < 1e-3, f"{name}: rel_rms {err:.3e} (rope.py's expectation is ~4e-4)"


# The head_dim <= 128 kernels rotate Q in shared memory (K goes through the
# pre-pass).  Cases for the rotation's branches: 64-byte-swizzle boxes (D = 32,
# 96), tile pairs at different positions (odd group sizes: MHA, G = 3) and at
# the same positions (even G), partial last tiles, key_seq_len != seq_len.
Q_ROTATION_CASES = [
    # (B, H, Hkv, S, KS, D, causal)
    (1, 4, 4, 200, 200, 32, True),
    (2, 6, 2, 333, 333, 32, False),
    (1, 4, 4, 257, 257, 96, True),
    (1, 8, 2, 300, 300, 96, False),
    (2, 6, 2, 129, 400, 64, False),
    (1, 3, 1, 384, 384, 128, True),
    (1, 8, 2, 70, 600, 128, False),
    (1, 8, 4, 520, 260, 128, False),
]


@pytest.mark.parametrize("case", Q_ROTATION_CASES, ids=[f"B{c[0]}H{c[1]}/{c[2]}S{c[3]}KS{c[4]}D{c[5]}"
                                                        f"{'c' if c[6] else ''}" for c in Q_ROTATION_CASES])
def test_in_kernel_q_rotation(case):
    B, H, Hkv, S, KS, D, causal = case
    g = torch.Generator().manual_seed(B * 1000 + S + D)
    q = torch.randn(B, H, S, D, generator=g).half()
    k = torch.randn(B, Hkv, KS, D, generator=g).half()
    v = torch.randn(B, Hkv, KS, D, generator=g).half()
    cos, sin = rope_tables(max(S, KS), D, 500000.0)
    got = _run(q, k, v, causal, -1, cos, sin)
    # the kernel rounds rotated Q and K to fp16, like the reference kernel
    ref = c_oracle.attention_f16(q, k, v, causal=causal, rot_cos=cos, rot_sin=sin, rope_round=True)
    diff = (got.double() - ref).abs()
    assert diff.max().item() <= 2e-3 and diff.mean().item() <= 2e-4, \
        f"max {diff.max().item():.3e} mean {diff.mean().item():.3e}"


@pytest.mark.parametrize("family", ["dense_fp32", "head_dim", "rope", "gate_f16"])
def test_golden_fixtures(family):
    """Kernel output vs outputs produced by the reference's own oracles."""
    for m, a in golden_cases(family):
        scale = m.get("scale")
        got = R.flash_attn_strided(a["q"].cuda(), a["k"].cuda(), a["v"].cuda(), is_causal=m["causal"],
                                   window_size=m["window"],
                                   rot_cos=a["cos"].cuda() if "cos" in a else None,
                                   rot_sin=a["sin"].cuda() if "sin" in a else None, scale=scale).cpu()
        ref = torch.nan_to_num(a["out"].double(), nan=0.0)  # rows with no key: 0, as the reference kernel
        err = (got.double() - ref).abs()
        assert err.max().item() <= 2e-3, f"{family}/{m['name']}: max abs {err.max().item():.3e}"
        assert rel_rms(got, ref) < 3e-3, f"{family}/{m['name']}"


def test_baseline_config1_tolerance_gate():
    """MHA B=1,H=8,S=512,D=64 non-causal, N(0,1) fp16, vs the fp32 oracle:
    max-abs <= 2e-3 and mean-abs <= 2e-4."""
    g = torch.Generator().manual_seed(0)
    q = torch.randn(1, 8, 512, 64, generator=g).half()
    k = torch.randn(1, 8, 512, 64, generator=g).half()
    v = torch.randn(1, 8, 512, 64, generator=g).half()
    got = _run(q, k, v).double()
    ref32 = torch_oracle.attention(q, k, v).double()
    err = (got - ref32).abs()
    assert err.max().item() <= 2e-3, err.max().item()
    assert err.mean().item() <= 2e-4, err.mean().item()


def _sampled_rows(B, H, S, n, seed):
    rng = np.random.default_rng(seed)
    rows = set(rng.integers(0, B * H * S, size=n).tolist())
    for b in (0, B - 1):  # first/last row of a few heads, diagonal edges
        for h in (0, H - 1):
            rows.update([(b * H + h) * S, (b * H + h) * S + S - 1])
    return np.array(sorted(rows), dtype=np.int64)


def _unit_rows(H, Hkv, S, b, kvh):
    """Flat row indices ((b * H + h) * S + q) of every row of one (batch, KV-head) unit:
    the G query heads of KV head kvh, all S rows."""
    G = H // Hkv
    heads = np.arange(kvh * G, (kvh + 1) * G, dtype=np.int64)
    return ((b * H + heads)[:, None] * S + np.arange(S, dtype=np.int64)[None, :]).reshape(-1)


# Llama-3-8B-shaped prefill workloads at full size: causal GQA S=4096 (RoPE 5e5),
# causal window 4096 at S=16384 and two-sided +-1024 at S=8192 (RoPE 1e6).
FULL_SIZE = {
    "gqa_causal_b4_s4096": (4, 32, 8, 4096, 128, True, -1, 500000.0),
    "window4096_causal_s16384": (1, 32, 8, 16384, 128, True, 4096, 1e6),
    "window_pm1024_s8192": (1, 32, 8, 8192, 128, False, 2048, 1e6),
}


@pytest.mark.parametrize("cfg", sorted(FULL_SIZE))
def test_full_size_configs_whole_unit_and_sampled_rows(cfg):
    """The benchmarked prefill shapes at full size, against the fp64 oracle with
    max-abs <= 2e-3 and mean-abs <= 2e-4: every row of one whole (batch, KV-head) unit
    (the last batch element's last KV head for the causal GQA shape, whose causal
    diagonal tiles run last; KV head 0 of the window shapes, every row of which
    crosses a window edge) plus a random row sample over all units."""
    B, H, Hkv, S, D, causal, window, theta = FULL_SIZE[cfg]
    g = torch.Generator().manual_seed(0)
    q = torch.randn(B, H, S, D, generator=g).half()
    k = torch.randn(B, Hkv, S, D, generator=g).half()
    v = torch.randn(B, Hkv, S, D, generator=g).half()
    cos, sin = rope_tables(S, D, theta)
    got = _run(q, k, v, causal, window, cos, sin)
    unit = _unit_rows(H, Hkv, S, B - 1, Hkv - 1) if causal and window <= 0 else _unit_rows(H, Hkv, S, 0, 0)
    rows = np.union1d(unit, _sampled_rows(B, H, S, 96, seed=1))
    ref = c_oracle.attention_f16(q, k, v, causal=causal, window=window, rot_cos=cos, rot_sin=sin, rows=rows)
    err = (got.reshape(-1, D)[torch.from_numpy(rows)].double() - ref).abs()
    assert err.max().item() <= 2e-3, err.max().item()
    assert err.mean().item() <= 2e-4, err.mean().item()


def test_rotate_half_equivalence():
    """The Llama-shaped prefill workloads name rotate-half RoPE; the ABI is interleaved pairs
    (docs/api.md:92-93).  Permuting Q and K channels (2i <- i, 2i+1 <- i+D/2)
    turns one into the other and leaves Q K^T unchanged."""
    B, H, Hkv, S, D = 1, 4, 2, 200, 128
    g = torch.Generator().manual_seed(5)
    q = torch.randn(B, H, S, D, generator=g).half()
    k = torch.randn(B, Hkv, S, D, generator=g).half()
    v = torch.randn(B, Hkv, S, D, generator=g).half()
    cos, sin = rope_tables(S, D, 500000.0)
    perm = torch.empty(D, dtype=torch.long)
    perm[0::2] = torch.arange(D // 2)
    perm[1::2] = torch.arange(D // 2) + D // 2
    got = _run(q[..., perm].contiguous(), k[..., perm].contiguous(), v, True, -1, cos, sin)
    # rotate-half reference in fp64
    def rot_half(x):
        x = x.double()
        c = torch.cat([cos, cos], -1).double()
        s = torch.cat([sin, sin], -1).double()
        x1, x2 = x[..., : D // 2], x[..., D // 2:]
        return x * c + torch.cat([-x2, x1], -1) * s
    qr, kr = rot_half(q), rot_half(k)
    ref = torch.empty(B, H, S, D, dtype=torch.float64)
    mask = torch.ones(S, S, dtype=torch.bool).tril()
    for h in range(H):
        s_ = (qr[0, h] @ kr[0, h // 2].T) * D ** -0.5
        s_ = s_.masked_fill(~mask, float("-inf"))
        ref[0, h] = s_.softmax(-1) @ v[0, h // 2].double()
    assert (got.double() - ref).abs().max().item() <= 2e-3


def test_strided_kv_decode_layout():
    """K/V stored [B, KS, Hkv, D] (a KV-cache layout) passed with strides."""
    B, H, Hkv, S, KS, D = 2, 16, 4, 3, 700, 128
    g = torch.Generator().manual_seed(9)
    q = torch.randn(B, H, S, D, generator=g).half()
    kb = torch.randn(B, KS, Hkv, D, generator=g).half()
    vb = torch.randn(B, KS, Hkv, D, generator=g).half()
    k, v = kb.transpose(1, 2), vb.transpose(1, 2)
    got = R.flash_attn_strided(q.cuda(), kb.cuda().transpose(1, 2), vb.cuda().transpose(1, 2)).cpu()
    ref = c_oracle.attention_f16(q, k, v)
    assert rel_rms(got, ref) < 3e-3
    assert (got.double() - ref).abs().max().item() <= 2e-3


def test_strided_output_and_query():
    """Non-contiguous Q and O views ([B, S, H, D] storage) through the C ABI."""
    B, H, S, D = 2, 4, 130, 64
    g = torch.Generator().manual_seed(10)
    qb = torch.randn(B, S, H, D, generator=g).half()
    k = torch.randn(B, H, S, D, generator=g).half()
    v = torch.randn(B, H, S, D, generator=g).half()
    ob = torch.zeros(B, S, H, D, dtype=torch.float16, device="cuda")
    R.flash_attn_strided(qb.cuda().transpose(1, 2), k.cuda(), v.cuda(), is_causal=True, out=ob.transpose(1, 2))
    ref = c_oracle.attention_f16(qb.transpose(1, 2), k, v, causal=True)
    assert rel_rms(ob.cpu().transpose(1, 2), ref) < 3e-3


def test_empty_rows_are_zero():
    """Causal with seq_len > key_seq_len: rows q < S-KS see no key -> 0 (fa2_forward_f16.hip:733)."""
    q = torch.randn(1, 2, 300, 64).half()
    k = torch.randn(1, 2, 100, 64).half()
    v = torch.randn(1, 2, 100, 64).half()
    got = _run(q, k, v, causal=True)
    assert torch.equal(got[:, :, :200], torch.zeros_like(got[:, :, :200]))
    ref = c_oracle.attention_f16(q, k, v, causal=True)
    assert rel_rms(got, ref) < 3e-3


def test_zero_key_length_writes_zeros():
    q = torch.randn(1, 2, 10, 64).half().cuda()
    k = torch.empty(1, 2, 0, 64, dtype=torch.float16, device="cuda")
    out = R.flash_attn_strided(q, k, k)
    assert torch.equal(out.cpu(), torch.zeros(1, 2, 10, 64, dtype=torch.float16))


def test_deterministic_run_to_run():
    g = torch.Generator().manual_seed(11)
    q = torch.randn(2, 8, 700, 128, generator=g).half().cuda()
    k = torch.randn(2, 2, 700, 128, generator=g).half().cuda()
    a = R.flash_attn(q, k, k, is_causal=True)
    b = R.flash_attn(q, k, k, is_causal=True)
    assert torch.equal(a, b)


def test_runs_on_non_default_stream():
    q = torch.randn(1, 4, 256, 64).half().cuda()
    s = torch.cuda.Stream()
    with torch.cuda.stream(s):
        out = R.flash_attn(q, q, q)
    s.synchronize()
    ref = c_oracle.attention_f16(q.cpu(), q.cpu(), q.cpu())
    assert rel_rms(out.cpu(), ref) < 3e-3


@pytest.mark.parametrize("S,KS,causal,rope,axis", [
    (300, 300, True, True, "head"),     # prefill, RoPE pre-pass reading the broadcast K
    (257, 700, False, False, "head"),   # prefill, cross-attention
    (1, 1000, False, False, "head"),    # decode kernel
    (200, 200, True, False, "batch"),   # one K/V shared by every batch element
])
def test_kv_stride_zero_broadcast(S, KS, causal, rope, axis):
    """K/V broadcast with element stride 0 on the head (MQA through a GQA-shaped call) or
    batch axis, as the reference's int64 strides allow (src/rdna/fa2_forward_f16.hip:885-894):
    the same result as the call on the materialised tensors."""
    B, H, Hkv, D = 2, 8, 4, 128
    g = torch.Generator().manual_seed(S + KS)
    q = torch.randn(B, H, S, D, generator=g).half()
    if axis == "head":
        k1 = torch.randn(B, 1, KS, D, generator=g).half()
        v1 = torch.randn(B, 1, KS, D, generator=g).half()
    else:
        k1 = torch.randn(1, Hkv, KS, D, generator=g).half()
        v1 = torch.randn(1, Hkv, KS, D, generator=g).half()
    k, v = k1.expand(B, Hkv, KS, D), v1.expand(B, Hkv, KS, D)
    cos, sin = rope_tables(max(S, KS), D) if rope else (None, None)
    kd, vd = k1.cuda().expand(B, Hkv, KS, D), v1.cuda().expand(B, Hkv, KS, D)
    assert 0 in kd.stride()[:2] and 0 in vd.stride()[:2]
    got = R.flash_attn_strided(q.cuda(), kd, vd, is_causal=causal, rot_cos=None if cos is None else cos.cuda(),
                               rot_sin=None if sin is None else sin.cuda()).cpu()
    ref = c_oracle.attention_f16(q, k.contiguous(), v.contiguous(), causal=causal, rot_cos=cos, rot_sin=sin)
    err = (got.double() - ref).abs()
    assert err.max().item() <= 2e-3 and err.mean().item() <= 2e-4


def test_kernel_timing_hook_times_the_attention_kernel_alone():
    """rdna_debug_set_kernel_events: the events bracket the attention kernel of a
    RoPE call (not its K pre-pass), the output is unchanged, and the hook is off
    again afterwards."""
    B, H, Hkv, S, D = 2, 8, 2, 2048, 128
    g = torch.Generator().manual_seed(7)
    q = torch.randn(B, H, S, D, generator=g).half().cuda()
    k = torch.randn(B, Hkv, S, D, generator=g).half().cuda()
    v = torch.randn(B, Hkv, S, D, generator=g).half().cuda()
    cos, sin = rope_tables(S, D, 500000.0, device="cuda")
    ref = R.flash_attn(q, k, v, is_causal=True, rot_cos=cos, rot_sin=sin)
    outs = []
    kernel_ms = R.debug_time_kernel(
        lambda: outs.append(R.flash_attn(q, k, v, is_causal=True, rot_cos=cos, rot_sin=sin)), repeats=5)
    torch.cuda.synchronize()
    assert all(torch.equal(o, ref) for o in outs) and len(outs) == 5
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    for _ in range(5):
        R.flash_attn(q, k, v, is_causal=True, rot_cos=cos, rot_sin=sin)
    e.record()
    torch.cuda.synchronize()
    call_ms = s.elapsed_time(e) / 5
    assert 0.0 < kernel_ms < call_ms * 1.05, (kernel_ms, call_ms)
    assert R.debug_read_status() == (0, 0)
