"""Benchmark of the FA2 forward hot path on B200, one JSON line on rank 0.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--config 2] [--impl ours|reference]
    python -m torch.distributed.run --nproc-per-node N --master-addr 127.0.0.1 ... bench.py --gpus N

Workload (default): the Llama-3-8B-shaped causal GQA prefill in FP16 (B=4,
Hq=32, Hkv=8, S=4096, D=128, RoPE theta=5e5 applied in-kernel).  On one GPU a
step is one attention call over the whole batch.  On N GPUs (torchrun) the
same workload is sharded (strong scaling): each rank computes its rectangle
of (batch, KV-head group) units (rdnattention_b200.multigpu.plan) and the
step is the library's flash_attn_sharded call, so the NCCL all-gather that
assembles the full O on every rank is inside the timed step; the
compute-only time of the rank's shard is reported beside it.  `value` is the
workload's FLOPs over the max-over-ranks device time; FLOPs count exactly
the visible (query, key) pairs, both GEMMs at 2 FLOP/MAC
(tests/benchmark.py:77-88).

Inputs are synthetic N(0,1) fp16 (seed 0).  A step whose per-rank operands
are smaller than the 126 MB L2 (the INT8 and small workloads, and the shards
of the prefill at N >= 4) rotates through enough independent input sets that
no step finds its inputs in L2; larger ones stay resident, no flush.
`e2e` times the same call through the public Python API with the step's
inputs copied in from pinned host memory and the output read back.
`--impl reference` times the CPU restatement of the reference's algorithm
(oracle/torch_oracle.py: fp32 torch on the host cores; the reference itself
is HIP-only and cannot run here) on one query head of the same workload
per step.
"""
import argparse
import itertools
import json
import math
import os
import statistics
import sys
import threading
import time
from pathlib import Path

import torch

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

CONFIGS = {
    "1": dict(workload="cfg1_mha_b1_h8_s512_d64", B=1, H=8, Hkv=8, S=512, KS=512, D=64, causal=False, window=-1,
              theta=None, kind="fp16"),
    "2": dict(workload="cfg2_llama3_8b_gqa_causal_prefill_s4096_rope", B=4, H=32, Hkv=8, S=4096, KS=4096, D=128,
              causal=True, window=-1, theta=500000.0, kind="fp16"),
    "3": dict(workload="cfg3_int8_b8_h16_s2048_d64_pertoken_qk_perchannel_v", B=8, H=16, Hkv=16, S=2048, KS=2048,
              D=64, causal=False, window=-1, theta=None, kind="int8"),
    # INT8 at head_dim 128 (same scheme as config 3): the two-pass kernel
    "3h128": dict(workload="int8_b4_h16_s2048_d128_pertoken_qk_perchannel_v", B=4, H=16, Hkv=16, S=2048, KS=2048,
                  D=128, causal=False, window=-1, theta=None, kind="int8"),
    "4a": dict(workload="cfg4a_sliding_causal_w4096_s16384_rope", B=1, H=32, Hkv=8, S=16384, KS=16384, D=128,
               causal=True, window=4096, theta=1e6, kind="fp16"),
    "4b": dict(workload="cfg4b_two_sided_pm1024_s8192_rope", B=1, H=32, Hkv=8, S=8192, KS=8192, D=128,
               causal=False, window=2048, theta=1e6, kind="fp16"),
    "5": dict(workload="cfg5_decode_s1_ks32768_b64_h64_kv8_bshd_cache", B=64, H=64, Hkv=8, S=1, KS=32768, D=128,
              causal=False, window=-1, theta=None, kind="decode"),
}

NVML_REASONS = {0x1: "gpu_idle", 0x2: "applications_clocks_setting", 0x4: "sw_power_cap", 0x8: "hw_slowdown",
                0x10: "sync_boost", 0x20: "sw_thermal_slowdown", 0x40: "hw_thermal_slowdown",
                0x80: "hw_power_brake_slowdown", 0x100: "display_clock_setting"}


def metric_of(cfg):
    if cfg["kind"] == "decode":
        return "decode HBM GB/s", "GB/s"
    if cfg["kind"] == "int8":
        return "attention fwd TOPS (INT8)", "TOP/s"
    return "attention fwd TFLOPS (FP16)", "TFLOP/s"


def work_units(cfg, B=None):
    """Algorithmic work of one step: FLOPs (prefill) or HBM bytes (decode)."""
    from oracle.torch_oracle import flops  # pure arithmetic helper (pair counting)

    B = cfg["B"] if B is None else B
    if cfg["kind"] == "decode":
        kv = 2 * B * cfg["Hkv"] * cfg["KS"] * cfg["D"] * 2
        qo = 2 * B * cfg["H"] * cfg["S"] * cfg["D"] * 2
        return kv + qo
    return flops(B, cfg["H"], cfg["S"], cfg["KS"], cfg["D"], cfg["causal"], cfg["window"])


def algorithmic_bytes(cfg):
    e = 1 if cfg["kind"] == "int8" else 2
    q = cfg["B"] * cfg["H"] * cfg["S"] * cfg["D"] * e
    kv = 2 * cfg["B"] * cfg["Hkv"] * cfg["KS"] * cfg["D"] * e
    o = cfg["B"] * cfg["H"] * cfg["S"] * cfg["D"] * 2
    return q + kv + o


# ---------------------------------------------------------------- clocks
class ClockSampler:
    """Polls NVML SM clock and clock-event reasons on a thread while running."""

    def __init__(self, index):
        self.samples = []
        self.reasons = 0
        self.max_mhz = None
        self._stop = threading.Event()
        self._ok = False
        try:
            import pynvml

            pynvml.nvmlInit()
            self._nv = pynvml
            self._h = pynvml.nvmlDeviceGetHandleByIndex(index)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self._h, pynvml.NVML_CLOCK_SM)
            self._ok = True
        except Exception:
            self._ok = False

    def _reasons(self):
        nv = self._nv
        fn = getattr(nv, "nvmlDeviceGetCurrentClocksEventReasons", None) or \
            getattr(nv, "nvmlDeviceGetCurrentClocksThrottleReasons")
        return fn(self._h)

    def _run(self):
        while not self._stop.is_set():
            try:
                self.samples.append(self._nv.nvmlDeviceGetClockInfo(self._h, self._nv.NVML_CLOCK_SM))
                self.reasons |= int(self._reasons())
            except Exception:
                pass
            time.sleep(0.002)

    def __enter__(self):
        if self._ok:
            self._t = threading.Thread(target=self._run, daemon=True)
            self._t.start()
        return self

    def __exit__(self, *a):
        if self._ok:
            self._stop.set()
            self._t.join()

    def summary(self):
        if not self._ok:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvml_unavailable"]}
        names = [n for bit, n in NVML_REASONS.items() if self.reasons & bit and n != "gpu_idle"]
        return {"sm_mhz": statistics.median(self.samples) if self.samples else None, "sm_max_mhz": self.max_mhz,
                "reasons": names, "samples": len(self.samples)}


# ---------------------------------------------------------------- inputs
def make_inputs(cfg, device, seed):
    g = torch.Generator(device=device).manual_seed(seed)
    B, H, Hkv, S, KS, D = cfg["B"], cfg["H"], cfg["Hkv"], cfg["S"], cfg["KS"], cfg["D"]
    q = torch.randn(B, H, S, D, generator=g, device=device, dtype=torch.float16)
    if cfg["kind"] == "decode":
        # KV cache stored [B, KS, Hkv, D], viewed [B, Hkv, KS, D] through strides
        kc = torch.randn(B, KS, Hkv, D, generator=g, device=device, dtype=torch.float16)
        vc = torch.randn(B, KS, Hkv, D, generator=g, device=device, dtype=torch.float16)
        return dict(q=q, k=kc.transpose(1, 2), v=vc.transpose(1, 2), kc=kc, vc=vc)
    k = torch.randn(B, Hkv, KS, D, generator=g, device=device, dtype=torch.float16)
    v = torch.randn(B, Hkv, KS, D, generator=g, device=device, dtype=torch.float16)
    out = dict(q=q, k=k, v=v)
    if cfg["theta"]:
        rows = max(S, KS)
        pos = torch.arange(rows, device=device).unsqueeze(1).float()
        inv = cfg["theta"] ** (-torch.arange(0, D, 2, device=device).float() / D)
        ang = pos * inv
        out["cos"], out["sin"] = ang.cos().contiguous(), ang.sin().contiguous()
    if cfg["kind"] == "int8":
        import rdnattention_b200 as R

        _, _, vi, _, _, vs, vch = R.quantize_int8_perchannel_v(q, k, v)
        qi, ki, qsc, ksc = R.quantize_int8_qk_pertoken(q, k)
        out.update(qi=qi, ki=ki, vi=vi, qsc=qsc, ksc=ksc, vs=vs)
    return out


def step_fn(cfg, x):
    """One hot-path pass over resident device inputs (the launch the device timing measures)."""
    import rdnattention_b200 as R

    if cfg["kind"] == "int8":
        return lambda: R.flash_attn_int8qk(x["qi"], x["ki"], x["vi"], x["qsc"], x["ksc"], x["vs"])
    if cfg["kind"] == "decode":
        out = torch.empty_like(x["q"])
        return lambda: R.flash_attn_strided(x["q"], x["k"], x["v"], out=out)
    out = torch.empty_like(x["q"])
    return lambda: R.flash_attn_strided(x["q"], x["k"], x["v"], is_causal=cfg["causal"],
                                        window_size=cfg["window"], rot_cos=x.get("cos"), rot_sin=x.get("sin"),
                                        out=out)


def sharded_step_fns(cfg, x, world, rank, chunks, sym=None):
    """The N-GPU step on one rank: (full, compute_only, shard).  `full` is the library
    call a user makes, rdnattention_b200.multigpu.flash_attn_sharded on the full
    inputs: with `sym` (a SymmetricOutput) one kernel computes the rank's units and
    stores every O tile into all ranks' outputs over NVLink, then a barrier kernel
    (epoch flags over NVLink) orders those stores; else the rank's units, then the NCCL all-gather
    that gives every rank the whole O (overlapped piece by piece when chunks > 1).
    `compute_only` launches the same units' kernel alone."""
    import rdnattention_b200 as R
    from rdnattention_b200 import multigpu as M

    kw = {}
    if cfg["kind"] == "fp16":
        kw = dict(is_causal=cfg["causal"], window_size=cfg["window"], rot_cos=x.get("cos"), rot_sin=x.get("sin"))
    shard = M.plan(cfg["B"], cfg["Hkv"], world, rank, interleave=sym is not None or chunks > 1)
    names = ("qi", "ki", "vi") if cfg["kind"] == "int8" else ("q", "k", "v")
    qs, ks, vs = M.local_views(*(x[n] for n in names), shard)
    out = torch.empty(qs.shape, dtype=torch.float16, device="cuda")

    if cfg["kind"] == "int8":
        G = cfg["H"] // cfg["Hkv"]
        bsl = slice(shard.b0, shard.b1, shard.bstep)
        qsc = x["qsc"][bsl, shard.g0 * G:shard.g1 * G].contiguous()
        ksc = x["ksc"][bsl, shard.g0:shard.g1].contiguous()

        def full():
            return M.flash_attn_int8qk_sharded(x["qi"], x["ki"], x["vi"], x["qsc"], x["ksc"], x["vs"],
                                               out=sym, chunks=chunks)

        def compute_only():
            if qs.numel():
                R.flash_attn_int8qk_strided(qs, ks, vs, qsc, ksc, x["vs"], out=out)

        return full, compute_only, shard

    def full():
        if sym is not None:
            return M.flash_attn_sharded(x["q"], x["k"], x["v"], out=sym, **kw)
        return M.flash_attn_sharded(x["q"], x["k"], x["v"], chunks=chunks, **kw)

    def compute_only():
        if qs.numel():
            R.flash_attn_strided(qs, ks, vs, out=out, **kw)

    return full, compute_only, shard


L2_BYTES = 126 * 1024 * 1024


def input_sets(cfg, world=1):
    b = rank_bytes(cfg, world)
    return 1 if b >= L2_BYTES else min(256, math.ceil(2 * L2_BYTES / b) + 1)


def l2_note(cfg, n_sets, world=1):
    if n_sets == 1:
        return "inputs larger than L2, no flush"
    return (f"{n_sets} rotating input sets ({n_sets * rank_bytes(cfg, world) / 1e6:.0f} MB per rank > L2): "
            "each step's inputs were evicted by the steps before it, no flush")


def config_dict(cfg, world, n_sets, gather="fused"):
    """The workload description both arms print (the driver compares them)."""
    how = ("O gathered into every rank by peer stores from the attention epilogue" if gather == "fused"
           else "NCCL all-gather of O")
    return {"workload": cfg["workload"], "B": cfg["B"], "H": cfg["H"], "Hkv": cfg["Hkv"], "S": cfg["S"],
            "KS": cfg["KS"], "D": cfg["D"], "causal": cfg["causal"], "window": cfg["window"],
            "rope_theta": cfg["theta"], "global_batch": cfg["B"],
            "parallelism": ("one GPU" if world == 1 else
                            f"(batch, kv-head group) units sharded over {world} ranks; {how}"),
            "l2": l2_note(cfg, n_sets, world)}


def rank_bytes(cfg, world):
    """Operand bytes one rank reads and writes per step (its shard of the units)."""
    return algorithmic_bytes(cfg) / max(1, min(world, cfg["B"] * cfg["Hkv"]))


def launches_per_step(cfg):
    """Kernels of this library one step launches: the RoPE pre-pass (K rotation)
    and the attention kernel for RoPE prefill, else the attention kernel alone."""
    return 2 if cfg["kind"] == "fp16" and cfg["theta"] and cfg["S"] * (cfg["H"] // cfg["Hkv"]) > 64 else 1


# ---------------------------------------------------------------- timing
def barrier(dist_on):
    if dist_on:
        torch.distributed.barrier()
    torch.cuda.synchronize()


def time_device(fn, steps, warmup, dist_on, sampler=None):
    for _ in range(warmup):
        fn()
    barrier(dist_on)
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ctx = sampler if sampler is not None else _Null()
    with ctx:
        start.record()
        for _ in range(steps):
            fn()
        end.record()
        torch.cuda.synchronize()
    barrier(dist_on)
    ms = start.elapsed_time(end)
    if dist_on:
        t = torch.tensor([ms], device="cuda", dtype=torch.float64)
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        ms = t.item()
    return ms


class _Null:
    def __enter__(self):
        return self

    def __exit__(self, *a):
        pass


def time_e2e(cfg, x, steps, warmup, dist_on):
    """Public API with host buffers, pipelined as a serving loop would run it: every
    step copies its inputs from pinned host memory to the device (copy stream),
    calls the attention API on them (compute stream) and copies the output back to
    pinned host memory (a second copy stream), with two buffer sets so step i+1's
    upload and step i-1's download overlap step i's attention (the two copy
    directions use separate copy engines).  Timed from before the first upload to
    after the last download, with events, max over ranks."""
    import rdnattention_b200 as R

    names = ["qi", "ki", "vi", "qsc", "ksc"] if cfg["kind"] == "int8" else ["q", "k", "v"]
    if cfg["kind"] == "decode":
        names = ["q", "kc", "vc"]
    if cfg["kind"] == "fp16" and "cos" in x:
        names += ["cos", "sin"]
    host = {n: x[n].detach().to("cpu").pin_memory() for n in names}
    dev = [{n: torch.empty_like(x[n]) for n in names} for _ in range(2)]
    out_dev = [torch.empty(x["q"].shape, dtype=torch.float16, device="cuda") for _ in range(2)]
    out_host = [torch.empty(x["q"].shape, dtype=torch.float16).pin_memory() for _ in range(2)]
    h2d = sum(t.numel() * t.element_size() for t in host.values())
    d2h = out_host[0].numel() * out_host[0].element_size()
    s_in, s_cmp, s_out = torch.cuda.Stream(), torch.cuda.Stream(), torch.cuda.Stream()
    ev = lambda: torch.cuda.Event()  # noqa: E731
    in_done, cmp_done, out_done = [ev(), ev()], [ev(), ev()], [ev(), ev()]
    used = [False, False]

    def step(i):
        b = i % 2
        d = dev[b]
        with torch.cuda.stream(s_in):
            if used[b]:
                s_in.wait_event(cmp_done[b])  # step i-2's attention has read these inputs
            for n in names:
                d[n].copy_(host[n], non_blocking=True)
            in_done[b].record(s_in)
        with torch.cuda.stream(s_cmp):
            s_cmp.wait_event(in_done[b])
            if used[b]:
                s_cmp.wait_event(out_done[b])  # step i-2's download has read out_dev[b]
            o = out_dev[b]
            if cfg["kind"] == "int8":
                o.copy_(R.flash_attn_int8qk(d["qi"], d["ki"], d["vi"], d["qsc"], d["ksc"], x["vs"]))
            elif cfg["kind"] == "decode":
                R.flash_attn_strided(d["q"], d["kc"].transpose(1, 2), d["vc"].transpose(1, 2), out=o)
            else:
                R.flash_attn_strided(d["q"], d["k"], d["v"], is_causal=cfg["causal"], window_size=cfg["window"],
                                     rot_cos=d.get("cos"), rot_sin=d.get("sin"), out=o)
            cmp_done[b].record(s_cmp)
        with torch.cuda.stream(s_out):
            s_out.wait_event(cmp_done[b])
            out_host[b].copy_(out_dev[b], non_blocking=True)
            out_done[b].record(s_out)
        used[b] = True

    for i in range(warmup):
        step(i)
    torch.cuda.synchronize()
    barrier(dist_on)
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record(s_in)
    for i in range(steps):
        step(warmup + i)
    s_in.wait_stream(s_out)
    end.record(s_in)
    torch.cuda.synchronize()
    barrier(dist_on)
    ms = start.elapsed_time(end)
    if dist_on:
        t = torch.tensor([ms], device="cuda", dtype=torch.float64)
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        ms = t.item()
    return ms, h2d, d2h


def time_e2e_sharded(cfg, x, steps, warmup, world, rank, chunks=1, sym=None):
    """N GPUs, end to end through the public API with host buffers: every step each
    rank copies its own units' Q/K/V (and the RoPE tables) in from pinned host
    memory, computes them, gathers O into every rank (with `sym`: the kernel's own
    peer stores into every rank's SymmetricOutput plus the ordering barrier;
    else an NCCL all-gather) and copies its own units' output back to pinned host
    memory.  Events on the current stream, max over ranks."""
    import rdnattention_b200 as R
    from rdnattention_b200 import multigpu as M

    shard = M.plan(cfg["B"], cfg["Hkv"], world, rank, interleave=sym is not None or chunks > 1)
    int8 = cfg["kind"] == "int8"
    G = cfg["H"] // cfg["Hkv"]
    qs, ks, vs = M.local_views(*(x[n] for n in (("qi", "ki", "vi") if int8 else ("q", "k", "v"))), shard)
    host = {"q": qs.contiguous().cpu().pin_memory(), "k": ks.contiguous().cpu().pin_memory(),
            "v": vs.contiguous().cpu().pin_memory()}
    if int8:
        bsl = slice(shard.b0, shard.b1, shard.bstep)
        host["qsc"] = x["qsc"][bsl, shard.g0 * G:shard.g1 * G].contiguous().cpu().pin_memory()
        host["ksc"] = x["ksc"][bsl, shard.g0:shard.g1].contiguous().cpu().pin_memory()
    rope = "cos" in x and cfg["kind"] == "fp16"
    if rope:
        host["cos"], host["sin"] = x["cos"].cpu().pin_memory(), x["sin"].cpu().pin_memory()
    dev = {n: torch.empty_like(t, device="cuda") for n, t in host.items()}
    out_local = torch.empty(host["q"].shape, dtype=torch.float16, device="cuda")
    out_host = torch.empty(out_local.shape, dtype=torch.float16).pin_memory()
    elems = shard.units() * G * cfg["S"] * cfg["D"]
    units = [M.plan(cfg["B"], cfg["Hkv"], world, r, interleave=chunks > 1) for r in range(world)]
    cap = max(u.units() for u in units) * G * cfg["S"] * cfg["D"]
    send = torch.zeros(cap, dtype=torch.float16, device="cuda")
    recv = torch.empty(world * cap, dtype=torch.float16, device="cuda")
    kw = dict(is_causal=cfg["causal"], window_size=cfg["window"]) if cfg["kind"] == "fp16" else {}
    h2d = sum(t.numel() * t.element_size() for t in host.values())
    d2h = out_host.numel() * out_host.element_size()

    def local(o, peers=None):
        if int8:
            R.flash_attn_int8qk_strided(dev["q"], dev["k"], dev["v"], dev["qsc"], dev["ksc"], x["vs"], out=o,
                                        peer_outputs=peers)
        else:
            R.flash_attn_strided(dev["q"], dev["k"], dev["v"], out=o, rot_cos=dev.get("cos"),
                                 rot_sin=dev.get("sin"), peer_outputs=peers, **kw)

    def step():
        for n in host:
            dev[n].copy_(host[n], non_blocking=True)
        if sym is not None:
            dst, _ = sym.next_slot()
            mine = dst[shard.b0:shard.b1:shard.bstep, shard.g0 * G:shard.g1 * G]
            if qs.numel():
                local(mine, sym.peer_addresses(mine))
            sym.order_stores()
            out_host.copy_(mine, non_blocking=True)
            return
        if qs.numel():
            local(out_local)
        send[:elems].copy_(out_local.reshape(-1))
        torch.distributed.all_gather_into_tensor(recv, send)
        out_host.copy_(out_local, non_blocking=True)

    for _ in range(warmup):
        step()
    ms = time_device(step, steps, 0, True)
    return ms, h2d, d2h


# ---------------------------------------------------------------- CPU baseline
def cpu_baseline(cfg, max_seconds=10.0):
    """The oracle port (fp32 torch on the host cores) on a bounded sample: whole query
    heads of the same workload (the heads of one KV group, repeated for the next
    groups: each head is the same amount of work), until ~max_seconds of CPU work or
    the whole workload."""
    from oracle import torch_oracle

    torch.set_num_threads(os.cpu_count() or 1)
    g = torch.Generator().manual_seed(0)
    B, H, Hkv, S, KS, D = 1, cfg["H"], cfg["Hkv"], cfg["S"], cfg["KS"], cfg["D"]
    G = H // Hkv
    q = torch.randn(1, G, S, D, generator=g).half()  # heads of kv group 0
    k = torch.randn(1, 1, KS, D, generator=g).half()
    v = torch.randn(1, 1, KS, D, generator=g).half()
    cos = sin = None
    if cfg["theta"]:
        pos = torch.arange(max(S, KS)).unsqueeze(1).float()
        inv = cfg["theta"] ** (-torch.arange(0, D, 2).float() / D)
        cos, sin = (pos * inv).cos(), (pos * inv).sin()
    from oracle.torch_oracle import flops as _fl

    done_units, heads = 0.0, 0
    total_heads = cfg["B"] * H
    t0 = time.perf_counter()
    while heads < total_heads and (heads == 0 or (time.perf_counter() - t0) < max_seconds):
        h = heads % G
        torch_oracle.attention(q, k, v, causal=cfg["causal"], window=cfg["window"], rot_cos=cos, rot_sin=sin,
                               heads=range(h, h + 1), row_chunk=CPU_ROW_CHUNK)
        heads += 1
    secs = time.perf_counter() - t0
    if cfg["kind"] == "decode":
        groups = (heads + G - 1) // G  # each KV group streams its K/V once for its G heads
        done_units = groups * 2 * KS * D * 2 + 2 * S * D * 2 * heads  # K/V + q/o bytes
        value = done_units / secs / 1e9
    else:
        done_units = _fl(1, heads, S, KS, D, cfg["causal"], cfg["window"])
        value = done_units / secs / 1e12
    return {"value": value, "unit": metric_of(cfg)[1], "cores": torch.get_num_threads(), "kind": "port",
            "sample": f"{heads} query head(s) of {total_heads} (S={S}, KS={KS}, D={D}), fp32 torch oracle "
                      f"(masked key columns skipped), {secs:.1f} s",
            "host_cpu_count": os.cpu_count()}


# ---------------------------------------------------------------- roofline
def load_peaks():
    """(bf16 burst TFLOP/s, bf16 sustained TFLOP/s, HBM GB/s, source)."""
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return (d.get("bf16_tflops", 1590.0), d.get("bf16_tflops_sustained", 1400.0), d.get("hbm_gbs", 6650.0),
                "measured")
    return 1590.0, 1400.0, 6650.0, "fallback"


def tensor_peak(kind, clocks):
    """(peak, burst, sustained, source, regime) of the tensor roofline: the measured
    burst figure for a short timed region, the sustained one when NVML reported
    sw_power_cap during it (the regime the sustained figure was measured in)."""
    peak_tc, peak_tc_sus, _, peak_src = load_peaks()
    if kind == "int8":
        burst, sus = load_int8_peak("burst"), load_int8_peak("sustained")
        src = "measured (profiles/int8_peak.txt, torch._int_mm)"
        if burst is None or sus is None:
            burst, sus, src = 2 * peak_tc, 2 * peak_tc_sus, f"{peak_src} (MEASURED_PEAKS.json bf16 x2)"
    else:
        burst, sus, src = peak_tc, peak_tc_sus, f"{peak_src} (MEASURED_PEAKS.json bf16)"
    capped = "sw_power_cap" in (clocks.get("reasons") or [])
    regime = ("sustained (sw_power_cap active during the timed region)" if capped
              else "burst (no power cap during the timed region)")
    return (sus if capped else burst), burst, sus, src, regime


# Nominal dense peaks of one B200 (spec sheet), reported beside the measured ones.
SPEC_PEAKS = {"fp16": 2250.0, "int8": 4500.0, "hbm": 8000.0}


def load_int8_peak(which="burst"):
    """INT8 tensor peak measured on this pool (profiles/int8_peak.txt, written from
    `python bench.py --measure-int8-peak`): which = "burst" or "sustained"; or None."""
    f = ROOT / "profiles" / "int8_peak.txt"
    if not f.exists():
        return None
    for line in f.read_text().splitlines():
        if line.startswith(f"int8_tops_{which}:"):
            try:
                return float(line.split(":", 1)[1].split()[0])
            except ValueError:
                return None
    return None


def measure_int8_peak():
    """torch._int_mm (cuBLASLt int8 x int8 -> int32) at 8192^3: best of 10 single
    launches (burst) and a 4 s back-to-back loop (sustained), 2 OP per MAC."""
    n = 8192
    a = torch.randint(-127, 128, (n, n), dtype=torch.int8, device="cuda")
    b = torch.randint(-127, 128, (n, n), dtype=torch.int8, device="cuda").t().contiguous().t()
    for _ in range(5):
        torch._int_mm(a, b)
    torch.cuda.synchronize()
    ops = 2.0 * n ** 3
    best = float("inf")
    for _ in range(10):
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        torch._int_mm(a, b)
        e.record()
        torch.cuda.synchronize()
        best = min(best, s.elapsed_time(e))
    iters = max(1, int(4000.0 / best))
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    sampler = ClockSampler(torch.cuda.current_device())
    with sampler:
        s.record()
        for _ in range(iters):
            torch._int_mm(a, b)
        e.record()
        torch.cuda.synchronize()
    sus = s.elapsed_time(e) / iters
    print(json.dumps({"int8_tops_burst": ops / best / 1e9, "int8_tops_sustained": ops / sus / 1e9,
                      "iters_sustained": iters, "clocks": sampler.summary(),
                      "how": "torch._int_mm int8 8192^3 (2*N^3 OP): best of 10 launches; back to back for 4 s"}))


def compare_cudnn():
    """This library's FP16 kernel against cuDNN's SDPA (torch.nn.functional.
    scaled_dot_product_attention restricted to the cuDNN backend) on the same box, same
    tensors, no RoPE (cuDNN has no in-kernel RoPE): the Llama-3-8B GQA prefill shape
    causal and not, and the MHA head_dim-64 shape of the INT8 workload."""
    import torch.nn.functional as F
    from torch.nn.attention import SDPBackend, sdpa_kernel

    import rdnattention_b200 as R

    def timed(fn, n=20, w=5):
        for _ in range(w):
            fn()
        torch.cuda.synchronize()
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        for _ in range(n):
            fn()
        e.record()
        torch.cuda.synchronize()
        return s.elapsed_time(e) / n

    rows = []
    for B, H, Hkv, S, D, causal in [(4, 32, 8, 4096, 128, True), (4, 32, 8, 4096, 128, False),
                                    (8, 16, 16, 2048, 64, False)]:
        g = torch.Generator(device="cuda").manual_seed(0)
        q = torch.randn(B, H, S, D, generator=g, device="cuda", dtype=torch.float16)
        k = torch.randn(B, Hkv, S, D, generator=g, device="cuda", dtype=torch.float16)
        v = torch.randn(B, Hkv, S, D, generator=g, device="cuda", dtype=torch.float16)
        fl = 4 * B * H * D * (S * (S + 1) / 2 if causal else S * S)
        ours = timed(lambda: R.flash_attn(q, k, v, is_causal=causal))
        row = {"shape": f"B{B} Hq{H} Hkv{Hkv} S{S} D{D} causal={causal}", "ours_ms": ours,
               "ours_tflops": fl / ours / 1e9}
        try:
            with sdpa_kernel(SDPBackend.CUDNN_ATTENTION):
                cd = timed(lambda: F.scaled_dot_product_attention(q, k, v, is_causal=causal, enable_gqa=Hkv != H))
            row.update(cudnn_ms=cd, cudnn_tflops=fl / cd / 1e9, cudnn_over_ours=ours / cd)
        except Exception as ex:  # the backend may be missing from a torch build
            row["cudnn"] = f"unavailable: {type(ex).__name__}: {str(ex)[:120]}"
        rows.append(row)
    sampler_dev = torch.cuda.current_device()
    print(json.dumps({"compare_cudnn": rows, "torch": torch.__version__,
                      "gpu": torch.cuda.get_device_name(sampler_dev)}))


def load_traffic(workload):
    """DRAM bytes per launch from a committed ncu summary (profiles/<kernel>_<workload>.txt)."""
    for f in (ROOT / "profiles").glob("*.txt"):
        txt = f.read_text()
        if f"workload: {workload}" not in txt:
            continue
        for line in txt.splitlines():
            if line.startswith("traffic_bytes_per_launch:"):
                try:
                    return float(line.split(":", 1)[1].strip())
                except ValueError:
                    return None
    return None


# ---------------------------------------------------------------- main
def run_reference(args, cfg, world):
    """CPU arm: the oracle port of the reference algorithm (the reference itself is
    HIP-only) on the host cores, one query head of the workload per step, masked
    key columns skipped before the matmul (so the CPU does about the visible-pair
    work the metric counts)."""
    from oracle import torch_oracle
    from oracle.torch_oracle import flops

    torch.set_num_threads(os.cpu_count() or 1)  # every host core (torchrun sets OMP_NUM_THREADS=1)
    metric, unit = metric_of(cfg)
    g = torch.Generator().manual_seed(0)
    S, KS, D, G = cfg["S"], cfg["KS"], cfg["D"], cfg["H"] // cfg["Hkv"]
    q = torch.randn(1, G, S, D, generator=g).half()
    k = torch.randn(1, 1, KS, D, generator=g).half()
    v = torch.randn(1, 1, KS, D, generator=g).half()
    cos = sin = None
    if cfg["theta"]:
        pos = torch.arange(max(S, KS)).unsqueeze(1).float()
        inv = cfg["theta"] ** (-torch.arange(0, D, 2).float() / D)
        cos, sin = (pos * inv).cos(), (pos * inv).sin()

    def one(i):
        h = i % G
        torch_oracle.attention(q, k, v, causal=cfg["causal"], window=cfg["window"], rot_cos=cos, rot_sin=sin,
                               heads=range(h, h + 1), row_chunk=CPU_ROW_CHUNK)

    for i in range(args.warmup):
        one(i)
    t0 = time.perf_counter()
    for i in range(args.steps):
        one(i)
    secs = time.perf_counter() - t0
    if cfg["kind"] == "decode":
        per = 2 * KS * D * 2 + 2 * S * D * 2
        value = per * args.steps / secs / 1e9
    else:
        per = flops(1, 1, S, KS, D, cfg["causal"], cfg["window"])
        value = per * args.steps / secs / 1e12
    sample = (f"one query head per step ({cfg['H'] * cfg['B']} in the workload), fp32 torch restatement of "
              "tests/accuracy.py dense_attention_reference + masks + RoPE, masked key columns skipped")
    line = {"impl": "reference", "metric": metric, "value": value, "unit": unit, "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": secs * 1e3 / max(args.steps, 1),
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
            "dtype": "fp32", "data": "synthetic",
            "config": config_dict(cfg, world, input_sets(cfg, world), args.gather),
            "sample_per_step": "one query head (fp32 torch oracle on the host cores)",
            "cpu_baseline": {"value": value, "unit": unit, "cores": torch.get_num_threads(), "kind": "port",
                             "sample": sample},
            "e2e": {"value": value, "unit": unit, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


CPU_ROW_CHUNK = 256  # query rows per CPU matmul: causal chunks skip the keys no row sees


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--config", default="2", choices=sorted(CONFIGS))
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--e2e-steps", type=int, default=None)
    ap.add_argument("--cpu-seconds", type=float, default=10.0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--batch", type=int, default=None, help="override the batch (profiling runs)")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--gather", choices=["fused", "nccl"], default="fused",
                    help="N>1: how every rank receives O: peer stores from the kernels' epilogue into a "
                         "SymmetricOutput (fused), or an NCCL all-gather after the kernel")
    ap.add_argument("--chunks", type=int, default=None,
                    help="N>1 with --gather nccl: pieces of the rank's units whose all-gathers overlap the next "
                         "piece's kernel (default: rdnattention_b200.multigpu.auto_chunks)")
    ap.add_argument("--measure-int8-peak", action="store_true",
                    help="measure the INT8 tensor peak (torch._int_mm) and exit")
    ap.add_argument("--compare-cudnn", action="store_true",
                    help="time the FP16 kernel against cuDNN SDPA on the same shapes and exit")
    args = ap.parse_args()
    if args.measure_int8_peak:
        measure_int8_peak()
        return
    if args.compare_cudnn:
        compare_cudnn()
        return
    cfg = dict(CONFIGS[args.config])
    if args.batch is not None:
        cfg["B"] = args.batch
        cfg["workload"] += f"_b{args.batch}"

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))

    if args.impl == "reference":
        if rank == 0:
            run_reference(args, cfg, world)
        return

    dist_on = world > 1
    from rdnattention_b200.multigpu import auto_chunks

    n_pieces = args.chunks or auto_chunks(cfg["B"], cfg["H"], cfg["S"], cfg["D"], world)
    torch.cuda.set_device(local)
    if dist_on:
        import datetime

        torch.distributed.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                             device_id=torch.device("cuda", local))
    import rdnattention_b200 as R

    R.library_path()  # fail loudly if the CUDA library is missing
    # Steps whose per-rank operands are smaller than L2 rotate through enough
    # independent input sets that each step's data was evicted by the two steps
    # before it (no L2 reuse across steps without a flush in the timed region).
    # Every rank holds the same full inputs (the sharded call's contract).
    n_sets = input_sets(cfg, world)
    xs = [make_inputs(cfg, "cuda", seed=1000 + 7919 * i) for i in range(n_sets)]
    x = xs[0]
    sampler = ClockSampler(local)
    per_step_units = work_units(cfg)
    scale = 1e9 if cfg["kind"] == "decode" else 1e12
    compute = None
    sym = None
    gather_used = args.gather if dist_on else None
    if not dist_on:
        fns = [step_fn(cfg, xi) for xi in xs]
        turn = itertools.cycle(fns)
        ms = time_device(lambda: next(turn)(), args.steps, args.warmup, dist_on, sampler)
        shard = None
    else:
        if args.gather == "fused":
            from rdnattention_b200.multigpu import SymmetricOutput, SymmetricOutputUnavailable

            try:
                sym = SymmetricOutput((cfg["B"], cfg["H"], cfg["S"], cfg["D"]))
                n_pieces = 1
            except SymmetricOutputUnavailable as ex:  # raised on every rank alike
                gather_used = f"nccl (the fused gather was unavailable: {str(ex)[:200]})"
        trip = [sharded_step_fns(cfg, xi, world, rank, n_pieces, sym) for xi in xs]
        shard = trip[0][2]
        turn = itertools.cycle([t[0] for t in trip])
        ms = time_device(lambda: next(turn)(), args.steps, args.warmup, dist_on, sampler)
        cturn = itertools.cycle([t[1] for t in trip])
        c_ms = time_device(lambda: next(cturn)(), args.steps, args.warmup, dist_on)
        units_rank = shard.units()
        compute = {"what": "the rank's own units alone (no all-gather), max over ranks",
                   "ms_per_step": c_ms / args.steps,
                   "value": per_step_units * args.steps / (c_ms / 1e3) / scale,
                   "units_per_rank_max": None, "units_rank0": units_rank}
        u = torch.tensor([units_rank], device="cuda", dtype=torch.int64)
        torch.distributed.all_reduce(u, op=torch.distributed.ReduceOp.MAX)
        compute["units_per_rank_max"] = int(u.item())
    # The roofline's kernel time: the attention kernel alone, from CUDA events the
    # library records right around its launch (not around the RoPE pre-pass), in a
    # separate pass of the same steps after the timed region (the event between the
    # pre-pass and the kernel would cost their overlap inside it).  N > 1: the
    # rank's own units (the compute-only step), max over ranks.
    k_turn = turn if not dist_on else cturn
    kernel_ms = R.debug_time_kernel(lambda: next(k_turn)(), repeats=max(5, min(args.steps, 20)))
    if dist_on:
        km = torch.tensor([kernel_ms], device="cuda", dtype=torch.float64)
        torch.distributed.all_reduce(km, op=torch.distributed.ReduceOp.MAX)
        kernel_ms = km.item()
    status = R.debug_read_status()
    value = per_step_units * args.steps / (ms / 1e3) / scale
    ms_step = ms / args.steps

    e2e = None
    if not args.no_e2e:
        e2e_steps = args.e2e_steps or max(3, min(args.steps, 20))
        if not dist_on:
            e2e_ms, h2d, d2h = time_e2e(cfg, x, e2e_steps, min(args.warmup, 3), dist_on)
        else:
            e2e_ms, h2d, d2h = time_e2e_sharded(cfg, x, e2e_steps, min(args.warmup, 3), world, rank, n_pieces, sym)
        e2e_value = per_step_units * e2e_steps / (e2e_ms / 1e3) / scale
        e2e = {"value": e2e_value, "unit": metric_of(cfg)[1], "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
               "steps": e2e_steps}

    if sym is not None:
        trip = None
        sym.close()
    if rank != 0:
        if dist_on:
            torch.distributed.destroy_process_group()
        return

    metric, unit = metric_of(cfg)
    _, _, peak_hbm, peak_src = load_peaks()
    # the roofline is the per-GPU attention kernel's (at N > 1 on the rank's own units)
    k_ms = kernel_ms
    k_units = per_step_units * (compute["units_per_rank_max"] / (cfg["B"] * cfg["Hkv"]) if compute else 1.0)
    clocks = sampler.summary()
    if cfg["kind"] == "decode":
        roof = {"bound": "hbm", "achieved": k_units / (k_ms / 1e3) / 1e9, "peak": peak_hbm, "unit": "GB/s"}
        roof["peak_source"] = f"{peak_src} (MEASURED_PEAKS.json copy)"
    else:
        peak, burst, sus, src, regime = tensor_peak(cfg["kind"], clocks)
        achieved = k_units / (k_ms / 1e3) / 1e12
        roof = {"bound": "tensor", "achieved": achieved, "peak": peak,
                "unit": "TOP/s" if cfg["kind"] == "int8" else "TFLOP/s"}
        roof["peak_regime"] = regime
        roof["frac_of_burst"] = achieved / burst
        roof["frac_of_sustained"] = achieved / sus
        roof["peak_source"] = src
    roof["frac"] = roof["achieved"] / roof["peak"]
    spec = SPEC_PEAKS["hbm" if cfg["kind"] == "decode" else cfg["kind"] if cfg["kind"] == "int8" else "fp16"]
    roof["spec_peak"] = spec
    roof["frac_of_spec"] = roof["achieved"] / spec
    roof["traffic"] = load_traffic(cfg["workload"])
    roof["algorithmic_bytes"] = algorithmic_bytes(cfg)
    roof["kernel_ms"] = kernel_ms
    roof["timing"] = ("attention kernel alone: CUDA events recorded by the library right around its launch "
                      "(rdna_debug_set_kernel_events), a pass of the same steps after the timed region")

    line = {
        "metric": metric, "value": value, "unit": unit, "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms_step, "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "int8" if cfg["kind"] == "int8" else "fp16", "data": "synthetic",
        "config": config_dict(cfg, world, n_sets, args.gather),
        "clocks": clocks,
        "e2e": e2e,
        # (fused gather: the attention launch(es) plus the barrier kernel per step)
        "gpu_launches": args.steps * (launches_per_step(cfg) * (n_pieces if dist_on else 1)
                                      + (1 if sym is not None else 0)),
        "roofline": roof,
        "kernel_status": list(status),
    }
    if compute:
        line["compute_only"] = compute
        line["gather"] = gather_used
        if sym is not None:
            line["step"] = ("flash_attn_sharded(out=SymmetricOutput): one launch per rank computes its units and "
                            "stores every O tile into all ranks' outputs over NVLink (peer stores from the kernel "
                            "epilogue), then a barrier kernel (epoch flags written over NVLink) orders the stores")
        else:
            line["step"] = ("flash_attn_sharded: the rank's units (one kernel per piece), each piece's NCCL "
                            f"all-gather of O into every rank overlapping the next piece ({n_pieces} piece(s))")
    if world == 1 and not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_baseline(cfg, args.cpu_seconds)
    print(json.dumps(line), flush=True)
    if dist_on:
        torch.distributed.destroy_process_group()


if __name__ == "__main__":
    main()
