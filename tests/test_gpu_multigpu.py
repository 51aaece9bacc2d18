"""flash_attn_sharded on all visible B200s (2 to 8): every rank computes its (batch, KV-head
group) units through the C ABI and receives the full O, which must match the
one-GPU kernel on the same inputs (max-abs <= 2e-3, the north-star FP16 gate)
for each gather layout — consecutive batch ranges (one piece), round-robin
batches (several pieces, per-batch and staged collectives), a KV-head split, an
uneven split and the decode KV cache viewed through strides — both with the
NCCL all-gather and with the gather fused into the kernels (SymmetricOutput:
NVLink peer stores from the epilogue of the prefill, two-pass INT8 and decode
kernels).  Skipped with fewer than two GPUs."""
import os
import socket
from datetime import timedelta

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu

WORLD = min(torch.cuda.device_count(), 8) if torch.cuda.is_available() else 0

# (name, B, H, Hkv, S, KS, D, causal, window, rope, kv_cache_layout, chunks)
CASES = [
    ("batch_block", 4, 8, 2, 512, 512, 128, True, -1, True, False, 1),
    ("round_robin", 8, 8, 2, 256, 256, 64, True, -1, False, False, 4),
    ("round_robin_staged", 8, 8, 2, 256, 256, 128, False, 128, False, False, 2),
    ("auto_pieces", 4, 32, 8, 1024, 1024, 128, True, -1, True, False, None),
    ("kv_head", 1, 16, 4, 384, 384, 128, True, -1, False, False, 2),
    ("decode_cache", 8, 64, 8, 1, 4096, 128, False, -1, False, True, None),
    ("uneven", 3, 8, 2, 200, 300, 64, False, -1, False, False, 1),
]


def _free_port():
    with socket.socket() as sk:
        sk.bind(("127.0.0.1", 0))
        return sk.getsockname()[1]


def _inputs(case, device):
    _, B, H, Hkv, S, KS, D, causal, window, rope, cache, _ = case
    g = torch.Generator().manual_seed(B * 7919 + KS)
    q = torch.randn(B, H, S, D, generator=g).half().to(device)
    if cache:
        k = torch.randn(B, KS, Hkv, D, generator=g).half().to(device).transpose(1, 2)
        v = torch.randn(B, KS, Hkv, D, generator=g).half().to(device).transpose(1, 2)
    else:
        k = torch.randn(B, Hkv, KS, D, generator=g).half().to(device)
        v = torch.randn(B, Hkv, KS, D, generator=g).half().to(device)
    kw = dict(is_causal=causal, window_size=window)
    if rope:
        inv = 1.0 / (10000.0 ** (torch.arange(0, D, 2, dtype=torch.float64) / D))
        ang = torch.arange(max(S, KS), dtype=torch.float64)[:, None] * inv[None, :]
        kw.update(rot_cos=ang.cos().float().to(device), rot_sin=ang.sin().float().to(device))
    return q, k, v, kw


def _worker(rank, port, queue):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=WORLD, timeout=timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    try:
        import rdnattention_b200 as R
        from rdnattention_b200.multigpu import SymmetricOutput, flash_attn_int8qk_sharded, flash_attn_sharded

        errs = {}
        for case in CASES:
            q, k, v, kw = _inputs(case, f"cuda:{rank}")
            got = flash_attn_sharded(q, k, v, chunks=case[-1], **kw)
            ref = R.flash_attn_strided(q, k, v, **kw)
            torch.cuda.synchronize()
            errs[case[0]] = (got.float() - ref.float()).abs().max().item()
            # the fused gather, twice on different inputs: the first result stays in its slot
            sym = SymmetricOutput(q.shape)
            got1 = flash_attn_sharded(q, k, v, out=sym, **kw)
            q2 = torch.flip(q, dims=(2,)).contiguous()
            got2 = flash_attn_sharded(q2, k, v, out=sym, **kw)
            ref2 = R.flash_attn_strided(q2, k, v, **kw)
            torch.cuda.synchronize()
            errs["fused_" + case[0]] = max((got1.float() - ref.float()).abs().max().item(),
                                           (got2.float() - ref2.float()).abs().max().item())
            sym.close()
        # INT8 (two-pass kernel at head_dim 128, one-pass at 64), per-token Q/K scales sliced
        # with each rank's units: the NCCL gather and the fused one
        for D in (64, 128):
            g = torch.Generator().manual_seed(D)
            B, H, Hkv, S = WORLD * 2, 8, 4, 384
            qi = torch.randint(-127, 128, (B, H, S, D), generator=g, dtype=torch.int8).to(rank)
            ki = torch.randint(-127, 128, (B, Hkv, S, D), generator=g, dtype=torch.int8).to(rank)
            vi = torch.randint(-127, 128, (B, Hkv, S, D), generator=g, dtype=torch.int8).to(rank)
            qsc = (torch.rand(B, H, S, generator=g) * 0.02 + 0.001).to(rank)
            ksc = (torch.rand(B, Hkv, S, generator=g) * 0.02 + 0.001).to(rank)
            ref = R.flash_attn_int8qk(qi, ki, vi, qsc, ksc, 0.01, is_causal=True)
            got = flash_attn_int8qk_sharded(qi, ki, vi, qsc, ksc, 0.01, is_causal=True)
            sym = SymmetricOutput(qi.shape)
            fused = flash_attn_int8qk_sharded(qi, ki, vi, qsc, ksc, 0.01, is_causal=True, out=sym)
            torch.cuda.synchronize()
            errs[f"int8_d{D}"] = (got.float() - ref.float()).abs().max().item()
            errs[f"fused_int8_d{D}"] = (fused.float() - ref.float()).abs().max().item()
            sym.close()
        errs["status"] = R.debug_read_status()
        queue.put((rank, errs))
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(WORLD < 2, reason="needs two CUDA devices")
def test_sharded_forward_on_every_gpu():
    ctx = mp.get_context("spawn")
    queue = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, port, queue)) for r in range(WORLD)]
    for p in procs:
        p.start()
    results = dict(queue.get(timeout=300) for _ in procs)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank, errs in results.items():
        assert errs.pop("status") == (0, 0), f"rank {rank}: a kernel recorded an expired wait"
        for name, err in errs.items():
            assert err <= 2e-3, (rank, name, err)
