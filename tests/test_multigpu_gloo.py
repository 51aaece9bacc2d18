"""Host logic of the (batch, KV-head group) sharding with world_size 2 on CPU
(gloo): the plan covers every unit exactly once, and flash_attn_sharded's
views + all-gather reassemble the full output.  The per-rank compute is the
CPU oracle here (the GPU kernels are covered by the gpu-marked tests)."""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from rdnattention_b200.multigpu import (SymmetricOutput, SymmetricOutputUnavailable, _uniform_axis, flash_attn_sharded,
                                        local_views, pieces, plan)


@pytest.mark.parametrize("B,Hkv,world", [(4, 8, 2), (1, 8, 2), (3, 2, 2), (1, 1, 2), (8, 8, 8), (2, 3, 4), (5, 8, 8),
                                         (3, 3, 8), (2, 2, 8), (4, 8, 8)])
def test_plan_covers_every_unit_once(B, Hkv, world):
    seen = torch.zeros(B, Hkv, dtype=torch.int32)
    for r in range(world):
        s = plan(B, Hkv, world, r)
        seen[s.b0:s.b1:s.bstep, s.g0:s.g1] += 1
    assert torch.equal(seen, torch.ones_like(seen))


@pytest.mark.parametrize("B,Hkv,world,busy", [(2, 3, 4, 4), (4, 8, 8, 8), (1, 8, 8, 8), (3, 2, 4, 4), (2, 2, 8, 4),
                                           (1, 1, 2, 1), (3, 3, 8, 6)])
def test_plan_keeps_ranks_busy(B, Hkv, world, busy):
    """Neither axis alone covering the ranks no longer idles them: both axes are split."""
    owned = [plan(B, Hkv, world, r) for r in range(world)]
    assert sum(s.units() > 0 for s in owned) == busy


@pytest.mark.parametrize("B,Hkv,world,interleave,axis", [
    (8, 8, 2, True, "batch"), (8, 8, 2, False, "batch_block"), (8, 8, 4, False, "batch_block"),
    (2, 8, 4, True, "kv_head"), (3, 2, 2, True, None), (2, 3, 4, True, None)])
def test_in_place_gather_layouts(B, Hkv, world, interleave, axis):
    """Which plans let the all-gathers write straight into O: interleaved batches (one
    collective per piece), consecutive batch ranges (one collective for all of O) and
    even KV-head ranges; uneven plans take the staged path."""
    shards = [plan(B, Hkv, world, r, interleave=interleave) for r in range(world)]
    assert _uniform_axis(shards, Hkv) == axis
    seen = torch.zeros(B, Hkv, dtype=torch.int32)
    for s in shards:
        seen[s.b0:s.b1:s.bstep, s.g0:s.g1] += 1
    assert torch.equal(seen, torch.ones_like(seen))


def test_local_views_are_strided_views():
    q = torch.randn(4, 8, 16, 64)
    k = torch.randn(4, 2, 16, 64)
    s = plan(4, 2, 2, 1)  # round robin: batches 1 and 3
    qs, ks, vs = local_views(q, k, k, s)
    assert qs.data_ptr() == q[1].data_ptr() and qs.stride(0) == 2 * q.stride(0) and qs.stride()[1:] == q.stride()[1:]
    assert ks.shape == (2, 2, 16, 64)
    s = plan(3, 2, 2, 1)  # uneven: consecutive ranges
    qs, _, _ = local_views(q[:3], k[:3], k[:3], s)
    assert qs.data_ptr() == q[2].data_ptr() and qs.shape[0] == 1


def _free_port():
    with socket.socket() as sk:
        sk.bind(("127.0.0.1", 0))
        return sk.getsockname()[1]


def _worker(rank, world, port, shape, causal, window, queue, chunks=1):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from oracle import torch_oracle

        B, H, Hkv, S, D = shape
        g = torch.Generator().manual_seed(0)  # every rank holds the same full inputs
        q = torch.randn(B, H, S, D, generator=g).half()
        k = torch.randn(B, Hkv, S, D, generator=g).half()
        v = torch.randn(B, Hkv, S, D, generator=g).half()

        def compute(qs, ks, vs, out=None, **kw):
            o = torch_oracle.attention(qs, ks, vs, causal=kw["is_causal"], window=kw["window_size"]).half()
            if out is not None:
                out.copy_(o)
            return o

        out = flash_attn_sharded(q, k, v, is_causal=causal, window_size=window, compute=compute, chunks=chunks)
        ref = torch_oracle.attention(q, k, v, causal=causal, window=window).half()
        queue.put((rank, torch.equal(out, ref)))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("shape,causal,window", [((4, 8, 2, 24, 32), True, -1), ((1, 8, 4, 17, 32), False, 8),
                                                  ((3, 4, 1, 9, 32), True, 4)])
def test_sharded_forward_gathers_full_output(shape, causal, window):
    ctx = mp.get_context("spawn")
    queue = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, shape, causal, window, queue)) for r in range(2)]
    for p in procs:
        p.start()
    results = dict(queue.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert results == {0: True, 1: True}


@pytest.mark.parametrize("B,Hkv,world,chunks", [(4, 8, 2, 2), (3, 2, 2, 2), (1, 8, 2, 3), (2, 3, 4, 4), (5, 8, 8, 3)])
def test_pieces_cover_each_shard_once(B, Hkv, world, chunks):
    seen = torch.zeros(B, Hkv, dtype=torch.int32)
    for r in range(world):
        for p in pieces(plan(B, Hkv, world, r), chunks):
            seen[p.b0:p.b1:p.bstep, p.g0:p.g1] += 1
    assert torch.equal(seen, torch.ones_like(seen))


@pytest.mark.parametrize("shape,causal,window,chunks", [
    ((4, 8, 2, 24, 32), True, -1, 2),   # batch axis, even pieces
    ((3, 4, 1, 9, 32), True, 4, 2),     # batch axis: rank 1's second piece is empty (padded send)
    ((1, 8, 4, 17, 32), False, 8, 3),   # KV-head axis, uneven pieces
    ((4, 8, 2, 24, 32), False, -1, 3),  # a piece empty on every rank (skipped by all)
    ((8, 4, 2, 9, 32), True, -1, 2),    # round robin, two batch elements per piece: one staged collective each
    ((8, 4, 2, 9, 32), False, -1, None),  # the automatic piece count
])
def test_sharded_forward_overlapped_pieces(shape, causal, window, chunks):
    ctx = mp.get_context("spawn")
    queue = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, shape, causal, window, queue, chunks)) for r in range(2)]
    for p in procs:
        p.start()
    results = dict(queue.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert results == {0: True, 1: True}


@pytest.mark.parametrize("shape,world,chunks", [
    ((2, 8, 4, 9, 32), 4, 2),   # KV-head split (batch < ranks): per-batch in-place gathers, two pieces
    ((8, 4, 2, 9, 32), 4, 2),   # round-robin batch split, two batches per rank, two pieces
    ((8, 4, 2, 9, 32), 4, 1),   # consecutive batch ranges, one piece: one in-place gather of all of O
])
def test_sharded_forward_in_place_on_four_ranks(shape, world, chunks):
    """The in-place all-gathers with several ranks and pieces reassemble the full output."""
    ctx = mp.get_context("spawn")
    queue = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, shape, True, -1, queue, chunks)) for r in range(world)]
    for p in procs:
        p.start()
    results = dict(queue.get(timeout=180) for _ in procs)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert results == {r: True for r in range(world)}


def test_symmetric_output_slots_and_peer_addresses():
    """The fused gather's host bookkeeping (no GPU: the object is assembled over a
    host buffer): slots are used in turn, and a view of this rank's slot maps to the
    same offset in every peer's allocation."""
    shape = (2, 4, 8, 16)
    n = 2 * 4 * 8 * 16
    buf = torch.empty(2 * n, dtype=torch.float16)
    so = SymmetricOutput.__new__(SymmetricOutput)
    so._base = buf.data_ptr()
    so.slot_bytes = n * 2
    so.slots = [buf[:n].view(shape), buf[n:].view(shape)]
    so._turn = 0
    so._peer_bases = [1 << 40, 3 << 40]
    first, off0 = so.next_slot()
    second, off1 = so.next_slot()
    third, _ = so.next_slot()
    assert first.data_ptr() == buf.data_ptr() and off0 == 0
    assert second.data_ptr() == buf.data_ptr() + n * 2 and off1 == n * 2
    assert third.data_ptr() == first.data_ptr()
    view = second[1::2, 2:4]  # a rank's round-robin units of two KV heads
    off = view.data_ptr() - buf.data_ptr()
    assert so.peer_addresses(view) == [(1 << 40) + off, (3 << 40) + off]
    with pytest.raises(ValueError):
        so.peer_addresses(torch.empty(4, dtype=torch.float16))


def _int8_worker(rank, world, port, shape, chunks, queue):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from oracle import c_oracle

        B, H, Hkv, S, D = shape
        g = torch.Generator().manual_seed(5)  # every rank holds the same full inputs
        qi = torch.randint(-127, 128, (B, H, S, D), generator=g, dtype=torch.int8)
        ki = torch.randint(-127, 128, (B, Hkv, S, D), generator=g, dtype=torch.int8)
        vi = torch.randint(-127, 128, (B, Hkv, S, D), generator=g, dtype=torch.int8)
        qsc = torch.rand(B, H, S, generator=g) * 0.02 + 0.001
        ksc = torch.rand(B, Hkv, S, generator=g) * 0.02 + 0.001

        def compute(q, k, v, out=None, q_side=None, kv_side=None, **kw):
            # the shard's own per-token scales arrive sliced like its Q and K
            assert q_side.shape == q.shape[:3] and kv_side.shape == k.shape[:3]
            o = c_oracle.attention_int8(q, k, v, q_side.contiguous(), kv_side.contiguous(), 0.01,
                                        causal=kw["is_causal"]).half()
            if out is not None:
                out.copy_(o)
            return o

        got = flash_attn_sharded(qi, ki, vi, is_causal=True, compute=compute, chunks=chunks, q_side=qsc,
                                 kv_side=ksc)
        ref = c_oracle.attention_int8(qi, ki, vi, qsc, ksc, 0.01, causal=True).half()
        queue.put((rank, got.dtype == torch.float16 and torch.equal(got, ref)))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("shape,world,chunks", [
    ((4, 4, 2, 24, 32), 2, 1),   # consecutive batch ranges
    ((4, 4, 2, 24, 32), 2, 2),   # round robin in two pieces
    ((1, 8, 4, 17, 32), 2, 1),   # KV-head split: the scales' head axis is sliced too
    ((3, 4, 2, 9, 32), 2, 1),    # uneven: staged gather
])
def test_int8_sharded_slices_the_per_token_scales(shape, world, chunks):
    """INT8 sharding: each rank's compute receives its units' per-token Q/K
    scales (q_side / kv_side sliced like Q and K) and the gathered float16
    output equals the single-device oracle."""
    ctx = mp.get_context("spawn")
    queue = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_int8_worker, args=(r, world, port, shape, chunks, queue)) for r in range(world)]
    for p in procs:
        p.start()
    results = dict(queue.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert results == {r: True for r in range(world)}


def _agree_worker(rank, world, port, failing, queue):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        so = SymmetricOutput.__new__(SymmetricOutput)
        so.group, so.world, so.rank = None, world, rank
        so.device = torch.device("cpu")
        so._base, so._peer_bases = None, []
        why = f"no IPC here (rank {rank})" if rank in failing else None
        try:
            so._agree(why)
            queue.put((rank, "ok"))
        except SymmetricOutputUnavailable as ex:
            queue.put((rank, str(ex)))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("failing", [(), (1,), (0, 2)])
def test_symmetric_output_fails_on_every_rank_alike(failing):
    """A SymmetricOutput that cannot be set up on one rank fails on all of them,
    with every failing rank's reason, so the ranks' collectives never diverge."""
    world = 3
    ctx = mp.get_context("spawn")
    queue = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_agree_worker, args=(r, world, port, failing, queue)) for r in range(world)]
    for p in procs:
        p.start()
    results = dict(queue.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    if not failing:
        assert set(results.values()) == {"ok"}
    else:
        want = "; ".join(f"no IPC here (rank {r})" for r in failing)
        assert all(v == want for v in results.values()), results


def test_sharded_argument_checks_and_single_rank():
    """One-rank group (gloo, in this process): a SymmetricOutput of the wrong shape and
    chunks < 1 are rejected before any work, and a single rank computes everything."""
    from oracle import torch_oracle

    store = dist.TCPStore("127.0.0.1", _free_port(), 1, True)
    dist.init_process_group("gloo", store=store, rank=0, world_size=1)
    try:
        g = torch.Generator().manual_seed(3)
        q = torch.randn(2, 4, 9, 32, generator=g).half()
        k = torch.randn(2, 2, 9, 32, generator=g).half()

        def compute(qs, ks, vs, out=None, **kw):
            o = torch_oracle.attention(qs, ks, vs, causal=kw["is_causal"], window=kw["window_size"]).half()
            if out is not None:
                out.copy_(o)
            return o

        wrong = SymmetricOutput.__new__(SymmetricOutput)
        wrong.shape, wrong.world, wrong.rank = (2, 4, 9, 16), 1, 0
        with pytest.raises(ValueError):
            flash_attn_sharded(q, k, k, compute=compute, out=wrong)
        with pytest.raises(ValueError):
            flash_attn_sharded(q, k, k, compute=compute, chunks=0)
        got = flash_attn_sharded(q, k, k, is_causal=True, compute=compute)
        assert torch.equal(got, torch_oracle.attention(q, k, k, causal=True).half())
    finally:
        dist.destroy_process_group()
