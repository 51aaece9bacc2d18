"""(batch, KV-head group) sharding of the forward across the GPUs of one node.

The units of work — a batch element together with one KV head and the G
query heads that read it — are independent, so each rank computes its own
units and every rank receives the full output O.  Two ways to assemble O:

* fused (``out=SymmetricOutput(...)``): every rank's output buffer is mapped
  into every other rank's process (CUDA IPC), and the attention kernels store
  each finished O tile into all ranks' buffers over NVLink from their
  epilogue (TMA stores, one tensor map per peer), so the gather overlaps the
  tiles still being computed; a small
  barrier kernel (epoch flags written over NVLink) then orders the peers'
  stores before anything that reads O;
* NCCL: the rank's units are computed into its block of O and NCCL
  all-gathers the blocks (in place when the plan allows, in pieces that
  overlap the next piece's kernel).

Shards are strided views of the full tensors (base-pointer offsets, original
strides), so nothing is repacked.

The reference library is single-device; this module is the multi-GPU layer
the B200 build adds around its C ABI.
"""
from dataclasses import dataclass
from typing import Callable, Optional

import torch
import torch.distributed as dist


@dataclass(frozen=True)
class Shard:
    """The block of units a rank owns: batches b0, b0 + bstep, ... (< b1) x KV heads [g0, g1)."""
    axis: str  # "batch" or "kv_head"
    b0: int
    b1: int
    g0: int
    g1: int
    bstep: int = 1

    @property
    def batches(self):
        return range(self.b0, self.b1, self.bstep)

    def units(self) -> int:
        return len(self.batches) * (self.g1 - self.g0)


def _split(n: int, world: int, rank: int):
    base, extra = divmod(n, world)
    start = rank * base + min(rank, extra)
    return start, start + base + (1 if rank < extra else 0)


def plan(batch: int, kv_heads: int, world: int, rank: int, interleave: bool = True) -> Shard:
    """The rank's (batch, KV-head) units.  Batch-major when every rank gets whole batch
    elements (batch >= world): with `interleave`, round robin (rank r takes batches r,
    r + world, ...) when they divide evenly, so that the c-th batch of every rank forms
    one contiguous block of O in rank order (a step in several pieces gathers each piece
    in place); else consecutive ranges (rank r's block of O is contiguous and in rank
    order, so a step in one piece gathers the whole O in place at once).  Otherwise KV-head groups when they cover
    the ranks (kv_heads >= world); otherwise a grid of wb x wg ranks splits both axes,
    chosen to keep the most ranks busy and then to balance the units per rank (B=2, Hkv=3
    on 4 ranks: 2 x 2).  Uneven counts give the first ranks one more unit; ranks outside
    the grid (fewer units than ranks) own nothing."""
    if not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside world of {world}")
    if batch >= world:
        if interleave and batch % world == 0 and world > 1:
            return Shard("batch", rank, batch, 0, kv_heads, bstep=world)
        b0, b1 = _split(batch, world, rank)
        return Shard("batch", b0, b1, 0, kv_heads)
    if kv_heads >= world:
        g0, g1 = _split(kv_heads, world, rank)
        return Shard("kv_head", 0, batch, g0, g1)
    best = None
    for wb in range(1, min(batch, world) + 1):
        wg = min(kv_heads, world // wb)
        busy = wb * wg
        cost = -(-batch // wb) * -(-kv_heads // wg)
        key = (-busy, cost, -wb)
        if best is None or key < best[0]:
            best = (key, wb, wg)
    _, wb, wg = best
    if rank >= wb * wg:
        return Shard("batch", 0, 0, 0, 0)
    b0, b1 = _split(batch, wb, rank // wg)
    g0, g1 = _split(kv_heads, wg, rank % wg)
    return Shard("batch" if b1 - b0 > 1 else "kv_head", b0, b1, g0, g1)


def local_views(q, k, v, shard: Shard):
    """Strided views of the rank's units (no copies)."""
    G = q.shape[1] // k.shape[1]
    b = slice(shard.b0, shard.b1, shard.bstep)
    qs = q[b, shard.g0 * G:shard.g1 * G]
    ks = k[b, shard.g0:shard.g1]
    vs = v[b, shard.g0:shard.g1]
    return qs, ks, vs


def pieces(shard: Shard, chunks: int):
    """The shard split into `chunks` consecutive pieces along its own axis (some may
    be empty), in the order their outputs are all-gathered."""
    out = []
    for c in range(chunks):
        if shard.axis == "batch":
            n = len(shard.batches)
            lo, hi = _split(n, chunks, c)
            b0 = shard.b0 + lo * shard.bstep
            b1 = min(shard.b1, shard.b0 + hi * shard.bstep) if hi > lo else b0
            out.append(Shard("batch", b0, b1, shard.g0, shard.g1, shard.bstep))
        else:
            lo, hi = _split(shard.g1 - shard.g0, chunks, c)
            out.append(Shard("kv_head", shard.b0, shard.b1, shard.g0 + lo, shard.g0 + hi))
    return out


def _default_compute(q, k, v, out=None, peer_outputs=None, **kw):
    from . import flash_attn_strided

    return flash_attn_strided(q, k, v, out=out, peer_outputs=peer_outputs, **kw)


def _uniform_axis(shards, kv_heads: int):
    """How the plan lets every all-gather run in place: "batch" when rank r owns batches
    r, r + world, ... (so the c-th batch of every rank is one contiguous block of O in
    rank order), "batch_block" when rank r owns the r-th equal range of batches (its
    block of O is contiguous and in rank order), "kv_head" when rank r owns the r-th
    equal range of KV heads of every batch (each batch's block of O is contiguous in
    rank order); else None."""
    world = len(shards)
    first = shards[0]
    if first.units() == 0:
        return None
    whole_heads = all(s.g0 == 0 and s.g1 == kv_heads for s in shards)
    nb = len(first.batches)
    if whole_heads and all(s.bstep == world and s.b0 == r and len(s.batches) == nb for r, s in enumerate(shards)):
        return "batch"
    if whole_heads and all(s.bstep == 1 and s.b0 == r * nb and s.b1 == (r + 1) * nb for r, s in enumerate(shards)):
        return "batch_block"
    ng = first.g1 - first.g0
    if all(s.bstep == 1 and s.b0 == first.b0 and s.b1 == first.b1 and s.g1 - s.g0 == ng and s.g0 == r * ng
           for r, s in enumerate(shards)):
        return "kv_head"
    return None


# O bytes per batch element from which one piece (and one in-place all-gather) per batch
# element pays: below it the collectives' fixed cost dominates (a decode step's O)
AUTO_PIECE_BYTES = 4 << 20


def auto_chunks(batch: int, heads: int, seq: int, head_dim: int, world: int, elem_bytes: int = 2) -> int:
    """Pieces flash_attn_sharded uses with chunks=None: two when each rank holds at least
    two batch elements' worth of a large O (so the first piece's all-gather overlaps the
    second piece's kernel), else one."""
    per_batch = heads * seq * head_dim * elem_bytes
    local = batch // world if batch >= world else batch
    return 2 if per_batch >= AUTO_PIECE_BYTES and local >= 2 else 1


class SymmetricOutputUnavailable(RuntimeError):
    """Raised on every rank when a SymmetricOutput cannot be set up on some rank."""


class _DeviceArray:
    """A raw device allocation seen through __cuda_array_interface__ (torch.as_tensor)."""

    def __init__(self, ptr: int, shape, typestr: str):
        self.__cuda_array_interface__ = {"shape": tuple(shape), "typestr": typestr, "data": (ptr, False),
                                         "version": 3, "strides": None}


class SymmetricOutput:
    """Output buffers of one shape on every rank of `group`, each mapped into
    every other rank's process (CUDA IPC), for flash_attn_sharded(out=...): the
    kernels store each O tile into every rank's copy over NVLink, the
    all-gather fused into the attention epilogue.

    Collective: every rank constructs it with the same shape (on its current
    CUDA device) and calls close() together.  Construction fails on every rank
    alike (SymmetricOutputUnavailable, after undoing what succeeded) when any
    rank cannot allocate or map the buffers, so callers can fall back to the
    NCCL gather without the ranks' collectives diverging.  `slots` buffers are used in turn,
    one per call: the tensor a call returns holds the result until this rank
    makes its next call with this object (consume or copy it, on the current
    stream, before then); other ranks' next kernels only write the following
    slot."""

    def __init__(self, shape, dtype=torch.float16, group=None, slots: int = 2):
        import rdnattention_b200 as R

        if dtype != torch.float16:
            raise ValueError("the fused gather writes float16 outputs")
        if slots < 2:
            raise ValueError("slots must be >= 2 (a rank's next kernel writes the other slot)")
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        if self.world - 1 > R.MAX_PEER_OUTPUTS:
            raise ValueError(f"at most {R.MAX_PEER_OUTPUTS + 1} ranks")
        self.shape = tuple(int(x) for x in shape)
        self.dtype = dtype
        self.device = torch.device("cuda", torch.cuda.current_device())
        n = 1
        for x in self.shape:
            n *= x
        self.slot_bytes = (n * 2 + 255) // 256 * 256
        flags_off = self.slot_bytes * slots  # then one flag word per rank (the barrier's epochs)
        self._base = None
        self._peer_bases = []  # the other ranks' allocations, in rank order
        handle, why = bytes(R.IPC_HANDLE_BYTES), None
        try:
            with torch.cuda.device(self.device):
                self._base, handle = R._ipc_alloc(flags_off + 256)
            self._flags = torch.as_tensor(_DeviceArray(self._base + flags_off, (self.world,), "<i4"),
                                          device=self.device)
            self._flags.zero_()  # before the handles go out: no peer signals before it has them
        except Exception as ex:  # noqa: BLE001 - reported collectively below
            why = f"allocation failed on rank {self.rank}: {ex}"
        self._epoch = 0
        # every rank takes part in the exchange, whether or not its allocation succeeded
        mine = torch.frombuffer(bytearray(handle), dtype=torch.uint8).to(self.device)
        every = torch.empty(self.world * R.IPC_HANDLE_BYTES, dtype=torch.uint8, device=self.device)
        dist.all_gather_into_tensor(every, mine, group=group)
        self._agree(why)
        every = every.cpu().numpy().tobytes()
        try:
            with torch.cuda.device(self.device):
                for r in range(self.world):
                    if r != self.rank:
                        h = every[r * R.IPC_HANDLE_BYTES:(r + 1) * R.IPC_HANDLE_BYTES]
                        self._peer_bases.append(R._ipc_open(h))
        except Exception as ex:  # noqa: BLE001 - reported collectively below
            why = f"mapping a peer's buffer failed on rank {self.rank}: {ex}"
        self._agree(why)
        self._peer_flags = [b + flags_off for b in self._peer_bases]
        self.slots = [torch.as_tensor(_DeviceArray(self._base + i * self.slot_bytes, self.shape, "<f2"),
                                      device=self.device) for i in range(slots)]
        self._turn = 0

    def _agree(self, why):
        """Collective success check: if any rank failed, every rank undoes what it
        holds and raises SymmetricOutputUnavailable (the failing ranks' reasons)."""
        import rdnattention_b200 as R

        ok = torch.tensor([0 if why else 1], dtype=torch.int32, device=self.device)
        dist.all_reduce(ok, op=dist.ReduceOp.MIN, group=self.group)
        if int(ok.item()) == 1:
            return
        reasons = [None] * self.world
        dist.all_gather_object(reasons, why, group=self.group)
        for b in self._peer_bases:
            with torch.cuda.device(self.device):
                R._ipc_close(b)
        self._peer_bases = []
        dist.barrier(group=self.group)  # nobody maps this rank's buffer any more
        if self._base is not None:
            with torch.cuda.device(self.device):
                R._ipc_free(self._base)
            self._base = None
        raise SymmetricOutputUnavailable("; ".join(r for r in reasons if r))

    def next_slot(self):
        """The slot the next call writes, and its offset in every allocation."""
        i = self._turn
        self._turn = (self._turn + 1) % len(self.slots)
        return self.slots[i], i * self.slot_bytes

    def peer_addresses(self, view) -> list:
        """Addresses, in the other ranks' buffers, of the elements `view` (a view of
        one of this rank's slots) covers here."""
        off = view.data_ptr() - self._base
        if not 0 <= off < self.slot_bytes * len(self.slots):
            raise ValueError("view is not inside this SymmetricOutput")
        return [b + off for b in self._peer_bases]

    def order_stores(self):
        """Stream-ordered barrier (a one-block kernel over peer flag words): work
        queued after it on the current stream runs once every rank's kernels
        before it (and their peer stores) have completed.  Every rank calls it
        once per call of the fused path, in the same order."""
        import rdnattention_b200 as R

        self._epoch += 1
        R._peer_barrier(self.world, self.rank, self._peer_flags, self._flags.data_ptr(), self._epoch, self.device)

    def close(self):
        """Collective: unmaps the peers' buffers and frees this rank's."""
        import rdnattention_b200 as R

        if self._base is None:
            return
        torch.cuda.synchronize(self.device)
        dist.barrier(group=self.group)
        with torch.cuda.device(self.device):
            for b in self._peer_bases:
                R._ipc_close(b)
        self._peer_bases = []
        self._peer_flags = []
        self.slots = []
        self._flags = None
        dist.barrier(group=self.group)  # nobody maps this rank's buffer any more
        with torch.cuda.device(self.device):
            R._ipc_free(self._base)
        self._base = None


def flash_attn_sharded(query, key, value, is_causal: bool = False, window_size: int = -1, rot_cos=None,
                       rot_sin=None, group=None, compute: Optional[Callable] = None, chunks: Optional[int] = 1,
                       out: Optional[SymmetricOutput] = None, q_side=None, kv_side=None):
    """Forward attention over all ranks of `group`: every rank passes the same full
    [B, H, S, D] / [B, Hkv, KS, D] inputs, computes only its (batch, KV-head) units
    and receives the full output.  `compute(q, k, v, out=..., is_causal=...,
    window_size=..., rot_cos=..., rot_sin=...)` replaces the local kernel call
    (default: the sm_100a path through the C ABI); with `out` it also receives
    `peer_outputs`, and `q_side` / `kv_side` when given.

    When the plan splits one axis evenly (the usual case), each rank writes its
    units straight into its block of the result and the all-gathers run in place
    (`compute` is then called with an `out=` view to fill).  `chunks` > 1 computes
    the rank's units in that many pieces (of batch elements) and starts each
    piece's all-gathers (asynchronous, on the collective's own stream) as soon as
    the piece is enqueued, so the transfer of piece c overlaps the kernel of piece
    c + 1 (a batch split is then round robin, and a piece holding several batch
    elements of it is gathered through a staging buffer in one collective).  With
    one piece a batch split takes consecutive ranges and a single in-place
    all-gather.  chunks=None picks the count from O's size (auto_chunks).
    Uneven plans gather pieces into a staging buffer and copy them into place;
    every rank takes the same collective steps (pieces that are empty on some
    ranks are padded).

    With `out` (a SymmetricOutput of O's shape on `group`) the gather is fused
    into the kernels: one launch computes the rank's units and stores every O
    tile into all ranks' buffers over NVLink, then the barrier kernel orders
    those stores before what follows on the stream; `chunks` does not apply.
    Returns the slot of `out` the call wrote.

    `q_side` / `kv_side`: per-row companions of the query / key tensors (e.g. the
    INT8 per-token scales, [B, H, S] / [B, Hkv, KS]), sliced with each shard like
    them and passed to `compute` under those names; scalars pass through.  The
    output is float16 whatever the input type."""
    world = dist.get_world_size(group)
    rank = dist.get_rank(group)
    B, H, S, D = query.shape
    odt = torch.float16
    Hkv = key.shape[1]
    G = H // Hkv
    compute = compute or _default_compute

    def run(piece, out_view=None, peers=None):
        """The local kernel call for one rectangle of units."""
        qs, ks, vs = local_views(query, key, value, piece)
        kw = dict(is_causal=is_causal, window_size=window_size, rot_cos=rot_cos, rot_sin=rot_sin)
        bsl = slice(piece.b0, piece.b1, piece.bstep)
        if q_side is not None:
            kw["q_side"] = q_side[bsl, piece.g0 * G:piece.g1 * G] if torch.is_tensor(q_side) else q_side
        if kv_side is not None:
            kw["kv_side"] = kv_side[bsl, piece.g0:piece.g1] if torch.is_tensor(kv_side) else kv_side
        if peers is not None:
            kw["peer_outputs"] = peers
        return compute(qs, ks, vs, out=out_view, **kw)

    if out is not None:
        if tuple(out.shape) != (B, H, S, D):
            raise ValueError(f"out has shape {out.shape}, the output is {(B, H, S, D)}")
        if out.world != world or out.rank != rank:
            raise ValueError("out was built on another process group")
        me = plan(B, Hkv, world, rank)
        dst, _ = out.next_slot()
        if me.units():
            mine = dst[me.b0:me.b1:me.bstep, me.g0 * G:me.g1 * G]
            run(me, mine, out.peer_addresses(mine))
        out.order_stores()
        return dst
    if chunks is None:
        chunks = auto_chunks(B, H, S, D, world, 2)
    if chunks < 1:
        raise ValueError("chunks must be >= 1")
    shards = [plan(B, Hkv, world, r, interleave=chunks > 1) for r in range(world)]
    axis = _uniform_axis(shards, Hkv)
    if axis == "batch_block":
        # One piece, consecutive batch ranges: the rank fills its contiguous block of O
        # and one in-place all-gather assembles the rest around it.
        out = torch.empty(B, H, S, D, dtype=odt, device=query.device)
        me = shards[rank]
        mine = out[me.b0:me.b1]
        run(me, mine)
        dist.all_gather_into_tensor(out.view(-1), mine.view(-1), group=group)
        return out
    if axis is not None:
        # In place: the rank writes its units straight into its block of O and NCCL
        # gathers the blocks around it, one collective per batch element (the c-th
        # batch of every rank for a round-robin batch split, the rank's KV heads of
        # that batch for a KV-head split: contiguous in rank order either way), with no
        # staging buffer and no reassembly copy.  The rank's units run in `chunks`
        # pieces of batch elements; each piece's collectives (asynchronous, on NCCL's
        # stream) overlap the next piece's kernel.
        out = torch.empty(B, H, S, D, dtype=odt, device=query.device)
        me = shards[rank]
        h0, h1 = me.g0 * G, me.g1 * G
        nb = len(me.batches) if axis == "batch" else B
        works, staged = [], []
        for c in range(min(chunks, nb)):
            lo, hi = _split(nb, min(chunks, nb), c)
            if axis == "batch":
                piece = Shard("batch", me.b0 + lo * world, me.b0 + hi * world, me.g0, me.g1, world)
            else:
                piece = Shard("kv_head", lo, hi, me.g0, me.g1)
            mine = out[piece.b0:piece.b1:piece.bstep, h0:h1]
            run(piece, mine)
            if axis == "batch" and len(piece.batches) > 1:
                # several batch elements of every rank, interleaved in O: one staged
                # collective (cheap when O per batch element is small, e.g. decode)
                n = len(piece.batches)
                recv = torch.empty((world, n) + tuple(mine.shape[1:]), dtype=out.dtype, device=out.device)
                send = mine.contiguous()
                works.append(dist.all_gather_into_tensor(recv.view(-1), send.view(-1), group=group, async_op=True))
                c0 = piece.b0 - rank
                staged.append((send, out[c0:c0 + n * world].view(n, world, *out.shape[1:]), recv))
                continue
            for b in piece.batches:
                if axis == "batch":
                    whole = out[b - rank:b - rank + world]  # the c-th batch of every rank
                    works.append(dist.all_gather_into_tensor(whole.reshape(-1), out[b].reshape(-1), group=group,
                                                             async_op=True))
                else:
                    works.append(dist.all_gather_into_tensor(out[b].view(-1), out[b, h0:h1].reshape(-1),
                                                             group=group, async_op=True))
        for w in works:
            w.wait()
        for _, dst, recv in staged:
            dst.copy_(recv.transpose(0, 1))
        return out
    per_rank = [pieces(s, chunks) for s in shards]

    def elems(s: Shard):
        return s.units() * G * S * D

    gathered = []
    works = []
    for c in range(chunks):
        sizes = [elems(per_rank[r][c]) for r in range(world)]
        cap = max(sizes)  # every rank contributes the same number of elements
        if cap == 0:
            continue
        send = torch.zeros(cap, dtype=odt, device=query.device) if sizes[rank] < cap else None
        if sizes[rank] > 0:
            o_local = run(per_rank[rank][c]).reshape(-1)
            if send is None:
                send = o_local
            else:
                send[:sizes[rank]] = o_local
        recv = torch.empty(world * cap, dtype=odt, device=query.device)
        works.append(dist.all_gather_into_tensor(recv, send, group=group, async_op=True))
        gathered.append((c, cap, sizes, recv))
    for w in works:
        w.wait()

    out = torch.empty(B, H, S, D, dtype=odt, device=query.device)
    for c, cap, sizes, recv in gathered:
        for r in range(world):
            if sizes[r] == 0:
                continue
            s = per_rank[r][c]
            block = recv[r * cap:r * cap + sizes[r]].view(len(s.batches), (s.g1 - s.g0) * G, S, D)
            out[s.b0:s.b1:s.bstep, s.g0 * G:s.g1 * G] = block
    return out


def _int8_compute(v_scale):
    from . import flash_attn_int8qk_strided

    def compute(q, k, v, out=None, peer_outputs=None, q_side=None, kv_side=None, is_causal=False, window_size=-1,
                rot_cos=None, rot_sin=None):
        return flash_attn_int8qk_strided(q, k, v, q_side, kv_side, v_scale, is_causal, window_size, out=out,
                                         peer_outputs=peer_outputs)

    return compute


def flash_attn_int8qk_sharded(query, key, value, q_scale, k_scale, v_scale: float, is_causal: bool = False,
                              window_size: int = -1, group=None, chunks: Optional[int] = 1,
                              out: Optional[SymmetricOutput] = None):
    """flash_attn_int8qk over all ranks of `group` (same arguments, plus the
    gather options of flash_attn_sharded): every rank passes the same full int8
    inputs and per-token scales, computes its (batch, KV-head) units — the
    scales sliced with them — and receives the full float16 output, fused into
    the kernels with `out=SymmetricOutput(...)` or through NCCL otherwise."""
    return flash_attn_sharded(query, key, value, is_causal=is_causal, window_size=window_size, group=group,
                              compute=_int8_compute(v_scale), chunks=chunks, out=out, q_side=q_scale,
                              kv_side=k_scale)
