"""A bounded in-kernel wait that runs out, and the unwind after it.

Every mbarrier wait in the kernels gives up after a limit, records the wait's
site in the device status word and makes its CTA unwind: copies in flight
land, issued MMAs drain, TMEM is released and the output store is skipped.
The failure contract it stands in for is the reference's -3 plus a message
(src/c_api.cpp:83-87) for a kernel that cannot finish.

rdna_debug_set_wait_test makes one prefill launch withhold CTA 0's first K
tile (its TMA load is never issued, so its barrier never completes) and
limits CTA 0's waits to 1 ms.  Nothing faults or hangs: the test checks that
the call returns, that the status word names one of the waits that depend on
the withheld tile, and that the next ordinary call on the same device is
correct against the oracle.
"""
import numpy as np
import pytest
import torch

from cases import gate_i8_inputs, rel_rms
from oracle import c_oracle

pytestmark = pytest.mark.gpu

R = pytest.importorskip("rdnattention_b200")

# sites that wait, directly or through another role, for the withheld K tile
_SITES = {
    0x202: "MMA issuer: K tile",
    0x204: "MMA issuer: P",
    0x203: "MMA issuer: V tile",
    0x101: "producer: K slot",
    0x102: "producer: V slot",
    0x301: "softmax: S",
    0x302: "softmax: O",
    0x304: "softmax: key scales",
    0x306: "softmax: exponent token",
    0x307: "softmax: P V",
}


@pytest.fixture(autouse=True)
def _device():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    R.debug_read_status()  # start from a clear status word
    yield
    R._lib_handle().rdna_debug_set_wait_test(-1, 0)
    torch.cuda.synchronize()


def _expire(run):
    lib = R._lib_handle()
    lib.rdna_debug_set_wait_test(0, 1_000_000)  # CTA 0: K block 0 withheld, 1 ms wait limit
    try:
        run()
    finally:
        lib.rdna_debug_set_wait_test(-1, 0)
    torch.cuda.synchronize()  # the launch completes: its waits are bounded
    code, count = R.debug_read_status()
    assert code in _SITES, f"status word {code:#x} names no wait on the withheld tile"
    # every thread whose own wait ran out counts one event (a softmax warp waits in all
    # 32 lanes); only CTA 0, at most 512 threads, has the shortened limit
    assert 1 <= count <= 512, count
    assert R.debug_read_status() == (0, 0)  # reading clears it


@pytest.mark.parametrize("D,causal", [(128, True), (64, False)])
def test_fp16_expired_wait_unwinds_and_next_call_is_correct(D, causal):
    g = torch.Generator().manual_seed(D)
    B, H, Hkv, S = 1, 4, 2, 384
    q = torch.randn(B, H, S, D, generator=g).half()
    k = torch.randn(B, Hkv, S, D, generator=g).half()
    v = torch.randn(B, Hkv, S, D, generator=g).half()
    qd, kd, vd = q.cuda(), k.cuda(), v.cuda()
    _expire(lambda: R.flash_attn(qd, kd, vd, is_causal=causal))
    got = R.flash_attn(qd, kd, vd, is_causal=causal).cpu()
    assert R.debug_read_status() == (0, 0)
    ref = c_oracle.attention_f16(q, k, v, causal=causal)
    err = (got.double() - ref).abs()
    assert err.max().item() <= 2e-3 and err.mean().item() <= 2e-4


@pytest.mark.parametrize("D", [64, 128])
def test_int8_expired_wait_unwinds_and_next_call_is_correct(D):
    """The INT8 kernels (one-pass at head_dim 64, two-pass at 128: their own MMA issuer
    and softmax roles, key-scale hand-off and accumulator folds) unwind the same way."""
    B, H, Hkv, S = 1, 4, 4, 512
    qi, ki, vi, qs, ks, vs, qvec, kvec = gate_i8_inputs(B, H, Hkv, S, S, D, True)
    args = (qi.cuda(), ki.cuda(), vi.cuda(), qvec.cuda(), kvec.cuda(), vs)
    _expire(lambda: R.flash_attn_int8qk(*args))
    got = R.flash_attn_int8qk(*args).cpu()
    assert R.debug_read_status() == (0, 0)
    ref = c_oracle.attention_int8(qi, ki, vi, qvec, kvec, vs, scale=np.float32(1.0) / np.sqrt(np.float32(D)))
    assert rel_rms(got, ref) < 5e-2


def test_peer_barrier_signals_and_its_wait_expires():
    """The cross-GPU barrier kernel of the fused all-gather, on one GPU (its
    'peer' flag array is a local buffer).  With the other rank's word already at
    the epoch it passes and writes the epoch into its slot of the peer's array;
    with a word that nothing sets, its wait runs out after the debug limit,
    records 0x401 and returns."""
    dev = torch.device("cuda", 0)
    peer = torch.zeros(2, dtype=torch.int32, device=dev)
    mine = torch.tensor([0, 5], dtype=torch.int32, device=dev)
    R._peer_barrier(2, 0, [peer.data_ptr()], mine.data_ptr(), 5, dev)
    torch.cuda.synchronize()
    assert peer.tolist() == [5, 0]
    assert R.debug_read_status() == (0, 0)
    lib = R._lib_handle()
    lib.rdna_debug_set_wait_test(0, 1_000_000)  # barrier waits limited to 1 ms
    try:
        R._peer_barrier(2, 0, [peer.data_ptr()], mine.data_ptr(), 6, dev)  # word 1 stays at 5
        torch.cuda.synchronize()
    finally:
        lib.rdna_debug_set_wait_test(-1, 0)
    assert R.debug_read_status() == (0x401, 1)
    assert peer.tolist() == [6, 0]
    # epochs compare modulo 2^32: a word one past the wrap has reached 0xFFFFFFFF
    mine[1] = 0
    R._peer_barrier(2, 0, [peer.data_ptr()], mine.data_ptr(), 0xFFFFFFFF, dev)
    torch.cuda.synchronize()
    assert R.debug_read_status() == (0, 0)
