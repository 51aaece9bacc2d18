"""Compile-time resource audit of every kernel in librdnattention.so (no GPU).

The reference gates its kernels on the compiler's resource report
(tests/head_dim_resources.py:17-18, 74-79: no spills, occupancy, LDS
budget).  The B200 analogue: compile rdnattention_b200/csrc/forward.cu for
sm_100a with `-Xptxas -v` and read only the per-function summary ptxas prints
(registers, spill bytes, static shared memory; no generated code is looked at):

* no kernel spills registers to local memory;
* a prefill kernel that re-splits registers between its warp roles
  (setmaxnreg) is allocated exactly the per-thread count its register split
  was sized for (Traits::LAUNCH_REGS), which the host also checks at launch;
* every other kernel fits its launch bounds (65536 registers per block);
* static shared memory stays within the 227 KB a CTA can address (dynamic
  shared memory is bounded by a static_assert in the kernel source).
"""
import re
import shutil
import subprocess
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
CSRC = ROOT / "rdnattention_b200" / "csrc"
NVCC = "/usr/local/cuda/bin/nvcc"

pytestmark = pytest.mark.skipif(not Path(NVCC).exists() or shutil.which("c++filt") is None,
                                reason="needs nvcc and c++filt")


@pytest.fixture(scope="module")
def report(tmp_path_factory):
    out = tmp_path_factory.mktemp("ptxas") / "forward.o"
    cmd = [NVCC, "-gencode", "arch=compute_100a,code=sm_100a", "-O3", "-std=c++17", "-lineinfo",
           "-Xcompiler", "-fPIC", "--expt-relaxed-constexpr", f"-I{ROOT / 'include'}", f"-I{CSRC}",
           "-Xptxas", "-v", "-c", str(CSRC / "forward.cu"), "-o", str(out)]
    res = subprocess.run(cmd, capture_output=True, text=True, check=True)
    parts = re.split(r"ptxas info\s+: Compiling entry function '([^']+)' for 'sm_100a'", res.stderr)
    mangled, bodies = parts[1::2], parts[2::2]
    names = subprocess.run(["c++filt"], input="\n".join(mangled), capture_output=True, text=True,
                           check=True).stdout.splitlines()
    kernels = {}
    for name, body in zip(names, bodies):
        regs = re.search(r"Used (\d+) registers", body)
        spill = re.search(r"(\d+) bytes spill stores, (\d+) bytes spill loads", body)
        smem = re.search(r"(\d+) bytes smem", body)
        assert regs and spill, f"no resource summary for {name}"
        kernels[name] = dict(regs=int(regs.group(1)), spill_st=int(spill.group(1)), spill_ld=int(spill.group(2)),
                             smem=int(smem.group(1)) if smem else 0)
    return kernels


def _prefill_traits(name):
    m = re.search(r"fa_prefill_kernel<rdna::prefill::Traits<([^>]*)> >", name)
    if not m:
        return None
    a = [x.strip() for x in m.group(1).split(",")]
    D, DVMAX, BC, NT, NSK, NSV = map(int, a[:6])
    I8, SDB = a[6] == "true", a[7] == "true"
    twopass = len(a) > 9 and a[9] == "true"
    return dict(D=D, NT=NT, I8=I8, SDB=SDB, TWOPASS=twopass)


def _launch_regs(t):
    """Traits::LAUNCH_REGS / RESPLIT (fa_prefill.cuh): one-tile double-buffered kernels (FP16,
    and INT8 at head_dim 64) run two CTAs per SM at 128 registers; two-tile kernels launch at
    the most their thread count allows (384 threads: 168); both re-split them."""
    min_blocks = 2 if (t["NT"] == 1 and t["SDB"]) else 1
    resplit = t["NT"] == 2 or min_blocks == 2
    threads = 128 * t["NT"] + 128
    return (128 if min_blocks == 2 else (65536 // threads) // 8 * 8) if resplit else None


def test_every_kernel_is_reported(report):
    prefill = [n for n in report if "fa_prefill_kernel" in n]
    assert len(prefill) >= 20, sorted(report)
    assert any("fa_decode_kernel" in n for n in report)
    assert any("rope_rotate_kernel" in n for n in report)
    assert any("quantize_qkv_kernel" in n for n in report)


def test_no_register_spills(report):
    bad = {n: (r["spill_st"], r["spill_ld"]) for n, r in report.items() if r["spill_st"] or r["spill_ld"]}
    assert not bad, "kernels spill registers (store, load bytes): " + "; ".join(f"{n[:120]}: {v}"
                                                                             for n, v in bad.items())


def test_register_split_matches_launch(report):
    for name, r in report.items():
        t = _prefill_traits(name)
        if t is None:
            continue
        want = _launch_regs(t)
        if want is not None:
            assert r["regs"] == want, f"{name[:120]}: {r['regs']} registers, split sized for {want}"
        else:
            assert r["regs"] <= 255, name


def test_static_shared_memory_budget(report):
    for name, r in report.items():
        assert r["smem"] <= 227 * 1024, f"{name[:120]}: {r['smem']} bytes of static shared memory"
