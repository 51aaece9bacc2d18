"""Builds the reference's own fp64 gate oracles into oracle/_ref/libgate_ref.so.

    python oracle/build_ref.py [REFERENCE_ROOT]   (else $RDNA_REFERENCE_ROOT, else ../reference)

The reference pins its kernels with two CPU oracles written in plain C++ but
living inside HIP test drivers (tests/hip_forward_gate.hip and
tests/hip_forward_int8qk_gate.hip), which need hipcc as a whole.  This recipe
lifts only the CPU functions out of those files at build time — struct RefCfg,
applyRope and refAttention (FP16 gate, lines 52-129), quantize and
refAttention (INT8 gate, lines 61-120) — into a generated translation unit
under oracle/_ref/ (git-ignored, never committed), adds extern "C" shims that
mirror the gates' own runCase() glue, and compiles it with g++.

The result is the checker of the checker: tests/golden/make_golden.py runs it
to produce committed golden fixtures, and tests/test_oracle_golden.py compares
the in-repo restatement (oracle/attn_oracle.c) with it when it is present.
Nothing in the product links it.
"""
import os
import re
import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
OUT_DIR = HERE / "_ref"
LIB = OUT_DIR / "libgate_ref.so"


def reference_root(arg=None):
    """The reference checkout: an explicit argument, else $RDNA_REFERENCE_ROOT, else a
    directory named `reference` beside this repository; None when none of them holds
    the reference's gate drivers."""
    cands = [arg] if arg else []
    if os.environ.get("RDNA_REFERENCE_ROOT"):
        cands.append(os.environ["RDNA_REFERENCE_ROOT"])
    cands.append(HERE.parent.parent / "reference")
    for c in cands:
        root = Path(c)
        if (root / "tests" / "hip_forward_gate.hip").exists():
            return root
    return None


def _extract(text: str, start_pattern: str) -> str:
    """Returns the definition starting at start_pattern through its matching closing brace."""
    m = re.search(start_pattern, text)
    if not m:
        raise RuntimeError(f"pattern not found: {start_pattern}")
    i = text.index("{", m.start())
    depth = 0
    j = i
    while True:
        c = text[j]
        if c == "{":
            depth += 1
        elif c == "}":
            depth -= 1
            if depth == 0:
                break
        j += 1
    end = j + 1
    if text[m.start():].startswith("struct"):
        end = text.index(";", end) + 1
    return text[m.start():end]


SHIM = r"""
extern "C" {

// Mirrors tests/hip_forward_gate.hip runCase(): Q/K/V are fp16-rounded
// values as float, contiguous [B,H,S,D] / [B,Hkv,KS,D]; RoPE (if rot tables
// are given) is applied to the oracle's copies exactly as runCase() does.
int gate_f16_ref(const float* q, const float* k, const float* v, const float* rotCos, const float* rotSin,
                 int batch, int numHeads, int numKvHeads, int seqLen, int keySeqLen, int headDim,
                 float scale, int causal, int windowSize, double* out) {
    size_t qCount = (size_t)batch * numHeads * seqLen * headDim;
    size_t kvCount = (size_t)batch * numKvHeads * keySeqLen * headDim;
    std::vector<float> qf(q, q + qCount), kf(k, k + kvCount), vf(v, v + kvCount);
    bool hasRope = rotCos != nullptr;
    if (hasRope) {
        f16gate::applyRope(qf, seqLen, batch * numHeads, headDim, rotCos, rotSin);
        f16gate::applyRope(kf, keySeqLen, batch * numKvHeads, headDim, rotCos, rotSin);
    }
    f16gate::RefCfg c{batch, numHeads, numKvHeads, seqLen, keySeqLen, headDim, scale, causal != 0, windowSize,
                      hasRope};
    std::vector<double> o(qCount);
    f16gate::refAttention(qf, kf, vf, o, c);
    std::copy(o.begin(), o.end(), out);
    return 0;
}

// Mirrors tests/hip_forward_int8qk_gate.hip runCase(): dequantised float
// operands in, fp64 out.
int gate_int8_ref(const float* qDeq, const float* kDeq, const float* vDeq, int batch, int numHeads,
                  int numKvHeads, int seqLen, int keySeqLen, int headDim, float scale, int causal,
                  int windowSize, double* out) {
    size_t qCount = (size_t)batch * numHeads * seqLen * headDim;
    size_t kvCount = (size_t)batch * numKvHeads * keySeqLen * headDim;
    std::vector<float> qf(qDeq, qDeq + qCount), kf(kDeq, kDeq + kvCount), vf(vDeq, vDeq + kvCount);
    std::vector<double> o(qCount);
    i8gate::refAttention(qf, kf, vf, o, batch, numHeads, numKvHeads, seqLen, keySeqLen, headDim, scale,
                         causal != 0, windowSize);
    std::copy(o.begin(), o.end(), out);
    return 0;
}

int8_t gate_int8_quantize(float x, float scale) { return i8gate::quantize(x, scale); }

}  // extern "C"
"""


def build(ref_root=None, force: bool = False) -> Path:
    found = reference_root(ref_root)
    if found is None:
        raise FileNotFoundError("reference checkout not found (pass its root or set RDNA_REFERENCE_ROOT)")
    ref_root = found
    f16_src = ref_root / "tests" / "hip_forward_gate.hip"
    i8_src = ref_root / "tests" / "hip_forward_int8qk_gate.hip"
    if not f16_src.exists() or not i8_src.exists():
        raise FileNotFoundError(f"reference gate sources not found under {ref_root}")
    OUT_DIR.mkdir(exist_ok=True)
    if not force and LIB.exists():
        return LIB
    f16 = f16_src.read_text()
    i8 = i8_src.read_text()
    parts = [
        "// GENERATED by oracle/build_ref.py from the reference's gate files; not committed.",
        "#include <algorithm>", "#include <cmath>", "#include <cstdint>", "#include <cstdlib>",
        "#include <vector>",
        "namespace f16gate {",
        _extract(f16, r"struct RefCfg\s*\{"),
        _extract(f16, r"void applyRope\("),
        _extract(f16, r"void refAttention\("),
        "}  // namespace f16gate",
        "namespace i8gate {",
        "constexpr double kPScale = 1.0 / 127.0;",
        _extract(i8, r"int8_t quantize\("),
        _extract(i8, r"void refAttention\("),
        "}  // namespace i8gate",
        SHIM,
    ]
    src = OUT_DIR / "gate_ref.cpp"
    src.write_text("\n\n".join(parts))
    tmp = LIB.with_suffix(f".so.tmp{os.getpid()}")
    subprocess.run(["g++", "-O2", "-std=c++17", "-fPIC", "-shared", "-o", str(tmp), str(src)], check=True)
    os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    root = sys.argv[1] if len(sys.argv) > 1 and not sys.argv[1].startswith("-") else None
    print(build(root, force="--force" in sys.argv))
