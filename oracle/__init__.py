"""CPU oracle for the rdnattention forward path — TEST INFRASTRUCTURE ONLY.

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg import
this package, as the checker.  The product package (rdnattention_b200) never
imports it and has no CPU fallback.

Two restatements of the reference's algorithm live here:

* ``attn_oracle.c`` (wrapped by :mod:`oracle.c_oracle`): fp64 accumulation,
  the semantics of the reference's fp64 gates
  (tests/hip_forward_gate.hip:59-129, tests/hip_forward_int8qk_gate.hip:61-120).
* :mod:`oracle.torch_oracle`: fp32 torch-on-CPU, the semantics of
  tests/accuracy.py:39-47 (dense_attention_reference) extended with the masks
  of tests/head_dim.py:23-44 and the RoPE of tests/rope.py:29-37.  This is the
  "fp32 math oracle" the FP16 tolerance gate is stated against, and the
  workload timed as the CPU baseline.

Both are pinned against fixtures generated from the reference's own oracle
code (tests/golden/make_golden.py) by tests/test_oracle_golden.py.
"""
