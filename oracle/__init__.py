"""CPU oracle for the dynamic block-sparse prefill path (TEST INFRASTRUCTURE ONLY).

This package restates, in numpy, the reference algorithm of
accion-intelligence/Qwen38-sparse-attn (`sm120_attn/sparse_prefill.py` and
`sm120_attn/kernels/kai_fa_fp8.py`).  It is the checker for the CUDA path, never
part of it: only `tests/`, `__graft_entry__.smoke()` and the `cpu_baseline` /
`--impl reference` legs of `bench.py` may import it.  The product package
(`sm120_attn` under `qwen38-sparse-attn_b200/`) never imports it and fails
loudly when its CUDA library is missing.

Parity is pinned: `tests/test_oracle_golden.py` checks every function here
against golden vectors that `tests/golden/gen_golden.py` produced by running the
reference's own PyTorch code on CPU.
"""
from .sparse_oracle import *  # noqa: F401,F403
