"""The paired-tile FP8 attention kernel (SA_ATTN_KERNEL=pair, csrc/attn_pair.cu) against the oracle.

The library reads SA_ATTN_KERNEL once per process, so the FP8 attention tests of test_gpu_kernels.py
and the 65536-key slice tests run again in a child process with the variable set; they compare with
the oracle's P-rounding model of the paired walk (tests/kmodel.py) and the fp32 reference at the
same tolerances as the default kernel.
"""
from __future__ import annotations

import os
import subprocess
import sys
from pathlib import Path

import pytest

pytestmark = pytest.mark.gpu

ROOT = Path(__file__).resolve().parent.parent


def test_fp8_attention_suite_with_paired_kernel():
    env = dict(os.environ, SA_ATTN_KERNEL='pair')
    cmd = [sys.executable, '-m', 'pytest', '-q', '-x', '-p', 'no:cacheprovider', '-m', 'gpu',
           str(ROOT / 'tests' / 'test_gpu_kernels.py'), str(ROOT / 'tests' / 'test_gpu_long.py'), '-k', 'fp8']
    r = subprocess.run(cmd, cwd=ROOT, env=env, capture_output=True, text=True, timeout=1200)
    tail = (r.stdout + r.stderr)[-3000:]
    assert r.returncode == 0, tail
    assert 'passed' in tail and 'failed' not in tail, tail
