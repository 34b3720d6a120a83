"""Build the C-ABI library `sm120_attn/_lib/libsa_b200.so` in-tree with nvcc for sm_100a.

    python qwen38-sparse-attn_b200/build.py [--verbose] [--force]

Sources are the CUDA files of `csrc/`; the CUDA runtime is linked statically so the library only
needs the driver at run time.  The build is skipped when the library is newer than every source.
"""
from __future__ import annotations

import argparse
import os
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

HERE = Path(__file__).resolve().parent
CSRC = HERE / 'csrc'
INCLUDE = HERE.parent / 'include'
OUT_DIR = HERE / 'sm120_attn' / '_lib'
LIB = OUT_DIR / 'libsa_b200.so'
SOURCES = ['common.cu', 'prep.cu', 'select.cu', 'attn_fwd.cu', 'attn_pair.cu', 'decoder.cu']
ARCH = ['-gencode', 'arch=compute_100a,code=sm_100a']


def nvcc() -> str:
    cand = os.environ.get('NVCC') or '/usr/local/cuda/bin/nvcc'
    return cand if Path(cand).exists() else 'nvcc'


def stale() -> bool:
    if not LIB.exists():
        return True
    t = LIB.stat().st_mtime
    deps = [CSRC / s for s in SOURCES] + list(CSRC.glob('*.cuh')) + list(INCLUDE.glob('*.h')) + [Path(__file__)]
    return any(d.stat().st_mtime > t for d in deps)


def build(verbose: bool = False, force: bool = False) -> Path:
    if not force and not stale():
        return LIB
    OUT_DIR.mkdir(parents=True, exist_ok=True)
    objs = []
    build_dir = HERE / '_build'
    build_dir.mkdir(exist_ok=True)
    flags = ARCH + ['-O3', '-lineinfo', '-std=c++17', '-Xcompiler', '-fPIC', '-I', str(INCLUDE),
                    '-Xcompiler', '-fvisibility=hidden']
    if verbose:
        flags += ['-Xptxas', '-v']
    def compile_one(src):
        obj = build_dir / (Path(src).stem + '.o')
        cmd = [nvcc()] + flags + ['-c', str(CSRC / src), '-o', str(obj)]
        return src, obj, subprocess.run(cmd, capture_output=True, text=True)

    # the translation units are independent: compile them concurrently, report in source order
    with ThreadPoolExecutor(max_workers=min(len(SOURCES), os.cpu_count() or 1)) as pool:
        results = list(pool.map(compile_one, SOURCES))
    for src, obj, r in results:
        if r.returncode != 0:
            sys.stderr.write(r.stdout + r.stderr)
            raise RuntimeError(f'nvcc failed on {src}')
        if verbose and (r.stdout or r.stderr):
            sys.stderr.write(r.stdout + r.stderr)
        objs.append(str(obj))
    tmp = LIB.with_suffix('.so.tmp')
    cmd = [nvcc()] + ARCH + ['-shared', '-o', str(tmp)] + objs
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        sys.stderr.write(r.stdout + r.stderr)
        raise RuntimeError('link failed')
    os.replace(tmp, LIB)
    return LIB


if __name__ == '__main__':
    ap = argparse.ArgumentParser()
    ap.add_argument('--verbose', action='store_true')
    ap.add_argument('--force', action='store_true')
    a = ap.parse_args()
    print(build(verbose=a.verbose, force=a.force))
