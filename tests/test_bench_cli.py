"""bench.py's reference arm on the CPU, as the driver launches it: one JSON line with the contracted keys
(and the explicit `unavailable` form for workloads that have no CPU arm)."""
import json
import subprocess
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parent.parent


def _run(*args, timeout=300):
    r = subprocess.run([sys.executable, str(ROOT / 'bench.py'), *args], capture_output=True, text=True,
                       timeout=timeout, cwd=str(ROOT))
    assert r.returncode == 0, r.stderr[-2000:]
    lines = [l for l in r.stdout.splitlines() if l.startswith('{')]
    assert len(lines) == 1, r.stdout
    return json.loads(lines[0])


def test_reference_arm_line():
    d = _run('--impl', 'reference', '--steps', '1', '--warmup', '1')
    for key in ('metric', 'value', 'unit', 'impl', 'n_gpus', 'steps', 'warmup', 'higher_is_better', 'scaling',
                'vs_baseline', 'dtype', 'data', 'config', 'cpu_baseline', 'e2e'):
        assert key in d, key
    assert d['impl'] == 'reference' and d['unit'] == 'TFLOPS' and d['value'] > 0 and d['warmup'] == 1
    cb = d['cpu_baseline']
    assert cb['kind'] == 'port' and cb['cores'] >= 1 and cb['value'] == d['value'] and cb['sample']
    assert d['e2e'] == {'value': d['value'], 'unit': 'TFLOPS', 'h2d_bytes_per_step': 0, 'd2h_bytes_per_step': 0}


def test_reference_arm_selection_and_unavailable():
    d = _run('--impl', 'reference', '--workload', 'selection', '--steps', '1', '--warmup', '0')
    assert d['unit'] == 'GB/s' and d['value'] > 0 and 'selection path' in d['config']['workload']
    for workload in ('dense', 'chunked', 'hook', 'ttft', 'decoder_kernels'):
        u = _run('--impl', 'reference', '--workload', workload)
        assert u['impl'] == 'reference' and u['unavailable'], workload


def test_reference_arm_under_torchrun_prints_once():
    """The driver launches the reference arm like the GPU arm for N > 1: rank 0 alone runs and prints one
    line, the other ranks exit 0 without work."""
    import socket
    with socket.socket() as sk:
        sk.bind(('127.0.0.1', 0))
        port = sk.getsockname()[1]
    r = subprocess.run([sys.executable, '-m', 'torch.distributed.run', '--nnodes=1', '--nproc-per-node', '2',
                        '--master-addr', '127.0.0.1', '--master-port', str(port), str(ROOT / 'bench.py'),
                        '--impl', 'reference', '--gpus', '2', '--steps', '1', '--warmup', '0', '--workload', 'selection'],
                       capture_output=True, text=True, timeout=300, cwd=str(ROOT))
    assert r.returncode == 0, r.stderr[-2000:]
    lines = [l for l in r.stdout.splitlines() if l.startswith('{')]
    assert len(lines) == 1
    d = json.loads(lines[0])
    assert d['impl'] == 'reference' and d['n_gpus'] == 2 and d['value'] > 0
