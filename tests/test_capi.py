"""The C-ABI library loads without a GPU, exports every symbol include/*.h declares, and rejects bad
arguments before touching the device."""
from __future__ import annotations

import ctypes
import re
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent


def declared_symbols():
    names = set()
    for h in (ROOT / 'include').glob('*.h'):
        names |= set(re.findall(r'^SA_API\s+(?:const\s+char\s*\*|int|int64_t|size_t)\s+(sa_\w+)\s*\(', h.read_text(), flags=re.M))
    return names


def test_library_exports_every_declared_symbol():
    from sm120_attn import _native as N
    L = N.lib()
    declared = declared_symbols()
    assert declared, 'no declarations parsed'
    for name in declared:
        assert hasattr(L, name), name
    assert set(N.exported_symbols()) == declared
    assert L.sa_version() == 1


@pytest.mark.parametrize('call,code', [
    (lambda L: L.sa_select(None, 0, 0, None, 0, 0, 0, 0, 0, 0, 0, 0, 0, 0.0, 0.0, 0, None, None, 0, None, None, 0,
                           None), -1),
    (lambda L: L.sa_block_means_bf16(None, 0, 0, 10, 2, 100, 0, 64, None, 0, 0, 0, None, 0, 0, None, 0, 0, None), -3),
    (lambda L: L.sa_attn_fwd_fp8(None, 0, 0, None, 0, 0, None, 0, 0, None, 0, 0, 10, 8, 2, 64, 100, 0, 0, None, None,
                                 0, 128, 64, None, 0, None, 0, None, 0, 1.0, None, None), -3),
    (lambda L: L.sa_attn_fwd_bf16(None, 0, 0, None, 0, 0, None, 0, 0, None, 0, 0, 10, 8, 3, 128, 100, 0, 0, None,
                                  None, 0, 128, 64, 1.0, None, None), -1),
    (lambda L: L.sa_quantize_e4m3(None, 0, 0, 4, 2, 128, None, 0, 9, None, 0, 0, 0, 0, None), -1),
    # paged entries: no page table
    (lambda L: L.sa_block_means_paged_bf16(None, 0, 0, 0, None, 16, 10, 2, 128, 0, 64, None, 0, 0, 0, None), -1),
    (lambda L: L.sa_absmax_paged_bf16(None, 0, 0, 0, None, 16, 0, 10, 2, 128, 1, None, None), -1),
    (lambda L: L.sa_quantize_paged_e4m3(None, 0, 0, 0, None, 16, 0, 4, 2, 128, None, 0, 1, None, 0, 0, None), -1),
    (lambda L: L.sa_rope_qkv_means_bf16(None, 0, 4, 8, 2, 128, None, 0, 8, None, None, 0, None, 0, 128, None, 0, 0,
                                        0, None), -1),
    # wait self-test: no status word; a limit below 1 us (the pointer is never dereferenced)
    (lambda L: L.sa_wait_selftest(None, 1000000, None), -1),
    (lambda L: L.sa_wait_selftest(64, 10, None), -1),
    # one-pass selection: no heads; head_dim 64 (not served: SA_ERR_UNSUPPORTED); no query pointer
    (lambda L: L.sa_select_q(None, 0, 0, 100, 0, 128, 0, 1, None, 0, 0, 0, 0, 0, 128, 16, 0.1, 0.95, 0, None, None,
                             0, None, None, 0, 0, None, 0, None, None), -1),
    (lambda L: L.sa_select_q(None, 0, 0, 100, 0, 128, 0, 1, None, 0, 0, 0, 8, 2, 64, 16, 0.1, 0.95, 0, None, None,
                             0, None, None, 0, 0, None, 0, None, None), -3),
    (lambda L: L.sa_select_q(None, 0, 0, 100, 0, 128, 0, 1, None, 0, 0, 0, 8, 2, 128, 16, 0.1, 0.95, 0, None, None,
                             0, None, None, 0, 0, None, 0, None, None), -1),
])
def test_argument_validation_without_gpu(call, code):
    from sm120_attn import _native as N
    L = N.lib()
    assert call(L) == code
    assert L.sa_last_error()


def test_paged_attention_and_split_refusals():
    """sa_attn_fwd_bf16_paged refuses page sizes it does not read in place, and sa_attn_fwd_fp8_split
    too many splits or a short workspace, before any device work (host buffers stand in for device
    pointers: nothing is dereferenced)."""
    from sm120_attn import _native as N
    L = N.lib()
    buf = (ctypes.c_uint8 * 4096)()
    b = (ctypes.addressof(buf) + 15) // 16 * 16
    rc = L.sa_attn_fwd_bf16_paged(b, 1024, 128, b, b, 24 * 256, 256, 128, b, 24, 4, b, 1024, 128, 10, 8, 2, 128, 60,
                                  0, 50, None, None, 0, 128, 64, 0.1, None, None)
    assert rc == -3 and b'page_size' in L.sa_last_error()
    args = [b, 1024, 128, b, 256, 128, b, 256, 128, b, 1024, 128, 10, 8, 2, 128, 60, 0, 50, None, None, 0, 128, 64,
            b, 0, b, 0, b, 0, 0.1, None]
    assert L.sa_attn_fwd_fp8_split(*args, 20, 8, b, 1 << 30, None) == -1
    assert b'splits' in L.sa_last_error()
    need = L.sa_attn_split_workspace_bytes(10, 0, 8, 4, 8)
    assert need == 8 * 4 * (128 * 128 + 256) * 4 + 32
    assert L.sa_attn_fwd_fp8_split(*args, 4, 8, b, need - 16, None) == -1
    assert b'workspace' in L.sa_last_error()


def test_native_error_message():
    from sm120_attn import _native as N
    with pytest.raises(N.NativeError, match='bad sizes'):
        N.call('sa_select', None, 0, 0, None, 0, 0, 0, 0, 0, 0, 0, 0, 0, ctypes.c_float(0), ctypes.c_float(0), 0,
               None, None, 0, None, None, 0, None)


def test_select_workspace_size_and_refusal():
    from sm120_attn import _native as N
    L = N.lib()
    need = L.sa_select_workspace_bytes(64, 64, 512)
    assert need == 64 * 64 * 512 * 4
    assert L.sa_select_workspace_bytes(64, 64, 500) == 64 * 64 * 512 * 4      # rows padded to 32 blocks
    assert L.sa_select_workspace_bytes(0, 64, 512) == 0
    # valid sizes but no workspace: refused before any launch (no GPU needed)
    buf = (ctypes.c_float * 4)()
    rc = L.sa_select(ctypes.addressof(buf), 0, 0, ctypes.addressof(buf), 0, 0, 0, 8, 2, 128, 4, 16, 0, 0.1, 0.95, 0,
                     None, None, 0, None, None, 0, None)
    assert rc == -1 and b'workspace' in L.sa_last_error()


def test_ops_refuse_cpu_tensors():
    import torch
    from sm120_attn import ops
    x = torch.zeros(4, 2, 128, dtype=torch.bfloat16)
    with pytest.raises(ValueError, match='CUDA'):
        ops.absmax(x, per_head=True)


def test_plain_c_caller(tmp_path):
    """The header is valid C99 and the library links and answers from a C program (no Python, no GPU)."""
    import shutil
    import subprocess
    from sm120_attn import _native as N
    gcc = shutil.which('gcc')
    if gcc is None:
        pytest.skip('gcc not available')
    lib = Path(N.LIB_PATH)
    exe = tmp_path / 'c_caller'
    cmd = [gcc, '-std=c99', '-Wall', '-Wextra', '-Werror', '-I', str(ROOT / 'include'), str(ROOT / 'tests' / 'c_caller.c'),
           '-o', str(exe), '-L', str(lib.parent), '-l:' + lib.name, '-Wl,-rpath,' + str(lib.parent)]
    subprocess.run(cmd, check=True, capture_output=True, text=True)
    r = subprocess.run([str(exe)], capture_output=True, text=True, timeout=120)
    assert r.returncode == 0, r.stdout + r.stderr
    assert '0 failures' in r.stdout
