"""ctypes binding of the C-ABI library `_lib/libsa_b200.so` (declared in include/sparse_attn_b200.h).

The library is the only compute path: there is no CPU or PyTorch fallback.  `lib()` raises
`NativeLibraryError` when the library is missing or does not load, and every op raises
`NativeError` with the library's message when an entry point returns an error code.
"""
from __future__ import annotations

import ctypes
import os
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / '_lib' / 'libsa_b200.so'

SA_OK = 0
SA_ERR_ARG, SA_ERR_ALIGN, SA_ERR_UNSUPPORTED, SA_ERR_CUDA, SA_ERR_TMA, SA_ERR_DEVICE = -1, -2, -3, -4, -5, -6
SA_DEV_WAIT_Q, SA_DEV_WAIT_KV, SA_DEV_WAIT_S, SA_DEV_WAIT_P, SA_DEV_WAIT_O, SA_DEV_BAD_LIST = 1, 2, 4, 8, 16, 32
SA_DEV_BAD_PAGE, SA_DEV_WAIT_KM, SA_DEV_WAIT_TEST = 64, 128, 256
SA_SELECT_PER_HEAD, SA_SELECT_KV_UNION, SA_SELECT_PAIR_UNION = 0, 1, 2
SA_QUANT_MUL, SA_QUANT_MUL_BF16, SA_QUANT_DIV = 0, 1, 2

_i32, _i64, _f32, _p, _sz = ctypes.c_int32, ctypes.c_int64, ctypes.c_float, ctypes.c_void_p, ctypes.c_size_t

# name -> argument types (return type is int for all but sa_last_error and the size queries)
SIGNATURES = {
    'sa_version': [],
    'sa_read_status': [_p, _p, _p],
    'sa_wait_selftest': [_p, _i64, _p],
    'sa_block_means_bf16': [_p, _i64, _i64, _i32, _i32, _i32, _i32, _i32, _p, _i64, _i64, _i32, _p, _i64, _i64, _p,
                            _i32, _i32, _p],
    'sa_select': [_p, _i64, _i64, _p, _i64, _i64, _i32, _i32, _i32, _i32, _i32, _i32, _i32, _f32, _f32, _i32, _p, _p,
                  _i64, _p, _p, _sz, _p],
    'sa_select_workspace_bytes': [_i32, _i32, _i32],
    'sa_select_q': [_p, _i64, _i64, _i32, _i32, _i32, _i32, _i32, _p, _i64, _i64, _i32, _i32, _i32, _i32, _i32, _f32,
                    _f32, _i32, _p, _p, _i64, _p, _p, _i64, _i64, _p, _i32, _p, _p],
    'sa_select_static': [_p, _i64, _i64, _p, _i64, _i64, _i32, _i32, _i32, _i32, _i32, _i32, _i32, _f32, _f32, _i32,
                         _p, _p, _i64, _p, _p],
    'sa_quantize_e4m3': [_p, _i64, _i64, _i32, _i32, _i32, _p, _i32, _i32, _p, _i64, _i64, _i32, _i32, _p],
    'sa_absmax_bf16': [_p, _i64, _i64, _i32, _i32, _i32, _i32, _p, _p],
    'sa_attn_fwd_fp8': [_p, _i64, _i64, _p, _i64, _i64, _p, _i64, _i64, _p, _i64, _i64, _i32, _i32, _i32, _i32, _i32,
                        _i32, _i32, _p, _p, _i64, _i32, _i32, _p, _i32, _p, _i32, _p, _i32, _f32, _p, _p],
    'sa_attn_fwd_bf16': [_p, _i64, _i64, _p, _i64, _i64, _p, _i64, _i64, _p, _i64, _i64, _i32, _i32, _i32, _i32, _i32,
                         _i32, _i32, _p, _p, _i64, _i32, _i32, _f32, _p, _p],
    'sa_add_rmsnorm_bf16': [_p, _i64, _p, _i64, _p, _p, _i64, _i32, _i32, _f32, _p],
    'sa_rope_qkv_bf16': [_p, _i64, _i32, _i32, _i32, _i32, _p, _i32, _i32, _p, _p, _i64, _p, _i64, _p],
    'sa_silu_mul_bf16': [_p, _i64, _i32, _i32, _p, _i64, _p],
    'sa_rope_qkv_means_bf16': [_p, _i64, _i32, _i32, _i32, _i32, _p, _i32, _i32, _p, _p, _i64, _p, _i64, _i32, _p,
                               _i64, _i64, _i32, _p],
    'sa_block_means_paged_bf16': [_p, _i64, _i64, _i64, _p, _i32, _i32, _i32, _i32, _i32, _i32, _p, _i64, _i64, _i32,
                                  _p],
    'sa_absmax_paged_bf16': [_p, _i64, _i64, _i64, _p, _i32, _i32, _i32, _i32, _i32, _i32, _p, _p],
    'sa_quantize_paged_e4m3': [_p, _i64, _i64, _i64, _p, _i32, _i32, _i32, _i32, _i32, _p, _i32, _i32, _p, _i64, _i64,
                               _p],
    'sa_attn_split_count': [_i32, _i32, _i32],
    'sa_attn_split_workspace_bytes': [_i32, _i32, _i32, _i32, _i32],
    'sa_attn_fwd_fp8_split': [_p, _i64, _i64, _p, _i64, _i64, _p, _i64, _i64, _p, _i64, _i64, _i32, _i32, _i32, _i32,
                              _i32, _i32, _i32, _p, _p, _i64, _i32, _i32, _p, _i32, _p, _i32, _p, _i32, _f32, _p,
                              _i32, _i32, _p, _i64, _p],
    'sa_attn_fwd_bf16_paged': [_p, _i64, _i64, _p, _p, _i64, _i64, _i64, _p, _i32, _i32, _p, _i64, _i64, _i32, _i32,
                               _i32, _i32, _i32, _i32, _i32, _p, _p, _i64, _i32, _i32, _f32, _p, _p],
}


# entry points that return a size instead of a status code
SIZE_QUERIES = {'sa_select_workspace_bytes': _sz, 'sa_attn_split_workspace_bytes': _i64}


class NativeLibraryError(RuntimeError):
    """The CUDA library is missing or failed to load (there is no fallback path)."""


class NativeError(RuntimeError):
    def __init__(self, fn: str, code: int, msg: str):
        super().__init__(f'{fn} failed ({code}): {msg}')
        self.code = code


_LIB = None


def lib():
    global _LIB
    if _LIB is None:
        path = os.environ.get('SA_B200_LIB', str(LIB_PATH))
        if not Path(path).exists():
            raise NativeLibraryError(f'{path} not found: build it with `python qwen38-sparse-attn_b200/build.py`')
        try:
            L = ctypes.CDLL(path)
        except OSError as e:
            raise NativeLibraryError(f'cannot load {path}: {e}') from e
        for name, args in SIGNATURES.items():
            f = getattr(L, name)
            f.argtypes = args
            f.restype = SIZE_QUERIES.get(name, ctypes.c_int)
        L.sa_last_error.argtypes = []
        L.sa_last_error.restype = ctypes.c_char_p
        _LIB = L
    return _LIB


def call(name: str, *args) -> None:
    L = lib()
    rc = getattr(L, name)(*args)
    if rc != SA_OK:
        raise NativeError(name, rc, (L.sa_last_error() or b'').decode(errors='replace'))


def exported_symbols() -> list:
    return list(SIGNATURES) + ['sa_last_error']
