"""Dynamic block-sparse FP8/BF16 prefill attention for vLLM, B200 (sm_100a) implementation.

Drop-in for accion-intelligence/Qwen38-sparse-attn's `sm120_attn` package: same modules, entry points,
SM120_SPARSE_* knobs and cache semantics, with every kernel hand-written CUDA for sm_100a behind a
C ABI (include/sparse_attn_b200.h, built into _lib/libsa_b200.so).
"""
__version__ = '0.1.0'
from .kernels import attention_sm120, attention_sm120_fp8, attention_sm120_fp8_tma  # noqa: F401,E402
