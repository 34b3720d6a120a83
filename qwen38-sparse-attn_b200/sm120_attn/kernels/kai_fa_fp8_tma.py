"""Import-compatible module name of the reference's TMA FP8 driver (sm120_attn/kernels/kai_fa_fp8_tma.py)."""
from .attention import attention_sm120_fp8_tma  # noqa: F401
