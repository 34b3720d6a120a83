"""Import-compatible module name of the reference's BF16 driver (sm120_attn/kernels/kai_fa_bf16.py)."""
from .attention import attention_sm120  # noqa: F401
