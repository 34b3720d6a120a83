"""Import-compatible module name of the reference's FP8 driver and helpers (sm120_attn/kernels/kai_fa_fp8.py)."""
from .attention import (VT_KEY_PERM, attention_sm120_fp8, permute_vt_keys, quantize_e4m3,  # noqa: F401
                        vt_key_index)

P_SCALE = 448.0
