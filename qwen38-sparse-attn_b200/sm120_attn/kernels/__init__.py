"""B200 (sm_100a) block-sparse prefill attention kernels behind the reference's driver names.

attention_sm120          BF16 operands (kai_fa_bf16.py:1206)
attention_sm120_fp8      e4m3 operands (kai_fa_fp8.py:331)
attention_sm120_fp8_tma  e4m3 operands, same kernel (kai_fa_fp8_tma.py:447)
All support GQA, chunked-prefill causal masking with a query offset, and per-(head, query block)
block lists.  One tcgen05 / TMEM / TMA kernel serves all of them (see csrc/attn_fwd.cu).
"""
from .attention import (VT_KEY_PERM, attention_sm120, attention_sm120_fp8, attention_sm120_fp8_tma,
                        permute_vt_keys, quantize_e4m3, vt_key_index)

__all__ = ['attention_sm120', 'attention_sm120_fp8', 'attention_sm120_fp8_tma', 'quantize_e4m3', 'permute_vt_keys',
           'vt_key_index', 'VT_KEY_PERM']
