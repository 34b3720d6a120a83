"""Arguments that make `oracle.attention_fp8_kernel_model` follow the schedule of the FP8 attention
kernel in use (keys per online-softmax step, and the partner tile of the paired-tile kernel)."""
from __future__ import annotations


def fp8_model_kwargs(H: int, Hk: int, n_tiles: int) -> dict:
    from sm120_attn import ops
    keys, paired = ops.attn_schedule(fp8=True)
    kw = {'group': keys // 64}
    if paired:
        if (H // Hk) % 2 == 0:
            kw['partner_of'] = lambda h, t: (h ^ 1, t)
        else:
            kw['partner_of'] = lambda h, t: (h, t ^ 1) if (t ^ 1) < n_tiles else None
    return kw
