"""Arguments that make `oracle.attention_fp8_kernel_model` follow the schedule of the FP8 attention
kernel in use (keys per online-softmax step, the partner tile of the paired-tile kernel, and the split
walks of a launch whose partial last wave is split)."""
from __future__ import annotations


def fp8_model_kwargs(H: int, Hk: int, n_tiles: int, launch=None) -> dict:
    """launch: (H_launch, n_q, q_front, head_of, tile_of) of the whole attention launch when the model
    covers a slice of it (head_of / tile_of map the model's head and tile indices to the launch's),
    so that the units the launch splits (ops.attn_splits: the partial last wave on this GPU) are
    modelled as split walks.  Without it the launch is taken to be the model's own problem."""
    import torch
    from sm120_attn import ops
    keys, paired = ops.attn_schedule(fp8=True)
    kw = {'group': keys // 64}
    if paired:
        if (H // Hk) % 2 == 0:
            kw['partner_of'] = lambda h, t: (h ^ 1, t)
        else:
            kw['partner_of'] = lambda h, t: (h, t ^ 1) if (t ^ 1) < n_tiles else None
        return kw                                          # the paired kernel runs its units whole
    if launch is None:
        launch = (H, n_tiles * 128, 0, lambda h: h, lambda t: t)
    HL, n_q, q_front, head_of, tile_of = launch
    k = ops.attn_splits(n_q, q_front, HL, 'cuda')
    if k > 1:
        tiles = -(-(q_front + n_q) // 128)
        units = HL * tiles
        slots = 2 * torch.cuda.get_device_properties(torch.cuda.current_device()).multi_processor_count
        n_whole = (units // slots) * slots if units >= slots else units
        kw.update(splits=k, split_min_steps=32 * k,
                  split_units=lambda h, t: head_of(h) * tiles + (tiles - 1 - tile_of(t)) >= n_whole)
    return kw
