"""Worker for the two-rank gloo test of KV-head sharding (imported by spawned processes)."""
from __future__ import annotations

import os
import sys
from datetime import timedelta
from pathlib import Path

ROOT = Path(__file__).resolve().parent.parent
for p in (str(ROOT), str(ROOT / 'qwen38-sparse-attn_b200'), str(ROOT / 'tests')):
    if p not in sys.path:
        sys.path.insert(0, p)

N, KV, H, HK, D, BLOCK, TAU = 200, 1024, 8, 2, 128, 64, 0.95


def _shard_problem(rank, world):
    """Full problem built identically on every rank; returns it and this rank's result on its shard."""
    import numpy as np
    import oracle as O
    import synth
    from sm120_attn.shard import head_ranges
    q, k, v, _ = synth.make_qkv(N, KV, H, HK, D, block=BLOCK, seed=11, strength='strong')
    q, k, v = (t.float().numpy() for t in (q, k, v))
    q_start = KV - N
    (q_lo, q_hi), (kv_lo, kv_hi) = head_ranges(rank, world, H, HK)
    qs = q_start - q_start % BLOCK

    def select(qq, kk, h, hk):
        qm = O.q_block_means(qq, q_start, BLOCK)
        _, km = O.block_means(kk, 0, BLOCK)
        return O.select_masks(qm, km, qs, BLOCK, h, hk, TAU)

    masks = select(q[:, q_lo:q_hi], k[:, kv_lo:kv_hi], q_hi - q_lo, kv_hi - kv_lo)
    out = O.attention_ref(q[:, q_lo:q_hi], k[:, kv_lo:kv_hi], v[:, kv_lo:kv_hi], q_start, masks,
                          q_block=BLOCK, kv_block=BLOCK, q_front=q_start % BLOCK)
    full = (q, k, v, select, q_start)
    return full, masks, out, (q_lo, q_hi)


def run(rank, world, port, result_dir):
    import numpy as np
    import oracle as O
    import torch
    import torch.distributed as dist
    from sm120_attn.shard import reduce_over_ranks
    os.environ['MASTER_ADDR'] = '127.0.0.1'
    os.environ['MASTER_PORT'] = str(port)
    dist.init_process_group('gloo', rank=rank, world_size=world, timeout=timedelta(seconds=60))
    try:
        (q, k, v, select, q_start), masks, out, (q_lo, q_hi) = _shard_problem(rank, world)
        # gather every rank's shard: masks [H/world, MB, NB] and outputs [n, H/world, D]
        mt = torch.from_numpy(masks.astype(np.uint8))
        ot = torch.from_numpy(out)
        mg = [torch.empty_like(mt) for _ in range(world)]
        og = [torch.empty_like(ot) for _ in range(world)]
        dist.all_gather(mg, mt)
        dist.all_gather(og, ot)
        masks_all = torch.cat(mg, 0).numpy().astype(bool)
        out_all = torch.cat(og, 1).numpy()
        # the unsharded problem on one rank must give the same masks bit for bit and the same output
        ref_masks = select(q, k, H, HK)
        ref_out = O.attention_ref(q, k, v, q_start, ref_masks, q_block=BLOCK, kv_block=BLOCK,
                                  q_front=q_start % BLOCK)
        assert np.array_equal(masks_all, ref_masks), 'sharded selection differs from the full problem'
        assert np.array_equal(out_all, ref_out), 'sharded attention differs from the full problem'
        # measurement reduction: slowest rank's times, summed work
        slow, tot = reduce_over_ranks([1.0 + rank, 5.0 - rank], [10.0 * (rank + 1)])
        assert slow == [float(world), 5.0] and tot == [10.0 * world * (world + 1) / 2], (slow, tot)
        Path(result_dir, f'ok{rank}').write_text('ok')
    finally:
        dist.destroy_process_group()


def _install_oracle_ops():
    """Host-side stand-ins for the CUDA entry points the glue calls (test infrastructure only): block
    means, amax and block selection computed by the oracle into CPU tensors."""
    import numpy as np
    import oracle as O
    import torch
    from sm120_attn import ops

    def block_means(x, pos0, block, out, out_block0, q8=None, inv_scale=None, fixed_divisor=0):
        b0, means = O.block_means(x.float().numpy(), pos0, block)
        out[:, b0 - out_block0:b0 - out_block0 + means.shape[1]] = torch.from_numpy(means)

    def absmax(x, per_head, out=None):
        a = x.float().abs()
        return a.amax(dim=(0, 2)) if per_head else a.amax().reshape(1)

    def select(qm, km, num_heads, num_kv_heads, nb_total, qblk0, scale, tau, mode, counts=None, lists=None,
               masks=None, workspace=None):
        MB, _, _ = qm.shape
        m = O.select_masks(qm.numpy(), km.numpy(), qblk0 * ops_block[0], ops_block[0], num_heads, num_kv_heads, tau,
                           nb_total=nb_total)
        if masks is not None:
            masks.copy_(torch.from_numpy(m.reshape(-1, nb_total).astype(np.uint8)))
        if counts is not None:
            c, li = O.masks_to_lists(m)
            counts.copy_(torch.from_numpy(c))
            lists[:, :nb_total].copy_(torch.from_numpy(li))

    ops_block = [64]
    ops.block_means, ops.absmax, ops.select = block_means, absmax, select
    ops.select_q_supported = lambda *a, **k: False          # the pooled path: block means + select
    return ops_block


def glue_run(rank, world, block=64):
    """This rank's shard of a chunked prefill through the product's host glue: block-mean cache
    (aligned and unaligned chunk boundaries, a stale entry rebuilt from the history), e4m3 scales and
    per-head block masks.  Returns (km [Hk_r, NB, D], masks per chunk, scales per chunk)."""
    import torch
    import synth
    import sm120_attn.sparse_prefill as ksp
    from sm120_attn.shard import head_ranges
    ops_block = _install_oracle_ops()
    ops_block[0] = block
    ksp.BLOCK = block
    ksp._KMEAN_CACHE.clear()
    ksp._SCALE_CACHE.clear()
    H_, HK_, total = 8, 2, 2600
    q, k, v, _ = synth.make_qkv(total, total, H_, HK_, D, block=block, q_start=0, seed=21, strength='strong')
    (q_lo, q_hi), (kv_lo, kv_hi) = head_ranges(rank, world, H_, HK_)
    q, k, v = q[:, q_lo:q_hi], k[:, kv_lo:kv_hi], v[:, kv_lo:kv_hi]
    sp = ksp.SparsePrefill(q_hi - q_lo, kv_hi - kv_lo, D, 'cpu', tau=TAU, min_kv=0, min_q=0, kernel='sm120')
    masks, scales = [], []
    # (layer key, first page, chunk start, chunk end): a new request, a continuation off the block
    # grid, and a later chunk of another layer whose cache entry does not exist (rebuilt from history)
    for layer, page, c0, c1 in (('L0', 7, 0, 1000), ('L0', 7, 1000, 2300), ('L1', 7, 2300, total)):
        km = ksp._cached_block_means(layer, page, k[c0:c1], c0, c1, key_all=k[:c1])
        scales.append(ksp._cached_scales(layer, page, q[c0:c1], k[:c1], v[:c1], c0))
        front = c0 % block
        q_pad = torch.zeros(front + (c1 - c0) + (-(front + c1 - c0)) % block, q.shape[1], D, dtype=q.dtype)
        q_pad[front:front + c1 - c0] = q[c0:c1]
        masks.append(sp.block_masks(q_pad, None, c0 - front, valid=(front, c1 - c0), union=False, km=km))
    return ksp._KMEAN_CACHE[('L0', 7)]['km'][:, :-(-2300 // block)].clone(), masks, scales


def run_glue(rank, world, port, result_dir):
    """The product's host glue on KV-head shards (two gloo ranks, oracle-backed stand-ins for the
    CUDA entry points): every rank's block-mean cache and block masks, gathered over the ranks, equal
    the unsharded run's bit for bit, and each rank's scales come from its own heads."""
    import torch
    import torch.distributed as dist
    os.environ['MASTER_ADDR'] = '127.0.0.1'
    os.environ['MASTER_PORT'] = str(port)
    dist.init_process_group('gloo', rank=rank, world_size=world, timeout=timedelta(seconds=60))
    try:
        km, masks, scales = glue_run(rank, world)
        kms = [torch.empty_like(km) for _ in range(world)]
        dist.all_gather(kms, km.contiguous())
        ref_km, ref_masks, _ = glue_run(0, 1)
        assert torch.equal(torch.cat(kms, 0), ref_km), 'sharded block-mean cache differs'
        for m, rm in zip(masks, ref_masks):
            parts = [torch.empty_like(m) for _ in range(world)]
            dist.all_gather(parts, m.contiguous())
            assert torch.equal(torch.cat(parts, 0), rm), 'sharded block masks differ'
        assert scales[0] == scales[1] and scales[2] != scales[0]  # continued request / fresh entry
        Path(result_dir, f'ok{rank}').write_text('ok')
    finally:
        dist.destroy_process_group()


TP_CFG = dict(layers=2, hidden=64, heads=8, kv_heads=2, head_dim=16, inter=96, vocab=48, init_std=0.1)


def tp_logits(rank, world, all_reduce):
    """Last-token logits of the tiny decoder from this rank's weight slices (fp32 torch on the CPU)."""
    import math
    import torch
    from sm120_attn import decoder as dd
    cfg = dd.DecoderConfig(**TP_CFG)
    sh = dd.shard(cfg, rank, world)
    weights = [dd.layer_weights(cfg, L, sh, 5, 'cpu') for L in range(cfg.layers)]
    embed = dd.full_weight((cfg.vocab, cfg.hidden), dd._seed(5, -1, 'embed'), cfg.init_std, 'cpu')
    v0, v1 = sh.vocab
    lm = dd.full_weight((cfg.vocab, cfg.hidden), dd._seed(5, -1, 'lm_head'), cfg.init_std, 'cpu')[v0:v1]
    ids = torch.randint(0, cfg.vocab, (40,), generator=torch.Generator().manual_seed(3))
    attn = lambda L, q, k, v: dd.causal_attention(q, k, v, 1 / math.sqrt(cfg.head_dim))
    return dd.reference_prefill(cfg, weights, embed, lm, ids, attn, all_reduce)


def run_tp_decoder(rank, world, port, result_dir):
    """Tensor-parallel decoder decomposition: each rank's head / intermediate / vocabulary slices
    with all-reduces after the row-parallel projections give the unsharded model's logits."""
    import torch
    import torch.distributed as dist
    os.environ['MASTER_ADDR'] = '127.0.0.1'
    os.environ['MASTER_PORT'] = str(port)
    dist.init_process_group('gloo', rank=rank, world_size=world, timeout=timedelta(seconds=60))
    try:
        def all_reduce(t):
            t = t.contiguous()
            dist.all_reduce(t)
            return t
        local = tp_logits(rank, world, all_reduce)
        parts = [torch.empty_like(local) for _ in range(world)]
        dist.all_gather(parts, local.contiguous())
        got = torch.cat(parts, dim=1)
        ref = tp_logits(0, 1, lambda t: t)
        err = (got - ref).abs().max().item() / ref.abs().max().item()
        assert err < 1e-5, err
        Path(result_dir, f'ok{rank}').write_text(f'{err}')
    finally:
        dist.destroy_process_group()
