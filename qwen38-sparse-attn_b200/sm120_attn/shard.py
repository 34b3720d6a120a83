"""KV-head sharding of the sparse prefill across ranks (one process per GPU).

Every stage of the path - K block means, Q pooling, block selection, quantisation and the
attention itself - works per KV head and the g = H / Hk query heads that share it
(sparse_prefill.py:41-85 scores `qm[m, hk*g + i]` only against `km[hk]`; the kernels read K/V of
head `h // g` only).  N ranks therefore split the KV heads, rank r owning KV heads
[r*Hk/N, (r+1)*Hk/N) and query heads [r*H/N, (r+1)*H/N), and exchange nothing on the data path.
The only cross-rank traffic is the reduction of measurements (the slowest rank's time, the sum of
the work done).
"""
from __future__ import annotations


def kv_head_range(rank: int, world: int, num_kv_heads: int) -> tuple[int, int]:
    """[lo, hi) of the KV heads rank `rank` of `world` owns; world must divide num_kv_heads."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError(f'rank {rank} outside world {world}')
    if num_kv_heads % world:
        raise ValueError(f'{world} ranks cannot split {num_kv_heads} KV heads evenly')
    per = num_kv_heads // world
    return rank * per, (rank + 1) * per


def head_ranges(rank: int, world: int, num_heads: int, num_kv_heads: int) -> tuple[tuple[int, int], tuple[int, int]]:
    """((q_lo, q_hi), (kv_lo, kv_hi)): the query heads that go with the rank's KV heads."""
    if num_heads % num_kv_heads:
        raise ValueError('num_heads must be a multiple of num_kv_heads')
    g = num_heads // num_kv_heads
    lo, hi = kv_head_range(rank, world, num_kv_heads)
    return (lo * g, hi * g), (lo, hi)


def reduce_over_ranks(slowest, totals, device=None):
    """(max over ranks of each entry of `slowest`, sum over ranks of each entry of `totals`).

    Plain lists of floats in and out.  Without an initialised process group (one rank) the inputs
    come back unchanged.  With NCCL the tensors live on `device`; with gloo on the CPU.
    """
    import torch
    import torch.distributed as dist
    slowest = [float(x) for x in slowest]
    totals = [float(x) for x in totals]
    if not (dist.is_available() and dist.is_initialized()) or dist.get_world_size() == 1:
        return slowest, totals
    dev = device if (device is not None and dist.get_backend() == 'nccl') else torch.device('cpu')
    a = torch.tensor(slowest, dtype=torch.float64, device=dev)
    b = torch.tensor(totals, dtype=torch.float64, device=dev)
    dist.all_reduce(a, op=dist.ReduceOp.MAX)
    dist.all_reduce(b, op=dist.ReduceOp.SUM)
    return a.tolist(), b.tolist()
