"""Seeded synthetic inputs with the shapes and value distributions of the benchmark configurations.

Q/K/V ~ N(0, 1) in bf16.  Attention structure is injected per KV head with a direction u:
K rows of the sink block and of `hot` random blocks get +k_boost*u, every query row of the
head's group gets +q_boost*u.  `strength='unit'` uses a random unit u (the literal benchmark
recipe: near-dense masks at tau 0.95); `strength='strong'` uses u ~ N(0, I) un-normalised as the
reference's own tests do (tests/test_sparse_prefill.py:23-25), which gives sparse masks.
`local` adds a positional direction shared by nearby queries and keys so that the blocks just
before each query block carry mass (the chunked long-context configuration).

Generated with a torch.Generator so that the same seed gives the same tensors on CPU here and in
tests on the GPU box (generation happens on CPU unless `device` is a CUDA device, in which case
a CUDA generator is used - only the benchmark does that, for speed).
"""
from __future__ import annotations

import math

import torch


def _gen(device, seed):
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    return g


def make_qkv(n, kv_len, H, Hk, D, block=128, q_start=None, seed=0, strength='unit', hot=3,
             k_boost=4.0, q_boost=1.5, local=0, device='cpu', with_v=True):
    """Returns q [n, H, D], k [kv_len, Hk, D], v [kv_len, Hk, D] (bf16) and the hot block ids.

    q holds the chunk at absolute positions q_start.. (default kv_len - n).
    """
    if q_start is None:
        q_start = kv_len - n
    dev = torch.device(device)
    g = _gen(dev, seed)
    q = torch.randn(n, H, D, generator=g, device=dev, dtype=torch.float32)
    k = torch.randn(kv_len, Hk, D, generator=g, device=dev, dtype=torch.float32)
    v = torch.randn(kv_len, Hk, D, generator=g, device=dev, dtype=torch.float32) if with_v else None
    u = torch.randn(Hk, D, generator=g, device=dev, dtype=torch.float32)
    if strength == 'unit':
        u = u / u.norm(dim=-1, keepdim=True)
    nblk = -(-kv_len // block)
    hot_ids = []
    for hk in range(Hk):
        ids = torch.randperm(max(nblk - 1, 1), generator=g, device=dev)[:hot] + 1
        ids = torch.cat([torch.zeros(1, dtype=ids.dtype, device=dev), ids]).clamp_max(nblk - 1)
        hot_ids.append(ids)
        rows = (ids[:, None] * block + torch.arange(block, device=dev)[None, :]).reshape(-1)
        rows = rows[rows < kv_len]
        k[rows, hk] += k_boost * u[hk]
    g_heads = H // Hk
    q += q_boost * u.repeat_interleave(g_heads, 0)[None, :, :]
    if local:
        # positional direction rotating once every `local` blocks: queries and keys close in
        # position share it, which puts mass on the blocks just before each query block
        w = torch.randn(2, Hk, D, generator=g, device=dev, dtype=torch.float32)
        w = w / w.norm(dim=-1, keepdim=True)
        period = float(local * block * 4)
        pk = torch.arange(kv_len, device=dev, dtype=torch.float32)
        pq = torch.arange(q_start, q_start + n, device=dev, dtype=torch.float32)
        for hk in range(Hk):
            ak = 2 * math.pi * pk / period
            k[:, hk] += 2.0 * (torch.cos(ak)[:, None] * w[0, hk] + torch.sin(ak)[:, None] * w[1, hk])
            aq = 2 * math.pi * pq / period
            dq = 1.0 * (torch.cos(aq)[:, None] * w[0, hk] + torch.sin(aq)[:, None] * w[1, hk])
            q[:, hk * g_heads:(hk + 1) * g_heads] += dq[:, None, :]
    out = (q.to(torch.bfloat16), k.to(torch.bfloat16), v.to(torch.bfloat16) if with_v else None)
    return out + (torch.stack(hot_ids).cpu(),)


def checksum(t: torch.Tensor) -> float:
    """Order-independent fingerprint of a tensor (detects generator drift between machines)."""
    x = t.detach().float().cpu().reshape(-1).double()
    w = torch.arange(1, x.numel() + 1, dtype=torch.float64).remainder_(7919).add_(1.0)
    return float((x * w).sum())
