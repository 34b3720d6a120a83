"""Tensor-parallel random-init GQA decoder prefill: the end-to-end TTFT harness of benchmark configuration 5.

The reference reports prefill TTFT of a served model whose attention goes through the sparse prefill
hook (README.md:29-31, measured by scripts/bench_ttft.py: a streamed completion request, chunked
prefill of 8192 tokens, time to the first token).  Here the same work runs without a server: a
dense GQA decoder (RMSNorm, RoPE, SwiGLU, vLLM's layer definitions) with random N(0, std) bf16
weights prefills the prompt chunk by chunk, every attention layer going through
`SparsePrefill.forward_sm120fp8` (or `forward_sm120`) with the per-layer block-mean, scale and
optional FP8 KV caches carried between chunks, and returns the greedy first token.

Tensor parallelism is by KV head (one process per GPU): rank r owns KV heads
[r Hk/N, (r+1) Hk/N) with their query heads, a 1/N slice of the MLP intermediate dimension and of
the vocabulary.  The attention output projection and the MLP down projection are row-parallel and
followed by an all-reduce (sum, bf16, NCCL); the last token's logits are all-gathered.  Every
rank draws the full weight matrices from the same seeds and keeps its slice, so the model is the
same at every N.

GEMMs are cuBLAS (torch.matmul); RMSNorm, RoPE with the KV-cache write and SwiGLU are this
library's kernels (ops.add_rmsnorm / rope_qkv / silu_mul); attention is the sparse prefill path.
"""
from __future__ import annotations

import math
from dataclasses import dataclass

import torch

from . import ops
from . import sparse_prefill as ksp


@dataclass(frozen=True)
class DecoderConfig:
    layers: int = 64
    hidden: int = 5120
    heads: int = 64
    kv_heads: int = 8
    head_dim: int = 128
    inter: int = 25600
    vocab: int = 151936
    rope_theta: float = 1e6
    eps: float = 1e-6
    init_std: float = 0.02

    def params(self) -> int:
        per_layer = (self.hidden * (self.heads + 2 * self.kv_heads) * self.head_dim
                     + self.heads * self.head_dim * self.hidden + 3 * self.hidden * self.inter + 2 * self.hidden)
        return self.layers * per_layer + 2 * self.vocab * self.hidden + self.hidden

    def prefill_flops(self, tokens: int) -> float:
        """GEMM FLOPs of a prefill (every token through every projection; the LM head on one token)."""
        per_tok = 2 * self.layers * (self.hidden * (self.heads + 2 * self.kv_heads) * self.head_dim
                                     + self.heads * self.head_dim * self.hidden + 3 * self.hidden * self.inter)
        return float(per_tok) * tokens + 2.0 * self.vocab * self.hidden


@dataclass(frozen=True)
class Shard:
    """The slices of heads, intermediate columns and vocabulary that one rank owns."""
    q_heads: tuple
    kv_heads: tuple
    inter: tuple
    vocab: tuple


def shard(cfg: DecoderConfig, rank: int, world: int) -> Shard:
    if world <= 0 or not 0 <= rank < world:
        raise ValueError(f'rank {rank} of {world}')
    if cfg.kv_heads % world or cfg.inter % world or cfg.vocab % world:
        raise ValueError(f'{world} ranks do not divide kv_heads {cfg.kv_heads}, inter {cfg.inter}, vocab {cfg.vocab}')
    g = cfg.heads // cfg.kv_heads
    k0, k1 = rank * cfg.kv_heads // world, (rank + 1) * cfg.kv_heads // world
    i0, i1 = rank * cfg.inter // world, (rank + 1) * cfg.inter // world
    v0, v1 = rank * cfg.vocab // world, (rank + 1) * cfg.vocab // world
    return Shard((k0 * g, k1 * g), (k0, k1), (i0, i1), (v0, v1))


def _seed(base: int, layer: int, name: str) -> int:
    return (base * 1_000_003 + (layer + 1) * 7919 + sum(ord(c) * 31 ** i for i, c in enumerate(name))) % (2 ** 62)


def full_weight(shape, seed: int, std: float, device) -> torch.Tensor:
    """One full weight matrix, N(0, std) in bf16, from its own seed (the same on every rank)."""
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    w = torch.randn(shape, generator=g, device=device, dtype=torch.float32)
    return w.mul_(std).to(torch.bfloat16)


def layer_weights(cfg: DecoderConfig, layer: int, sh: Shard, seed: int, device) -> dict:
    """This rank's slices of one layer: qkv [(hq + 2 hk) D, hidden] (q rows, then k, then v),
    o [hidden, hq D], gate_up [2 il, hidden] (gate rows, then up), down [hidden, il], norms."""
    D, E, std = cfg.head_dim, cfg.hidden, cfg.init_std
    (h0, h1), (k0, k1), (i0, i1) = sh.q_heads, sh.kv_heads, sh.inter
    wq = full_weight((cfg.heads * D, E), _seed(seed, layer, 'q'), std, device)[h0 * D:h1 * D]
    wk = full_weight((cfg.kv_heads * D, E), _seed(seed, layer, 'k'), std, device)[k0 * D:k1 * D]
    wv = full_weight((cfg.kv_heads * D, E), _seed(seed, layer, 'v'), std, device)[k0 * D:k1 * D]
    qkv = torch.cat([wq, wk, wv]).contiguous()
    del wq, wk, wv
    o = full_weight((E, cfg.heads * D), _seed(seed, layer, 'o'), std, device)[:, h0 * D:h1 * D].contiguous()
    gate = full_weight((cfg.inter, E), _seed(seed, layer, 'gate'), std, device)[i0:i1]
    up = full_weight((cfg.inter, E), _seed(seed, layer, 'up'), std, device)[i0:i1]
    gate_up = torch.cat([gate, up]).contiguous()
    del gate, up
    down = full_weight((E, cfg.inter), _seed(seed, layer, 'down'), std, device)[:, i0:i1].contiguous()
    ones = torch.ones(E, dtype=torch.bfloat16, device=device)
    return {'qkv': qkv, 'o': o, 'gate_up': gate_up, 'down': down, 'ln1': ones, 'ln2': ones.clone()}


def rope_table(max_pos: int, head_dim: int, theta: float, device) -> torch.Tensor:
    """fp32 [max_pos, head_dim]: cos of the head_dim/2 angles pos * theta^(-2i/head_dim), then their
    sin (vLLM's cos_sin_cache layout, rotary_embedding/base.py), computed in float64."""
    inv = 1.0 / theta ** (torch.arange(0, head_dim, 2, dtype=torch.float64) / head_dim)
    ang = torch.arange(max_pos, dtype=torch.float64)[:, None] * inv[None, :]
    return torch.cat([ang.cos(), ang.sin()], dim=1).to(torch.float32).contiguous().to(device)


class TPDecoder:
    """One rank of the tensor-parallel decoder.  `prefill(ids)` runs the prompt in chunks and returns
    the greedy first token (a device int64 scalar; with return_logits, the last token's fp32 logits
    over the whole vocabulary); every rank must call it with the same ids."""

    def __init__(self, cfg: DecoderConfig, device, rank: int = 0, world: int = 1, group=None, seed: int = 0,
                 tau: float = 0.95, kernel: str = 'sm120fp8', fp8_kv_cache: bool = False, max_tokens: int = 131072,
                 chunk: int = 8192, min_kv: int = 8192, comm_blocks: int = 2):
        self.cfg, self.device, self.rank, self.world, self.group = cfg, torch.device(device), rank, world, group
        self.sh = shard(cfg, rank, world)
        self.hq = self.sh.q_heads[1] - self.sh.q_heads[0]
        self.hk = self.sh.kv_heads[1] - self.sh.kv_heads[0]
        self.il = self.sh.inter[1] - self.sh.inter[0]
        self.chunk, self.max_tokens, self.fp8_kv_cache = chunk, max_tokens, fp8_kv_cache
        if max_tokens % 128:
            raise ValueError('max_tokens must be a multiple of 128')
        dev, D, E = self.device, cfg.head_dim, cfg.hidden
        self.layers = [layer_weights(cfg, L, self.sh, seed, dev) for L in range(cfg.layers)]
        self.embed = full_weight((cfg.vocab, E), _seed(seed, -1, 'embed'), cfg.init_std, dev)
        v0, v1 = self.sh.vocab
        self.lm_head = full_weight((cfg.vocab, E), _seed(seed, -1, 'lm_head'), cfg.init_std, dev)[v0:v1].contiguous()
        self.final_norm = torch.ones(E, dtype=torch.bfloat16, device=dev)
        self.cos_sin = rope_table(max_tokens, D, cfg.rope_theta, dev)
        self.k_cache = [torch.empty(max_tokens, self.hk, D, dtype=torch.bfloat16, device=dev) for _ in self.layers]
        self.v_cache = [torch.empty(max_tokens, self.hk, D, dtype=torch.bfloat16, device=dev) for _ in self.layers]
        self.sp = ksp.SparsePrefill(self.hq, self.hk, D, dev, tau=tau, min_kv=min_kv, min_q=0, kernel=kernel)
        if fp8_kv_cache:                       # this model's e4m3 K/V (every layer at max_tokens) must fit
            rows = 8192
            while rows < max_tokens:           # entries grow by doubling from 8192 rows
                rows *= 2
            need = cfg.layers * 2 * rows * self.hk * D
            ksp.KV8_CACHE_MAX_BYTES = max(ksp.KV8_CACHE_MAX_BYTES, need + (1 << 30))
        c, bf = chunk, torch.bfloat16
        self.buf = {'h': torch.empty(c, E, dtype=bf, device=dev), 'x': torch.empty(c, E, dtype=bf, device=dev),
                    'qkv': torch.empty(c, (self.hq + 2 * self.hk) * D, dtype=bf, device=dev),
                    'q': torch.empty(c, self.hq, D, dtype=bf, device=dev),
                    'attn': torch.empty(c, self.hq, D, dtype=bf, device=dev),
                    'o': torch.empty(c, E, dtype=bf, device=dev), 'gu': torch.empty(c, 2 * self.il, dtype=bf, device=dev),
                    'a': torch.empty(c, self.il, dtype=bf, device=dev), 'd': torch.empty(c, E, dtype=bf, device=dev)}
        self._key = ('tp-decoder', id(self))
        # With several ranks the row-parallel projections run in `comm_blocks` row blocks whose
        # all-reduces go to a side stream, each overlapping the next block's GEMMs (1: no overlap).
        self.comm_blocks = max(1, int(comm_blocks)) if world > 1 else 1
        if self.comm_blocks > 1:
            self.comm_stream = torch.cuda.Stream(dev)
            self._ev = [[torch.cuda.Event() for _ in range(self.comm_blocks)] for _ in range(4)]

    def _all_reduce(self, t):
        if self.world > 1:
            torch.distributed.all_reduce(t, group=self.group)

    def _rope(self, L: int, qkv, q, c0: int, n: int) -> bool:
        """RoPE of the chunk's q and k into q and the layer's K/V cache rows, with the key block means
        written into the layer's block-mean cache in the same pass when that entry continues at c0.
        Returns whether it did (else _attention computes them from the cache rows)."""
        D = self.cfg.head_dim
        km = ksp.km_slot((self._key, L), 0, c0, c0 + n, self.hk, D, self.device)
        ops.rope_qkv(qkv, self.hq, self.hk, D, self.cos_sin, c0, q, self.k_cache[L][c0:c0 + n],
                     self.v_cache[L][c0:c0 + n], km=km, block=ksp.BLOCK)
        return km is not None

    def _attention(self, L: int, q, c0: int, n: int, out, means_written: bool = False):
        kv_len = c0 + n
        kc, vc = self.k_cache[L], self.v_cache[L]
        key = (self._key, L)
        km = ksp._cached_block_means(key, 0, kc[c0:kv_len], c0, kv_len, key_all=kc, written=means_written)
        if self.sp.kernel == 'sm120fp8':
            scales = ksp._cached_scales(key, 0, q, kc[:kv_len], vc[:kv_len], c0)
            kv8 = ksp._cached_kv8(key, 0, kc, vc, c0, kv_len, scales) if self.fp8_kv_cache else None
            self.sp.forward_sm120fp8(q, kc[:kv_len], vc[:kv_len], c0, out=out, km=km, scales=scales, kv8=kv8)
        else:
            self.sp.forward_sm120(q, kc[:kv_len], vc[:kv_len], c0, out=out, km=km)

    @torch.no_grad()
    def prefill(self, ids: torch.Tensor, return_logits: bool = False) -> torch.Tensor:
        cfg, b = self.cfg, self.buf
        T = int(ids.numel())
        if T <= 0 or T > self.max_tokens:
            raise ValueError(f'{T} tokens: expected 1..{self.max_tokens}')
        ids = ids.reshape(-1).to(self.device)
        D = cfg.head_dim
        n = 0
        for c0 in range(0, T, self.chunk):
            n = min(self.chunk, T - c0)
            h, x, qkv, q, attn = b['h'][:n], b['x'][:n], b['qkv'][:n], b['q'][:n], b['attn'][:n]
            o, gu, a, d = b['o'][:n], b['gu'][:n], b['a'][:n], b['d'][:n]
            torch.index_select(self.embed, 0, ids[c0:c0 + n], out=h)
            for L, W in enumerate(self.layers):
                ops.add_rmsnorm(h, W['ln1'], x, cfg.eps, delta=d if L > 0 else None)
                torch.matmul(x, W['qkv'].t(), out=qkv)
                written = self._rope(L, qkv, q, c0, n)
                self._attention(L, q, c0, n, attn, means_written=written)
                if self.comm_blocks > 1:
                    self._mlp_overlapped(W, attn.view(n, self.hq * D), h, x, o, gu, a, d, n)
                    continue
                torch.matmul(attn.view(n, self.hq * D), W['o'].t(), out=o)
                self._all_reduce(o)
                ops.add_rmsnorm(h, W['ln2'], x, cfg.eps, delta=o)
                torch.matmul(x, W['gate_up'].t(), out=gu)
                ops.silu_mul(gu, a)
                torch.matmul(a, W['down'].t(), out=d)
                self._all_reduce(d)
        if self.comm_blocks > 1:
            torch.cuda.current_stream(self.device).wait_stream(self.comm_stream)
        last = slice(n - 1, n)
        x1 = b['x'][last]
        ops.add_rmsnorm(b['h'][last], self.final_norm, x1, cfg.eps, delta=b['d'][last])
        logits = torch.matmul(x1, self.lm_head.t()).float()
        if self.world > 1:
            parts = [torch.empty_like(logits) for _ in range(self.world)]
            torch.distributed.all_gather(parts, logits, group=self.group)
            logits = torch.cat(parts, dim=1)
        return logits[0] if return_logits else logits.argmax(dim=1)[0]

    def _mlp_overlapped(self, W, attn2d, h, x, o, gu, a, d, n):
        """o = attn W_o^T, all-reduce, h += o, x = rmsnorm(h), MLP, d = a W_down^T, all-reduce, in row
        blocks: block j's all-reduce runs on the side stream while block j+1's GEMMs run; the last
        block's all-reduce of d is the only one the compute stream waits for unoverlapped."""
        cfg, cur, comm = self.cfg, torch.cuda.current_stream(self.device), self.comm_stream
        nb = self.comm_blocks
        step = -(-n // nb)
        blocks = [(r, min(n, r + step)) for r in range(0, n, step)]
        ev_o, done_o, ev_d, done_d = self._ev
        comm.wait_stream(cur)                                    # buffers are free (previous layer's use done)
        for j, (r0, r1) in enumerate(blocks):
            torch.matmul(attn2d[r0:r1], W['o'].t(), out=o[r0:r1])
            ev_o[j].record(cur)
            comm.wait_event(ev_o[j])
            with torch.cuda.stream(comm):
                torch.distributed.all_reduce(o[r0:r1], group=self.group)
                done_o[j].record(comm)
        for j, (r0, r1) in enumerate(blocks):
            cur.wait_event(done_o[j])
            ops.add_rmsnorm(h[r0:r1], W['ln2'], x[r0:r1], cfg.eps, delta=o[r0:r1])
            torch.matmul(x[r0:r1], W['gate_up'].t(), out=gu[r0:r1])
            ops.silu_mul(gu[r0:r1], a[r0:r1])
            torch.matmul(a[r0:r1], W['down'].t(), out=d[r0:r1])
            ev_d[j].record(cur)
            comm.wait_event(ev_d[j])
            with torch.cuda.stream(comm):
                torch.distributed.all_reduce(d[r0:r1], group=self.group)
                done_d[j].record(comm)
        cur.wait_stream(comm)

    def release_caches(self):
        """Drop this model's entries from the module-level block-mean, scale and FP8 KV caches."""
        for cache in (ksp._KMEAN_CACHE, ksp._SCALE_CACHE, ksp._KV8_CACHE):
            for k in [k for k in cache if isinstance(k[0], tuple) and k[0][:1] == (self._key,)]:
                del cache[k]


def reference_prefill(cfg: DecoderConfig, weights: list, embed, lm_head, ids, attention,
                      all_reduce=lambda t: t) -> torch.Tensor:
    """Plain fp32 PyTorch forward of the same decoder (tests): returns the last token's logits over
    lm_head's rows.  `attention(layer, q [T, H, D], k [T, Hk, D], v [T, Hk, D])` -> [T, H, D] fp32.
    With one rank's weight slices, `all_reduce` (sum over ranks) follows the two row-parallel
    projections, as in TPDecoder."""
    D, E = cfg.head_dim, cfg.hidden
    T = ids.numel()
    cs = rope_table(T, D, cfg.rope_theta, ids.device).double()
    cos, sin = cs[:, :D // 2].float(), cs[:, D // 2:].float()

    def rms(x, w):
        return x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + cfg.eps) * w.float()

    def rope(x):
        x1, x2 = x[..., :D // 2], x[..., D // 2:]
        c, s = cos[:, None, :], sin[:, None, :]
        return torch.cat([x1 * c - x2 * s, x2 * c + x1 * s], dim=-1)

    h = embed.float()[ids]
    H = weights[0]['o'].shape[1] // D
    Hk = (weights[0]['qkv'].shape[0] // D - H) // 2
    il = weights[0]['down'].shape[1]
    for L, W in enumerate(weights):
        x = rms(h, W['ln1'])
        qkv = x @ W['qkv'].float().t()
        q = rope(qkv[:, :H * D].view(T, H, D))
        k = rope(qkv[:, H * D:(H + Hk) * D].view(T, Hk, D))
        v = qkv[:, (H + Hk) * D:].view(T, Hk, D)
        o = all_reduce(attention(L, q, k, v).reshape(T, H * D) @ W['o'].float().t())
        h = h + o
        x = rms(h, W['ln2'])
        gu = x @ W['gate_up'].float().t()
        a = torch.nn.functional.silu(gu[:, :il]) * gu[:, il:]
        h = h + all_reduce(a @ W['down'].float().t())
    x = rms(h[-1:], torch.ones(E, device=h.device))
    return x @ lm_head.float().t()


def causal_attention(q, k, v, scale: float) -> torch.Tensor:
    """fp32 causal GQA attention (tests)."""
    T, H, D = q.shape
    g = H // k.shape[1]
    kk = k.repeat_interleave(g, dim=1)
    vv = v.repeat_interleave(g, dim=1)
    s = torch.einsum('thd,shd->hts', q, kk) * scale
    s = s.masked_fill(torch.triu(torch.ones(T, T, dtype=torch.bool, device=q.device), 1)[None], -math.inf)
    return torch.einsum('hts,shd->thd', s.softmax(-1), vv)
