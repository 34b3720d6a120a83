"""Paged KV caches read in place, and the key block means written at KV-write time, on the GPU.

The reference gathers a request's key/value history out of vLLM's paged cache on every chunk
(sm120_attn/sparse_prefill.py:521-522).  The paged entry points read the pages where they lie; each is
checked bit for bit against its contiguous counterpart run on the gathered rows (same kernels, same
summation order).  Cache slots and pages the request does not own are filled with NaN, so a read of
any of them would show.  The fused RoPE + block-means write (sa_rope_qkv_means_bf16) is checked bit
for bit against sa_rope_qkv_bf16 followed by sa_block_means_bf16.
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

import oracle as O
import synth

pytestmark = pytest.mark.gpu
DEV = torch.device('cuda')


def _ops():
    from sm120_attn import ops
    return ops


def _paged_case(kv_len, Hk, D, page, seed, spare=6, n_q=0, H=0):
    """NaN-filled caches holding a request's keys/values in shuffled pages; returns the caches, the
    int32 page table row and the contiguous k, v (bf16, on the GPU)."""
    _, k, v, _ = synth.make_qkv(max(n_q, 1), kv_len, max(H, Hk), Hk, D, seed=seed)
    k, v = k.to(DEV), v.to(DEV)
    npages = -(-kv_len // page)
    total = npages + spare
    perm = torch.randperm(total, generator=torch.Generator().manual_seed(seed))[:npages]
    kc = torch.full((total, page, Hk, D), float('nan'), dtype=torch.bfloat16, device=DEV)
    vc = torch.full_like(kc, float('nan'))
    pad = npages * page - kv_len
    kp = torch.cat([k, torch.full((pad, Hk, D), float('nan'), dtype=torch.bfloat16, device=DEV)])
    vp = torch.cat([v, torch.full((pad, Hk, D), float('nan'), dtype=torch.bfloat16, device=DEV)])
    kc[perm.to(DEV)] = kp.view(npages, page, Hk, D)
    vc[perm.to(DEV)] = vp.view(npages, page, Hk, D)
    return kc, vc, perm.to(torch.int32).to(DEV), k, v


@pytest.mark.parametrize('page', [16, 64, 96])
@pytest.mark.parametrize('pos0,n,block', [(0, 3000, 128), (1000, 2100, 64), (4032, 100, 128)])
def test_block_means_paged_equals_gathered(page, pos0, n, block):
    ops = _ops()
    Hk, D = 8, 128
    kc, _, table, k, _ = _paged_case(pos0 + n, Hk, D, page, seed=page + n)
    b0, b1 = pos0 // block, -(-(pos0 + n) // block)
    ref = torch.full((Hk, b1 - b0, D), float('nan'), device=DEV)
    ops.block_means(k[pos0:pos0 + n], pos0, block, ref, b0)
    out = torch.full_like(ref, float('nan'))
    ops.block_means_paged(kc, table, pos0, n, block, out, b0)
    torch.cuda.synchronize()
    assert torch.equal(out, ref)


@pytest.mark.parametrize('page', [16, 128])
@pytest.mark.parametrize('per_head', [False, True])
def test_absmax_and_quantize_paged_equal_gathered(page, per_head):
    ops = _ops()
    from sm120_attn._native import SA_QUANT_MUL_BF16
    Hk, D, kv = 4, 128, 2500
    kc, _, table, k, _ = _paged_case(kv, Hk, D, page, seed=page)
    for row0, rows in ((0, kv), (700, 1800), (2499, 1)):
        a = ops.absmax_paged(kc, table, row0, rows, per_head)
        b = ops.absmax(k[row0:row0 + rows], per_head)
        assert torch.equal(a, b)
    inv = torch.linspace(30.0, 60.0, Hk, device=DEV) if per_head else torch.tensor([45.0], device=DEV)
    for row0, rows in ((0, kv), (1111, 1389)):
        got = torch.zeros(rows, Hk, D, dtype=torch.uint8, device=DEV)
        ops.quantize_paged(kc, table, row0, inv, SA_QUANT_MUL_BF16, got)
        want = torch.zeros_like(got)
        ops.quantize(k[row0:row0 + rows], inv, SA_QUANT_MUL_BF16, want)
        assert torch.equal(got, want)


def _lists(H, n_tiles, NB, q_offset, kv_block, density, seed):
    rng = np.random.default_rng(seed)
    m = rng.random((H, n_tiles, NB)) < density
    for t in range(n_tiles):
        lo, hi = q_offset + t * 128, q_offset + t * 128 + 127
        for b in range(NB):
            if b * kv_block > hi:
                m[:, t, b] = False
            elif (b + 1) * kv_block - 1 >= lo:
                m[:, t, b] = True
    counts, lists = O.masks_to_lists(m.reshape(H * n_tiles, NB))
    return torch.from_numpy(counts).to(DEV), torch.from_numpy(lists).to(DEV)


@pytest.mark.parametrize('page', [8, 16, 32, 64, 128])
@pytest.mark.parametrize('n,kv,q_front,sparse', [(700, 4001, 30, True), (300, 1500, 77, False),
                                                 (256, 2048, 0, True)])
def test_attn_bf16_paged_equals_contiguous(page, n, kv, q_front, sparse):
    """Same output bits as sa_attn_fwd_bf16 on the gathered K/V (kv_len ends inside a page for the
    odd lengths; unowned slots and pages are NaN)."""
    ops = _ops()
    H, Hk, D = 8, 2, 128
    kc, vc, table, k, v = _paged_case(kv, Hk, D, page, seed=page * 7 + n, n_q=n, H=H)
    q = synth.make_qkv(n, kv, H, Hk, D, seed=n + page)[0].to(DEV)
    q_offset = kv - n - q_front
    n_tiles = -(-(q_front + n) // 128)
    counts = lists = None
    kv_block = 64
    if sparse:
        kv_block = 128 if page != 8 else 64
        counts, lists = _lists(H, n_tiles, -(-kv // kv_block), q_offset, kv_block, 0.3, seed=n)
    ref = torch.full((n, H, D), float('nan'), dtype=torch.bfloat16, device=DEV)
    ops.attn_bf16(q, k, v, ref, kv, q_front, q_offset, counts, lists, kv_block, D ** -0.5)
    ops.check_status(DEV)
    out = torch.full_like(ref, float('nan'))
    ops.attn_bf16_paged(q, kc, vc, table, out, kv, q_front, q_offset, counts, lists, kv_block, D ** -0.5)
    ops.check_status(DEV)
    torch.cuda.synchronize()
    assert not torch.isnan(out).any()
    assert torch.equal(out, ref)


def test_attn_bf16_paged_64row_lists_and_bad_page():
    """Two 64-row lists per tile (the BF16 glue at BLOCK 64) read through pages; then a page id out of
    range sets SA_DEV_BAD_PAGE and reads as zeros (no fault)."""
    ops = _ops()
    from sm120_attn._native import SA_DEV_BAD_PAGE
    H, Hk, D, n, kv, page = 8, 2, 128, 640, 3000, 16
    kc, vc, table, k, v = _paged_case(kv, Hk, D, page, seed=11, n_q=n, H=H)
    q = synth.make_qkv(n, kv, H, Hk, D, seed=12)[0].to(DEV)
    q_offset = kv - n
    rows64 = -(-n // 64)
    rng = np.random.default_rng(3)
    m = rng.random((H, rows64, -(-kv // 64))) < 0.3
    for r in range(rows64):
        lo = q_offset + r * 64
        m[:, r, (lo + 63) // 64 + 1:] = False
        m[:, r, lo // 64:(lo + 63) // 64 + 1] = True
    counts, lists = O.masks_to_lists(m.reshape(H * rows64, -1))
    counts, lists = torch.from_numpy(counts).to(DEV), torch.from_numpy(lists).to(DEV)
    ref = torch.empty(n, H, D, dtype=torch.bfloat16, device=DEV)
    ops.attn_bf16(q, k, v, ref, kv, 0, q_offset, counts, lists, 64, D ** -0.5, q_block=64)
    out = torch.empty_like(ref)
    ops.attn_bf16_paged(q, kc, vc, table, out, kv, 0, q_offset, counts, lists, 64, D ** -0.5, q_block=64)
    ops.check_status(DEV)
    assert torch.equal(out, ref)
    bad = table.clone()
    bad[3] = kc.shape[0] + 5                       # a full page
    bad[-1] = -2                                   # the page holding the last key (read with plain loads)
    ops.attn_bf16_paged(q, kc, vc, bad, out, kv, 0, q_offset, None, None, 64, D ** -0.5)
    assert ops.read_status(DEV) & SA_DEV_BAD_PAGE
    assert not torch.isnan(out).any()


@pytest.mark.parametrize('hq,hk,pos0,rows,block', [(32, 8, 0, 8192, 128), (4, 1, 8192, 1000, 128),
                                                   (16, 2, 100, 900, 64), (8, 4, 65408, 300, 128)])
def test_rope_means_bit_parity(hq, hk, pos0, rows, block):
    """sa_rope_qkv_means_bf16 writes q, the cache rows of k and v, and the key block means exactly as
    sa_rope_qkv_bf16 followed by sa_block_means_bf16 over the written k rows."""
    ops = _ops()
    from sm120_attn.decoder import rope_table
    D = 128
    g = torch.Generator(device=DEV).manual_seed(rows + hq)
    qkv = torch.randn(rows, (hq + 2 * hk) * D, device=DEV, generator=g).to(torch.bfloat16)
    cs = rope_table(pos0 + rows, D, 1e6, DEV)
    outs = []
    for fused in (False, True):
        q = torch.empty(rows, hq, D, dtype=torch.bfloat16, device=DEV)
        kcache = torch.full((pos0 + rows, hk, D), float('nan'), dtype=torch.bfloat16, device=DEV)
        vcache = torch.full_like(kcache, float('nan'))
        b0, b1 = pos0 // block, -(-(pos0 + rows) // block)
        km = torch.full((hk, b1 + 3, D), float('nan'), device=DEV)
        kr, vr = kcache[pos0:], vcache[pos0:]
        if fused:
            ops.rope_qkv(qkv, hq, hk, D, cs, pos0, q, kr, vr, km=km, block=block)
        else:
            ops.rope_qkv(qkv, hq, hk, D, cs, pos0, q, kr, vr)
            ops.block_means(kr, pos0, block, km, 0)
        outs.append((q, kr, vr, km[:, b0:b1]))
    torch.cuda.synchronize()
    for a, b in zip(*outs):
        assert torch.equal(a, b)
    # and the rotation itself against an fp64 restatement (bf16 rounding of the fp32 result)
    x = qkv[:, hq * D:(hq + hk) * D].view(rows, hk, D).double()
    pos = torch.arange(pos0, pos0 + rows, device=DEV, dtype=torch.float64)
    inv = 1e6 ** (-torch.arange(0, D, 2, device=DEV, dtype=torch.float64) / D)
    ang = pos[:, None] * inv[None]
    c, s = torch.cos(ang)[:, None], torch.sin(ang)[:, None]
    x1, x2 = x[..., :D // 2], x[..., D // 2:]
    want = torch.cat([x1 * c - x2 * s, x2 * c + x1 * s], -1)
    assert (outs[1][1].double() - want).abs().max() < 2e-2 * want.abs().max()


def test_decoder_block_means_written_at_rope(monkeypatch):
    """Prefill chunks of a small decoder (later ones starting inside a key block): the block-mean cache
    it fills through the fused RoPE write equals sa_block_means_bf16 over its K cache rows, bit for bit
    (the block a chunk continues holds the mean of that chunk's rows there)."""
    import sm120_attn.sparse_prefill as ksp
    from sm120_attn.decoder import DecoderConfig, TPDecoder
    ops = _ops()
    monkeypatch.setattr(ksp, 'BLOCK', 128)
    ksp._KMEAN_CACHE.clear()
    cfg = DecoderConfig(layers=2, hidden=512, heads=8, kv_heads=2, head_dim=128, inter=1024, vocab=1000)
    dec = TPDecoder(cfg, DEV, max_tokens=4096, chunk=1000, min_kv=1024)
    T = 2500
    ids = torch.randint(0, cfg.vocab, (T,), generator=torch.Generator().manual_seed(0))
    dec.prefill(ids)
    torch.cuda.synchronize()
    nb = -(-T // 128)
    for L in range(cfg.layers):
        entry = ksp._KMEAN_CACHE[((dec._key, L), 0)]
        assert entry['nb'] == nb and entry['last_kv'] == T
        ref = torch.full((cfg.kv_heads, nb, 128), float('nan'), device=DEV)
        for c0 in range(0, T, 1000):               # chunk by chunk, later chunks overwriting shared blocks
            c1 = min(c0 + 1000, T)
            ops.block_means(dec.k_cache[L][c0:c1], c0, 128, ref, 0)
        assert torch.equal(entry['km'][:, :nb], ref)
    dec.release_caches()
