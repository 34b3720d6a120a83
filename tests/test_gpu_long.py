"""Parity at the benchmark's long-context shape: an 8192-row chunk at offset 57344 against 65536 keys.

The kernels run on the whole problem (two KV-head groups of eight query heads: the kernels work per
(query head, 128-row tile), so two groups exercise the same code as eight); the fp32 oracle checks a
slice that stays affordable on the host: the last three 128-row query tiles of every head of KV group
1, each attending over up to 65536 keys.  That is where the online softmax runs longest (about 1000
key tiles per row), where fp32 row-sum accumulation and e4m3 underflow of P are most exposed.

Tolerances (the parity bar): FP8 rel-L2 3e-2 against the fp32 reference on the same masks and the
same e4m3 operands, and rel-L2 1e-2 against the P-rounding model of the kernel; BF16 max-abs 2e-2.
The masks come from the product's own selection (`sa_select`); their parity with the oracle at this
shape is `test_select_matches_oracle[b128_*_65536_64]`.
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

import oracle as O
import synth
from kmodel import fp8_model_kwargs

pytestmark = pytest.mark.gpu

DEV = 'cuda'
N, KV, D, BLK = 8192, 65536, 128, 128
Q0 = KV - N
H, HK = 16, 2
TILES = 3                     # query tiles checked (the last ones: the longest rows)
GROUP = 1                     # KV group checked


def f32(t):
    return t.float().cpu().numpy()


def rel_l2(a, b):
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


@pytest.fixture(scope='module')
def inputs():
    q, k, v, _ = synth.make_qkv(N, KV, H, HK, D, block=BLK, seed=57344, strength='unit', hot=6)
    return q, k, v


def _slice_lists(counts, lists, heads, tiles_total):
    """counts/lists rows of the checked heads and tiles, re-indexed for a chunk of TILES tiles."""
    c = counts.cpu().numpy()
    li = lists.cpu().numpy()
    rows = [h * tiles_total + t for h in heads for t in range(tiles_total - TILES, tiles_total)]
    return c[rows].astype(np.int32), li[rows].astype(np.int32)


def _launch(heads):
    """The whole attention launch behind the checked slice (for the split walks of its last wave)."""
    return (H, N, 0, lambda h: heads[h], lambda t: N // 128 - TILES + t)


def _masks_from_lists(cs, ls, nheads, nb):
    m = np.zeros((nheads * TILES, nb), dtype=bool)
    for r in range(nheads * TILES):
        m[r, ls[r, :cs[r]]] = True
    return m.reshape(nheads, TILES, nb)


def _selected(inputs, kernel):
    import sm120_attn.sparse_prefill as ksp
    from sm120_attn import ops
    q, k, v = inputs
    ksp.BLOCK = BLK
    ksp._KMEAN_CACHE.clear()
    sp = ksp.SparsePrefill(H, HK, D, DEV, tau=0.95, min_kv=0, min_q=0, kernel=kernel)
    qd, kd, vd = q.to(DEV), k.to(DEV), v.to(DEV)
    km = ksp._cached_block_means('long', 0, kd[Q0:], Q0, KV, key_all=kd)
    return sp, ops, (qd, kd, vd), km


def test_fp8_sparse_65536_keys(inputs):
    sp, ops, (qd, kd, vd), km = _selected(inputs, 'sm120fp8')
    q, k, v = inputs
    amax = [float(np.abs(f32(t)).max()) for t in (q, k, v)]
    scales = tuple(a / 448.0 for a in amax)
    out = sp.forward_sm120fp8(qd, kd, vd, Q0, km=km, scales=scales)
    torch.cuda.synchronize()
    ops.check_status(DEV)
    heads = list(range(GROUP * (H // HK), (GROUP + 1) * (H // HK)))
    cs, ls = _slice_lists(sp.last_counts, sp.last_lists, heads, N // 128)
    nb = KV // BLK
    masks = _masks_from_lists(cs, ls, len(heads), nb)
    inv = [np.float32(1.0 / s) for s in scales]
    q8 = O.quantize_glue(f32(q)[-TILES * 128:, heads], inv[0])
    k8 = O.quantize_glue(f32(k)[:, GROUP:GROUP + 1], inv[1])
    v8 = O.quantize_glue(f32(v)[:, GROUP:GROUP + 1], inv[2])
    deq = [O.e4m3_decode(b) * np.float32(s) for b, s in zip((q8, k8, v8), scales)]
    got = f32(out)[-TILES * 128:, heads]
    assert np.isfinite(got).all()
    ref = O.attention_ref(*deq, KV - TILES * 128, masks, q_block=128, kv_block=BLK)
    model = O.attention_fp8_kernel_model(q8, k8, v8, *scales, KV - TILES * 128, cs, ls, q_block=128, kv_block=BLK,
                                         **fp8_model_kwargs(len(heads), 1, TILES, launch=_launch(heads)))
    print(f'fp8 65536 keys: kept {cs.sum() / (len(heads) * TILES * nb):.3f}, rel-L2 vs fp32 {rel_l2(got, ref):.3e}, '
          f'vs P-rounding model {rel_l2(got, model):.3e}')
    assert rel_l2(got, model) < 1e-2
    assert rel_l2(got, ref) < 3e-2


def test_fp8_dense_65536_keys_per_head_scales(inputs):
    """configs[2]'s shape (dense causal, per-head amax/448 scales), checked on the slice."""
    from sm120_attn import ops
    from sm120_attn._native import SA_QUANT_DIV
    q, k, v = inputs
    qd, kd, vd = q.to(DEV), k.to(DEV), v.to(DEV)
    scl = [ops.absmax(t, per_head=True).clamp_min_(1e-6) / 448.0 for t in (qd, kd, vd)]
    q8, k8, v8 = (torch.empty(t.shape, dtype=torch.uint8, device=DEV) for t in (qd, kd, vd))
    for t, s8, sc in zip((qd, kd, vd), (q8, k8, v8), scl):
        ops.quantize(t, sc, SA_QUANT_DIV, s8)
    out = torch.full((N, H, D), float('nan'), dtype=torch.bfloat16, device=DEV)
    ops.attn_fp8(q8, k8, v8, out, KV, 0, Q0, None, None, 64, scl[0], scl[1], scl[2], D ** -0.5)
    torch.cuda.synchronize()
    ops.check_status(DEV)
    heads = list(range(GROUP * (H // HK), (GROUP + 1) * (H // HK)))
    sq, sk, sv = (s.cpu().numpy() for s in scl)
    q8s = q8.cpu().numpy()[-TILES * 128:, heads]
    k8s = k8.cpu().numpy()[:, GROUP:GROUP + 1]
    v8s = v8.cpu().numpy()[:, GROUP:GROUP + 1]
    sqs, sks, svs = sq[heads], sk[GROUP:GROUP + 1], sv[GROUP:GROUP + 1]
    deq = [O.e4m3_decode(q8s) * sqs[None, :, None], O.e4m3_decode(k8s) * sks[None, :, None],
           O.e4m3_decode(v8s) * svs[None, :, None]]
    got = f32(out)[-TILES * 128:, heads]
    ref = O.attention_ref(*deq, KV - TILES * 128)
    model = O.attention_fp8_kernel_model(q8s, k8s, v8s, sqs, sks, svs, KV - TILES * 128, q_block=128, kv_block=64,
                                         **fp8_model_kwargs(len(heads), 1, TILES, launch=_launch(heads)))
    print(f'fp8 dense 65536 keys: rel-L2 vs fp32 {rel_l2(got, ref):.3e}, vs P-rounding model {rel_l2(got, model):.3e}')
    assert rel_l2(got, model) < 1e-2
    assert rel_l2(got, ref) < 3e-2


def test_bf16_sparse_65536_keys(inputs):
    sp, ops, (qd, kd, vd), km = _selected(inputs, 'sm120')
    q, k, v = inputs
    out = sp.forward_sm120(qd, kd, vd, Q0, km=km)
    torch.cuda.synchronize()
    ops.check_status(DEV)
    heads = list(range(GROUP * (H // HK), (GROUP + 1) * (H // HK)))
    cs, ls = _slice_lists(sp.last_counts, sp.last_lists, heads, N // 128)
    masks = _masks_from_lists(cs, ls, len(heads), KV // BLK)
    got = f32(out)[-TILES * 128:, heads]
    ref = O.attention_ref(f32(q)[-TILES * 128:, heads], f32(k)[:, GROUP:GROUP + 1], f32(v)[:, GROUP:GROUP + 1],
                          KV - TILES * 128, masks, q_block=128, kv_block=BLK)
    err = float(np.abs(got - ref).max())
    print(f'bf16 65536 keys: max-abs {err:.3e}')
    assert err < 2e-2
