"""The drop-in `sm120_attn` API end to end on the GPU against the oracle.

Covers the reference's glue tests (tests/test_sparse_prefill.py:28-48, :65-92;
tests/test_sparse_prefill_fp8.py:13-31) and benchmark configuration 1 (H 64, Hk 8, D 128, 1024 queries at
7168 against 8192 keys, block 128, tau 0.95, both injection strengths).  Masks: exact up to the
tau-boundary exemption.  Outputs: rel-L2 3e-2 (FP8) / max-abs 2e-2 (BF16) against the fp32
reference computed on the same masks and the same (quantised) operands.
"""
from __future__ import annotations

import types

import numpy as np
import pytest
import torch
import torch.nn.functional as F

import oracle as O
import synth

pytestmark = pytest.mark.gpu
DEV = torch.device('cuda')


def f32(t):
    return t.float().cpu().numpy()


def rel_l2(a, b):
    return float(np.linalg.norm(a - b) / np.linalg.norm(b))


@pytest.fixture
def ksp():
    import sm120_attn.sparse_prefill as m
    old = m.BLOCK
    m._KMEAN_CACHE.clear()
    m._SCALE_CACHE.clear()
    m._KV8_CACHE.clear()
    yield m
    m.BLOCK = old
    m._KMEAN_CACHE.clear()
    m._SCALE_CACHE.clear()
    m._KV8_CACHE.clear()


def _heads_subset(H, g):
    """A full GQA group plus a spread of other heads (keeps the fp32 oracle affordable)."""
    return sorted(set(list(range(g)) + list(range(g, H, max(1, H // 8)))))


@pytest.mark.parametrize('strength', ['unit', 'strong'])
def test_fp8_config1_block128(ksp, strength):
    ksp.BLOCK = 128
    H, Hk, D, n, kv = 64, 8, 128, 1024, 8192
    q_start = kv - n
    q, k, v, _ = synth.make_qkv(n, kv, H, Hk, D, block=128, q_start=q_start, seed=7, strength=strength, hot=3)
    qd, kd, vd = q.to(DEV), k.to(DEV), v.to(DEV)
    sp = ksp.SparsePrefill(H, Hk, D, DEV, tau=0.95, min_kv=0, min_q=0, kernel='sm120fp8')
    km = ksp._cached_block_means('c1', 0, kd[q_start:], q_start, kv, key_all=kd)
    scales = ksp._cached_scales('c1', 0, qd, kd, vd, q_start)
    out = sp.forward_sm120fp8(qd, kd, vd, q_start, km=km, scales=scales)
    torch.cuda.synchronize()
    from sm120_attn import ops
    ops.check_status(DEV)
    qf, kf, vf = f32(q), f32(k), f32(v)
    km_o = O.KMeanCacheOracle(128).update('c1', 0, kf[q_start:], q_start, kv, key_all=kf)
    np.testing.assert_allclose(f32(km), km_o, rtol=2e-6, atol=2e-7)
    qm = O.q_block_means(qf, q_start, 128)
    ref_masks, aux = O.select_masks(qm, km_o, q_start, 128, H, Hk, 0.95, return_aux=True)
    got = sp.block_masks(qd, None, q_start, union=False, km=km).cpu().numpy()
    nbad, unexplained = O.compare_masks(got, ref_masks, aux, 0.95, Hk)
    assert not unexplained, (nbad, unexplained[:5])
    kept = sp.kept_fraction()
    assert abs(kept - got.sum() / O.causal_blocks(q_start, n // 128, 128) / H) < 1e-9
    inv = [np.float32(1.0 / s) for s in scales]
    deq = [O.e4m3_decode(O.quantize_glue(x, i)) * np.float32(s) for x, i, s in zip((qf, kf, vf), inv, scales)]
    hs = _heads_subset(H, H // Hk)
    refs = _per_head_ref(deq[0], deq[1], deq[2], q_start, got, hs, H // Hk, 128, 128)
    o = f32(out)
    assert rel_l2(np.stack([o[:, h] for h in hs], 1), np.stack([refs[h] for h in hs], 1)) < 3e-2


def _per_head_ref(q, k, v, q_pos0, masks, hs, g, q_block, kv_block, q_front=0):
    out = {}
    for h in hs:
        out[h] = O.attention_ref(q[:, h:h + 1], k[:, h // g:h // g + 1], v[:, h // g:h // g + 1], q_pos0,
                                 masks[h:h + 1], q_block=q_block, kv_block=kv_block, q_front=q_front)[:, 0]
    return out


@pytest.mark.parametrize('q_start,n,kv_total', [(3072, 1024, 4096), (5000, 3000, 8000)])
def test_fp8_block64_pair_union(ksp, q_start, n, kv_total):
    """Reference default: BLOCK 64, 128-row query blocks as the union of two 64-row masks."""
    ksp.BLOCK = 64
    H, Hk, D = 16, 2, 128
    q, k, v, _ = synth.make_qkv(n, kv_total, H, Hk, D, block=64, q_start=q_start, seed=n, strength='strong')
    kv = q_start + n
    qd, kd, vd = q.to(DEV), k[:kv].to(DEV), v[:kv].to(DEV)
    sp = ksp.SparsePrefill(H, Hk, D, DEV, tau=0.95, min_kv=0, min_q=0)
    km = ksp._cached_block_means('p', 0, kd[q_start:], q_start, kv, key_all=kd)
    scales = ksp._cached_scales('p', 0, qd, kd, vd, q_start)
    out = sp.forward_sm120fp8(qd, kd, vd, q_start, km=km, scales=scales)
    torch.cuda.synchronize()
    qf, kf, vf = f32(q), f32(k[:kv]), f32(v[:kv])
    BM = 128
    front = q_start % BM
    M = -(-(front + n) // BM) * BM
    qs = q_start - front
    need = max(-(-kv // 64) * 64, qs + M)
    qm = np.zeros((M // 64, H, D), np.float32)
    b0, means = O.block_means(qf, q_start, 64)
    qm[b0 - qs // 64:b0 - qs // 64 + means.shape[1]] = means.transpose(1, 0, 2)
    km_o = O.KMeanCacheOracle(64).update('p', 0, kf[q_start:], q_start, kv, key_all=kf)
    m64, aux = O.select_masks(qm, km_o, qs, 64, H, Hk, 0.95, nb_total=need // 64, return_aux=True)
    ref_masks = O.pair_union(m64)
    # the kernel's masks: the glue's pair-union lists for this chunk
    from sm120_attn import ops
    from sm120_attn._native import SA_SELECT_PAIR_UNION
    counts = torch.empty(H * (M // BM), dtype=torch.int32, device=DEV)
    masks_d = torch.empty(H * (M // BM), need // 64, dtype=torch.uint8, device=DEV)
    ops.select(torch.from_numpy(qm).to(DEV), km, H, Hk, need // 64, qs // 64, D ** -0.5, 0.95, SA_SELECT_PAIR_UNION,
               counts=counts, masks=masks_d)
    got = masks_d.cpu().numpy().astype(bool).reshape(H, M // BM, -1)
    nbad, unexplained = O.compare_masks(got, ref_masks, aux, 0.95, Hk, pair=True)
    assert not unexplained, (nbad, unexplained[:5])
    inv = [np.float32(1.0 / s) for s in scales]
    deq = [O.e4m3_decode(O.quantize_glue(x, i)) * np.float32(s) for x, i, s in zip((qf, kf, vf), inv, scales)]
    hs = _heads_subset(H, H // Hk)
    refs = _per_head_ref(deq[0], deq[1], deq[2], q_start, got, hs, H // Hk, 128, 64, q_front=front)
    o = f32(out)
    assert rel_l2(np.stack([o[:, h] for h in hs], 1), np.stack([refs[h] for h in hs], 1)) < 3e-2


@pytest.mark.parametrize('block', [64, 128])
def test_bf16_glue_unaligned_chunks(ksp, block):
    """forward_sm120 over chunked prefill with unaligned boundaries (tests/test_sparse_prefill.py:40-48)."""
    ksp.BLOCK = block
    H, Hk, D, kv = 8, 2, 128, 9192
    _, k, v, _ = synth.make_qkv(16, kv, H, Hk, D, block=block, seed=5, strength='strong')
    kd, vd = k.to(DEV), v.to(DEV)
    sp = ksp.SparsePrefill(H, Hk, D, DEV, tau=0.95, min_kv=0, min_q=0, kernel='sm120')
    kc = O.KMeanCacheOracle(block)
    for q_start, n in ((0, 5000), (5000, 3192), (8192, 1000)):
        q, _, _, _ = synth.make_qkv(n, q_start + n, H, Hk, D, block=block, q_start=q_start, seed=q_start + 1,
                                    strength='strong', with_v=False)
        qd = q.to(DEV)
        km = ksp._cached_block_means('bf', 9, kd[q_start:q_start + n], q_start, q_start + n)
        km_o = kc.update('bf', 9, f32(k[q_start:q_start + n]), q_start, q_start + n)
        np.testing.assert_allclose(f32(km), km_o, rtol=2e-6, atol=2e-7)
        o = sp.forward_sm120(qd, kd[:q_start + n], vd[:q_start + n], q_start, km=km)
        front = q_start % block
        qpad = torch.cat([qd.new_zeros(front, H, D), qd])
        masks = sp.block_masks(torch.cat([qpad, qd.new_zeros((-(front + n)) % block, H, D)]), None, q_start - front,
                               valid=(front, n), union=False, km=km).cpu().numpy()
        refs = _per_head_ref(f32(q), f32(k[:q_start + n]), f32(v[:q_start + n]), q_start, masks, range(H), H // Hk,
                             block, block, q_front=front)
        ref = np.stack([refs[h] for h in range(H)], 1)
        assert np.abs(f32(o) - ref).max() < 2e-2, (q_start, n)


def test_cached_vs_direct_means_three_chunks(ksp):
    """tests/test_sparse_prefill.py:28-39: cached block means equal directly computed ones."""
    ksp.BLOCK = 64
    H, Hk, D, kv = 8, 2, 128, 3 * 2048
    _, k, v, _ = synth.make_qkv(16, kv, H, Hk, D, block=64, seed=2, strength='strong')
    kd, vd = k.to(DEV), v.to(DEV)
    sp = ksp.SparsePrefill(H, Hk, D, DEV, tau=0.95, min_kv=0, min_q=0, kernel='sm120')
    for c, q_start in enumerate((0, 2048, 4096)):
        n = 2048
        q, _, _, _ = synth.make_qkv(n, q_start + n, H, Hk, D, q_start=q_start, seed=c, with_v=False, strength='strong')
        qd = q.to(DEV)
        km = ksp._cached_block_means('three', 7, kd[q_start:q_start + n], q_start, q_start + n)
        nb = (q_start + n) // 64
        direct = kd[:nb * 64].view(nb, 64, Hk, D).float().mean(1).transpose(0, 1)
        assert (km - direct).abs().max().item() < 1e-5
        o_cached = sp.forward_sm120(qd, kd[:q_start + n], vd[:q_start + n], q_start, km=km)
        o_direct = sp.forward_sm120(qd, kd[:q_start + n], vd[:q_start + n], q_start)
        assert (o_cached.float() - o_direct.float()).abs().max().item() < 2e-2


def test_fp8_kv_cache_chunks_bit_identical(ksp):
    """The FP8 KV cache (each K/V row quantised once) gives the same output, bit for bit, as
    re-quantising the history on every chunk, over three chunks of one request."""
    ksp.BLOCK = 128
    ksp._KV8_CACHE.clear()
    H, Hk, D, n = 16, 2, 128, 1024
    kv_total = 3 * n + 512
    q, k, v, _ = synth.make_qkv(kv_total, kv_total, H, Hk, D, block=128, q_start=0, seed=17, strength='strong')
    qd, kd, vd = q.to(DEV), k.to(DEV), v.to(DEV)
    sp = ksp.SparsePrefill(H, Hk, D, DEV, tau=0.95, min_kv=0, min_q=0, kernel='sm120fp8')
    for q_start in (0, n, 2 * n + 512):
        kv_len = q_start + n
        qc = qd[q_start:kv_len]
        km = ksp._cached_block_means('kv8', 5, kd[q_start:kv_len], q_start, kv_len, key_all=kd)
        scales = ksp._cached_scales('kv8', 5, qc, kd[:kv_len], vd[:kv_len], q_start)
        o_plain = sp.forward_sm120fp8(qc, kd[:kv_len], vd[:kv_len], q_start, km=km, scales=scales)
        kv8 = ksp._cached_kv8('kv8', 5, kd, vd, q_start, kv_len, scales)
        o_cache = sp.forward_sm120fp8(qc, kd[:kv_len], vd[:kv_len], q_start, km=km, scales=scales, kv8=kv8)
        torch.cuda.synchronize()
        assert torch.equal(o_plain, o_cache), q_start
    ksp._KV8_CACHE.clear()


def test_fp8_per_head_scales_and_kv_cache(ksp):
    """Per-head e4m3 scales (SM120_SPARSE_FP8_SCALES=head): output within the FP8 bars of the fp32
    reference and of the P-rounding model on per-head dequantised operands, and the FP8 KV cache
    with per-head scales bit-identical to re-quantising the history."""
    from kmodel import fp8_model_kwargs
    ksp.BLOCK = 128
    ksp._KV8_CACHE.clear()
    H, Hk, D, n = 16, 2, 128, 1024
    kv_total = 2 * n + 256
    q, k, v, _ = synth.make_qkv(kv_total, kv_total, H, Hk, D, block=128, q_start=0, seed=23, strength='strong')
    qd, kd, vd = q.to(DEV), k.to(DEV), v.to(DEV)
    sp = ksp.SparsePrefill(H, Hk, D, DEV, tau=0.95, min_kv=0, min_q=0, kernel='sm120fp8')
    for q_start in (0, n + 256):
        kv_len = q_start + n
        qc = qd[q_start:kv_len]
        km = ksp._cached_block_means('ph', 3, kd[q_start:kv_len], q_start, kv_len, key_all=kd)
        scales = ksp._cached_scales('ph', 3, qc, kd[:kv_len], vd[:kv_len], q_start, per_head=True)
        assert len(scales[0]) == H and len(scales[1]) == Hk
        o_plain = sp.forward_sm120fp8(qc, kd[:kv_len], vd[:kv_len], q_start, km=km, scales=scales)
        kv8 = ksp._cached_kv8('ph', 3, kd, vd, q_start, kv_len, scales)
        o_cache = sp.forward_sm120fp8(qc, kd[:kv_len], vd[:kv_len], q_start, km=km, scales=scales, kv8=kv8)
        torch.cuda.synchronize()
        from sm120_attn import ops
        ops.check_status(DEV)
        assert torch.equal(o_plain, o_cache), q_start
    # oracle on the last chunk: per-head quantised operands, the kernel's lists
    sq, sk, sv = (np.asarray(x, np.float32) for x in scales)
    qf, kf, vf = f32(q)[q_start:kv_len], f32(k)[:kv_len], f32(v)[:kv_len]
    q8 = O.quantize_glue(qf, (1.0 / sq).astype(np.float32))
    k8 = O.quantize_glue(kf, (1.0 / sk).astype(np.float32))
    v8 = O.quantize_glue(vf, (1.0 / sv).astype(np.float32))
    deq = [O.e4m3_decode(b) * s[None, :, None] for b, s in ((q8, sq), (k8, sk), (v8, sv))]
    counts, lists = sp.last_counts.cpu().numpy(), sp.last_lists.cpu().numpy()
    n_tiles = n // 128
    masks = np.zeros((H * n_tiles, lists.shape[1]), dtype=bool)
    for r in range(H * n_tiles):
        masks[r, lists[r, :counts[r]]] = True
    masks = masks.reshape(H, n_tiles, -1)
    got = f32(o_plain)
    ref = O.attention_ref(*deq, q_start, masks, q_block=128, kv_block=128)
    model = O.attention_fp8_kernel_model(q8, k8, v8, sq, sk, sv, q_start, counts, lists, q_block=128, kv_block=128,
                                         **fp8_model_kwargs(H, Hk, n_tiles))
    assert rel_l2(got, model) < 1e-2, rel_l2(got, model)
    assert rel_l2(got, ref) < 3e-2, rel_l2(got, ref)
    ksp._KV8_CACHE.clear()


def test_stale_first_page(ksp):
    """tests/test_sparse_prefill.py:65-92: a recycled first page never supplies stale means or scales."""
    ksp.BLOCK = 64
    H, Hk, D = 8, 2, 128
    torch.manual_seed(1)
    _, kA, _, _ = synth.make_qkv(16, 16384, H, Hk, D, seed=41, with_v=False)
    kA = kA.to(DEV)
    for q_start, n in ((0, 8192), (8192, 8192)):
        ksp._cached_block_means('L2', 3, kA[q_start:q_start + n], q_start, q_start + n)
    qA = torch.randn(8192, H, D, device=DEV, dtype=torch.bfloat16)
    ksp._cached_scales('L2', 3, qA, kA[:8192], kA[:8192] * 0.5, 0)
    kB = (torch.randn(8192, Hk, D, device=DEV) * 3.0).to(torch.bfloat16)
    km = ksp._cached_block_means('L2', 3, kB[1000:8192], 1000, 8192, key_all=kB[:8192])
    direct = kB.view(128, 64, Hk, D).float().mean(1).transpose(0, 1)
    assert (km - direct).abs().max().item() < 1e-2
    qB = torch.randn(7192, H, D, device=DEV, dtype=torch.bfloat16) * 4.0
    sB = ksp._cached_scales('L2', 3, qB, kB, kB * 0.5, 1000)
    fresh = tuple(t.float().abs().amax().item() * ksp.SCALE_MARGIN / 448.0 for t in (qB, kB, kB * 0.5))
    assert all(abs(a - b) < 1e-6 for a, b in zip(sB, fresh))
    ksp._cached_block_means('L2', 3, torch.randn(64, Hk, D, device=DEV, dtype=torch.bfloat16), 8192, 8256)
    assert ksp._KMEAN_CACHE[('L2', 3)]['last_kv'] == 8256


def test_glue_vs_direct_kernel_identical(ksp):
    """tests/test_sparse_prefill_fp8.py:19-31: glue and direct kernel agree for identical masks and scales."""
    ksp.BLOCK = 64
    from sm120_attn.kernels import attention_sm120_fp8, permute_vt_keys
    H, Hk, D, q_start, n = 8, 2, 128, 4096, 2048
    q, k, v, _ = synth.make_qkv(n, q_start + n, H, Hk, D, block=64, q_start=q_start, seed=3, strength='strong')
    qd, kd, vd = q.to(DEV), k.to(DEV), v.to(DEV)
    sp = ksp.SparsePrefill(H, Hk, D, DEV, tau=0.95, min_kv=0, min_q=0)
    km = kd.view(-1, 64, Hk, D).float().mean(1).transpose(0, 1).contiguous()
    masks = sp.block_masks(qd, None, q_start, union=False, km=km)
    m2 = masks.view(H, -1, 2, masks.shape[2]).any(2)
    counts = m2.sum(2).to(torch.int32).flatten()
    lists = torch.argsort((~m2).to(torch.int8), dim=-1, stable=True).to(torch.int32).reshape(-1, m2.shape[2])
    sq, sk, sv = (float(t.float().abs().amax().item()) / 448.0 for t in (qd, kd, vd))
    # the operands exactly as the glue quantises them: bf16 arithmetic (sparse_prefill.py:230-233)
    pre = ((qd * (1.0 / sq)).to(torch.float8_e4m3fn), sq, (kd * (1.0 / sk)).to(torch.float8_e4m3fn), sk,
           permute_vt_keys((vd * (1.0 / sv)).to(torch.float8_e4m3fn).permute(1, 2, 0)), sv)
    o_direct = attention_sm120_fp8(qd, kd, vd, q_start, counts=counts, lists=lists, prequant=pre, m_block=128)
    o_glue = sp.forward_sm120fp8(qd, kd, vd, q_start, scales=(sq, sk, sv))
    np.testing.assert_array_equal(f32(o_glue), f32(o_direct))


def test_dropin_kernels_match_reference_semantics():
    """attention_sm120 (64-row lists), attention_sm120_fp8 with and without prequant (permuted V^T)."""
    from sm120_attn.kernels import attention_sm120, attention_sm120_fp8, attention_sm120_fp8_tma, quantize_e4m3
    from sm120_attn.kernels import permute_vt_keys
    H, Hk, D, n, kv = 8, 2, 128, 512, 2048
    q, k, v, _ = synth.make_qkv(n, kv, H, Hk, D, seed=12)
    qd, kd, vd = q.to(DEV), k.to(DEV), v.to(DEV)
    rng = np.random.default_rng(0)
    MB, NB = n // 64, kv // 64
    masks = rng.random((H, MB, NB)) < 0.3
    gi = (kv - n) // 64 + np.arange(MB)
    for m in range(MB):
        masks[:, m, gi[m]] = True
        masks[:, m, gi[m] + 1:] = False
    masks[:, :, 0] = True
    counts, lists = O.masks_to_lists(masks)
    o16 = attention_sm120(qd, kd, vd, kv - n, counts=torch.from_numpy(counts).to(DEV),
                          lists=torch.from_numpy(lists).to(DEV))
    ref = O.attention_ref(f32(q), f32(k), f32(v), kv - n, masks, q_block=64, kv_block=64)
    assert np.abs(f32(o16) - ref).max() < 2e-2
    m128 = O.pair_union(masks)
    c128, l128 = O.masks_to_lists(m128)
    c128, l128 = torch.from_numpy(c128).to(DEV), torch.from_numpy(l128).to(DEV)
    o8 = attention_sm120_fp8(qd, kd, vd, kv - n, counts=c128, lists=l128)
    q8, sq = quantize_e4m3(qd)
    k8, sk = quantize_e4m3(kd)
    v8, sv = quantize_e4m3(vd)
    pre = (q8, sq, k8, sk, permute_vt_keys(v8.permute(1, 2, 0)), sv)
    o8p = attention_sm120_fp8_tma(qd, kd, vd, kv - n, counts=c128, lists=l128, prequant=pre)
    np.testing.assert_array_equal(f32(o8), f32(o8p))
    deq = [O.e4m3_decode(t.view(torch.uint8).cpu().numpy()) * np.float32(s) for t, s in ((q8, sq), (k8, sk), (v8, sv))]
    ref8 = O.attention_ref(*deq, kv - n, m128, q_block=128, kv_block=64)
    assert rel_l2(f32(o8), ref8) < 3e-2
    # dense
    o8d = attention_sm120_fp8(qd, kd, vd)
    assert rel_l2(f32(o8d), O.attention_ref(*deq, kv - n)) < 3e-2


@pytest.mark.parametrize('kernel,kv_cache,scale_mode,page', [('sm120fp8', False, 'tensor', 16),
                                                               ('sm120fp8', True, 'tensor', 16),
                                                               ('sm120fp8', True, 'head', 16),
                                                               ('sm120', False, 'tensor', 16),
                                                               ('sm120', False, 'tensor', 24)])
def test_try_sparse_forward_paged(ksp, monkeypatch, kernel, kv_cache, scale_mode, page):
    """The vLLM hook with a paged KV cache and fake metadata: eligible requests go through the sparse path
    and match a direct forward_sm120fp8 / forward_sm120 call on the gathered history (FP8 with and
    without the FP8 KV cache, per-tensor or per-head e4m3 scales; BF16 reading the pages in place, and
    gathering them for a page size the kernel does not read in place); the ineligible one is handed to
    _dense_request."""
    ksp.BLOCK = 64
    monkeypatch.setattr(ksp, '_CONFIG', {'enabled': True, 'tau': 0.95, 'min_kv': 2048, 'min_q': 512,
                                         'kernel': kernel, 'fp8_pipeline': 'tma', 'fp8_kv_cache': kv_cache,
                                         'fp8_scales': scale_mode})
    ksp._STATE.clear()
    dense_calls = []
    monkeypatch.setattr(ksp, '_dense_request', lambda *a: dense_calls.append(a[-2:]))
    H, Hk, D = 8, 2, 128
    reqs = [(1024, 3072), (16, 4000), (600, 2600)]          # (query len, kv len)
    npages = [-(-kv // page) for _, kv in reqs]
    nblocks = sum(npages) + 4
    g = torch.Generator(device=DEV)
    g.manual_seed(0)
    key_cache = torch.randn(nblocks, page, Hk, D, device=DEV, generator=g).to(torch.bfloat16)
    value_cache = torch.randn(nblocks, page, Hk, D, device=DEV, generator=g).to(torch.bfloat16)
    bt = torch.zeros(len(reqs), max(npages), dtype=torch.int32, device=DEV)
    perm = torch.randperm(nblocks, generator=torch.Generator().manual_seed(1))[:sum(npages)].to(torch.int32)
    off = 0
    for r, p in enumerate(npages):
        bt[r, :p] = perm[off:off + p].to(DEV)
        off += p
    qlens = [ql for ql, _ in reqs]
    qsl = torch.tensor(np.concatenate([[0], np.cumsum(qlens)]), dtype=torch.int32, device=DEV)
    T = int(qsl[-1])
    query = torch.randn(T, H, D, device=DEV, generator=g).to(torch.bfloat16)
    key = torch.empty(T, Hk, D, dtype=torch.bfloat16, device=DEV)
    for r, (ql, kv) in enumerate(reqs):
        kfull = key_cache[bt[r, :npages[r]].long()].reshape(-1, Hk, D)
        key[qsl[r]:qsl[r + 1]] = kfull[kv - ql:kv]
    output = torch.zeros(T, H, D, dtype=torch.bfloat16, device=DEV)
    meta = types.SimpleNamespace(causal=True, max_query_len=max(qlens), max_seq_len=max(kv for _, kv in reqs),
                                 query_start_loc=qsl, seq_lens=torch.tensor([kv for _, kv in reqs], dtype=torch.int32,
                                                                            device=DEV), block_table=bt)
    impl = types.SimpleNamespace(sliding_window=(-1, -1), scale=D ** -0.5)
    assert ksp.try_sparse_forward(impl, query, key, key_cache, value_cache, output, meta) is True
    assert dense_calls == [(16, 4000)]
    sp2 = ksp.SparsePrefill(H, Hk, D, DEV, tau=0.95, min_kv=0, min_q=0)
    for r in (0, 2):
        ql, kv = reqs[r]
        kfull = key_cache[bt[r, :npages[r]].long()].reshape(-1, Hk, D)
        vfull = value_cache[bt[r, :npages[r]].long()].reshape(-1, Hk, D)
        q_r = query[qsl[r]:qsl[r + 1]]
        full = kv // 64
        km = torch.zeros(Hk, -(-kv // 64), D, device=DEV)
        km[:, :full] = kfull[:full * 64].float().view(full, 64, Hk, D).mean(1).transpose(0, 1)
        if kv % 64:      # the hook's cache path averages a partial last block over its present rows
            km[:, full] = kfull[full * 64:kv].float().mean(0)
        if kernel == 'sm120':
            o = sp2.forward_sm120(q_r, kfull, vfull, kv - ql, km=km.contiguous())
            assert rel_l2(f32(output[qsl[r]:qsl[r + 1]]), f32(o)) < 1e-6
            continue
        if scale_mode == 'head':
            scales = tuple(tuple(float(a) * ksp.SCALE_MARGIN / 448.0 for a in t.float().abs().amax(dim=(0, 2)).tolist())
                           for t in (q_r, kfull[:kv], vfull[:kv]))
        else:
            scales = tuple(float(t.float().abs().amax()) * ksp.SCALE_MARGIN / 448.0
                           for t in (q_r, kfull[:kv], vfull[:kv]))
        o = sp2.forward_sm120fp8(q_r, kfull, vfull, kv - ql, km=km.contiguous(), scales=scales)
        assert rel_l2(f32(output[qsl[r]:qsl[r + 1]]), f32(o)) < 1e-6
    assert torch.all(output[qsl[1]:qsl[2]] == 0)
    assert len(ksp._KV8_CACHE) == (2 if kv_cache else 0)


def test_hook_fp8_kv_cache_reads_only_chunk_pages(ksp, monkeypatch):
    """Three chunks of one request through the vLLM hook (1000-row chunks: boundaries off the page
    and block grid).  With the FP8 KV cache on, chunks after the first read only their own rows (the
    block means, scales and e4m3 history are cached): the chunk's keys once, for their block means
    and e4m3 copy together, and its values from the pages.  The output is the same, bit for bit, as
    the path that re-quantises the whole history from the pages every chunk."""
    ksp.BLOCK = 64
    H, Hk, D, page, n, chunks = 8, 2, 128, 16, 1000, 3
    total = n * chunks
    npages_all = -(-total // page)
    q, k, v, _ = synth.make_qkv(total, total, H, Hk, D, block=64, q_start=0, seed=23, strength='strong')
    qd, kd, vd = q.to(DEV), k.to(DEV), v.to(DEV)
    perm = torch.randperm(npages_all + 5, generator=torch.Generator().manual_seed(4))[:npages_all].to(DEV)
    key_cache = torch.zeros(npages_all + 5, page, Hk, D, dtype=torch.bfloat16, device=DEV)
    value_cache = torch.zeros_like(key_cache)
    key_cache[perm.long()] = F.pad(kd, (0, 0, 0, 0, 0, npages_all * page - total)).view(npages_all, page, Hk, D)
    value_cache[perm.long()] = F.pad(vd, (0, 0, 0, 0, 0, npages_all * page - total)).view(npages_all, page, Hk, D)
    bt = perm.to(torch.int32).view(1, -1)
    calls = []
    real_q, real_m = ksp.ops.quantize_paged, ksp.ops.block_means

    def spy_q(cache, table, row0, scale, mode, out):
        calls.append(('q', row0, out.shape[0]))
        return real_q(cache, table, row0, scale, mode, out)

    def spy_m(x, pos0, block, out, out_block0, q8=None, inv_scale=None, fixed_divisor=0):
        calls.append(('m', pos0, x.shape[0], q8 is not None))
        return real_m(x, pos0, block, out, out_block0, q8=q8, inv_scale=inv_scale, fixed_divisor=fixed_divisor)
    monkeypatch.setattr(ksp.ops, 'quantize_paged', spy_q)
    monkeypatch.setattr(ksp.ops, 'block_means', spy_m)
    outs, log = {}, {}
    for kv_cache in (False, True):
        monkeypatch.setattr(ksp, '_CONFIG', {'enabled': True, 'tau': 0.95, 'min_kv': 512, 'min_q': 512,
                                             'kernel': 'sm120fp8', 'fp8_pipeline': 'tma', 'fp8_kv_cache': kv_cache})
        ksp._STATE.clear()
        impl = types.SimpleNamespace(sliding_window=(-1, -1), scale=D ** -0.5)
        outs[kv_cache] = []
        for c in range(chunks):
            c0, kv_len = c * n, (c + 1) * n
            meta = types.SimpleNamespace(causal=True, max_query_len=n, max_seq_len=kv_len,
                                         query_start_loc=torch.tensor([0, n], dtype=torch.int32, device=DEV),
                                         seq_lens=torch.tensor([kv_len], dtype=torch.int32, device=DEV), block_table=bt)
            out = torch.zeros(n, H, D, dtype=torch.bfloat16, device=DEV)
            calls.clear()
            assert ksp.try_sparse_forward(impl, qd[c0:kv_len], kd[c0:kv_len], key_cache, value_cache, out, meta)
            outs[kv_cache].append(out)
            log[kv_cache, c] = list(calls)
    torch.cuda.synchronize()
    for a, b in zip(outs[False], outs[True]):
        assert torch.equal(a, b)
    for c in range(chunks):
        c0, kv_len = c * n, (c + 1) * n
        # cache off: every chunk quantises the whole history from the pages (no gather)
        assert [x for x in log[False, c] if x[0] == 'q'] == [('q', 0, kv_len), ('q', 0, kv_len)]
        if c == 0:                 # cache on, first chunk: the entry is built from the pages
            assert [x for x in log[True, c] if x[0] == 'q'] == [('q', 0, kv_len), ('q', 0, kv_len)]
        else:                      # later chunks: keys once (means + e4m3 together), values' own rows
            assert [x for x in log[True, c] if x[0] == 'q'] == [('q', c0, n)]
            assert ('m', c0, n, True) in log[True, c]
