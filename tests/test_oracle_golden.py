"""Pin the numpy oracle to golden vectors produced by the reference's own PyTorch code (CPU only)."""
from __future__ import annotations

import zlib

import numpy as np
import pytest
import torch

import oracle as O
import synth
from conftest import unpack_mask
from golden.gen_golden import CACHE_SEQS, H, HK, D, SEL_CASES  # noqa: E402


def f32(t):
    return t.float().numpy()


@pytest.mark.parametrize('case', SEL_CASES, ids=[c[0] for c in SEL_CASES])
def test_selection_matches_reference(golden, case):
    name, block, kv, q_start, n, strength, hot = case
    q, k, v, _ = synth.make_qkv(n, kv, H, HK, D, block=block, q_start=q_start,
                                seed=zlib.crc32(name.encode()) % 1000, strength=strength, hot=hot)
    assert synth.checksum(q) == golden[f'{name}/fp_q'], 'input generator drifted'
    assert synth.checksum(k) == golden[f'{name}/fp_k'], 'input generator drifted'
    kc = O.KMeanCacheOracle(block)
    km = kc.update('golden', 1, f32(k[q_start:q_start + n]), q_start, q_start + n, key_all=f32(k))
    np.testing.assert_allclose(km, golden[f'{name}/km'], rtol=2e-6, atol=2e-7)
    qm = O.q_block_means(f32(q), q_start, block)
    qs = q_start - q_start % block
    for union, key in ((False, 'masks'), (True, 'umasks')):
        ref = unpack_mask(golden, f'{name}/{key}')
        m, aux = O.select_masks(qm, golden[f'{name}/km'], qs, block, H, HK, 0.95, union=union, return_aux=True)
        assert m.shape == ref.shape
        if not union:
            nbad, unexplained = O.compare_masks(m, ref, aux, 0.95, HK)
            assert not unexplained, (nbad, unexplained[:5])
        else:
            assert (m != ref).mean() < 1e-3
    if block == 64:
        BM = 128
        front8 = q_start % BM
        M = -(-(front8 + n) // BM) * BM
        qs8 = q_start - front8
        need = max(-(-(q_start + n) // block) * block, qs8 + M)
        qm8 = np.zeros((M // block, H, D), np.float32)
        _, means = O.block_means(f32(q), q_start, block)
        b0 = q_start // block - qs8 // block
        qm8[b0:b0 + means.shape[1]] = means.transpose(1, 0, 2)
        m, aux = O.select_masks(qm8, golden[f'{name}/km'], qs8, block, H, HK, 0.95, nb_total=need // block,
                                return_aux=True)
        mu = O.pair_union(m)
        ref = unpack_mask(golden, f'{name}/fp8_masks')
        nbad, unexplained = O.compare_masks(mu, ref, aux, 0.95, HK, pair=True)
        assert not unexplained, (nbad, unexplained[:5])
        counts, lists = O.masks_to_lists(ref)
        np.testing.assert_array_equal(counts, golden[f'{name}/fp8_counts'])
        for r in range(len(counts)):
            np.testing.assert_array_equal(lists[r, :counts[r]], golden[f'{name}/fp8_lists'][r, :counts[r]])


@pytest.mark.parametrize('name', sorted(CACHE_SEQS))
def test_kmean_cache_sequence(golden, name):
    block, seq = CACHE_SEQS[name]
    kv = seq[-1][0] + seq[-1][1]
    _, k, _, _ = synth.make_qkv(16, kv, H, HK, D, block=block, seed=11, strength='strong', with_v=False)
    assert synth.checksum(k) == golden[f'{name}/fp_k']
    kc = O.KMeanCacheOracle(block)
    for i, (q_start, n) in enumerate(seq):
        km = kc.update('L', 7, f32(k[q_start:q_start + n]), q_start, q_start + n)
        np.testing.assert_allclose(km, golden[f'{name}/step{i}'], rtol=2e-6, atol=2e-7)
        assert kc.entries[('L', 7)]['last_kv'] == golden[f'{name}/last_kv{i}']


def test_kmean_cache_stale_first_page(golden):
    kc = O.KMeanCacheOracle(64)
    _, kA, _, _ = synth.make_qkv(16, 4096, H, HK, D, block=64, seed=21, with_v=False)
    _, kB, _, _ = synth.make_qkv(16, 2048, H, HK, D, block=64, seed=22, with_v=False)
    kB = (kB.float() * 3.0).to(torch.bfloat16)
    for q_start, n in ((0, 2048), (2048, 2048)):
        kc.update('L2', 3, f32(kA[q_start:q_start + n]), q_start, q_start + n)
    km = kc.update('L2', 3, f32(kB[500:2048]), 500, 2048, key_all=f32(kB[:2048]))
    np.testing.assert_allclose(km, golden['stale/km'], rtol=2e-6, atol=2e-7)
    nxt = synth.make_qkv(16, 64, H, HK, D, block=64, seed=23, with_v=False)[1]
    km2 = kc.update('L2', 3, f32(nxt), 2048, 2112)
    np.testing.assert_allclose(km2, golden['stale/km2'], rtol=2e-6, atol=2e-7)
    assert kc.entries[('L2', 3)]['last_kv'] == golden['stale/last_kv']
    kc2 = O.KMeanCacheOracle(64)
    km3 = kc2.update('L3', 5, f32(kA[1000:2000]), 1000, 2000, key_all=f32(kA[:2000]))
    np.testing.assert_allclose(km3, golden['rebuild_unaligned/km'], rtol=2e-6, atol=2e-7)
    with pytest.raises(RuntimeError):
        O.KMeanCacheOracle(64).update('L', 1, f32(kA[64:128]), 64, 128)


def test_scale_cache(golden):
    q, k, v, _ = synth.make_qkv(512, 2048, H, HK, D, block=64, seed=31)
    sc = O.ScaleCacheOracle()
    s0 = sc.update('L', 3, f32(q), f32(k[:1536]), f32(v[:1536]), 1024)
    s1 = sc.update('L', 3, f32(q), f32(k[:2048]), f32((v[:2048] * 2)), 1536)
    s2 = sc.update('L', 3, f32(q * 4), f32(k), f32(v), 1000)
    np.testing.assert_allclose(np.array([s0, s1, s2]), golden['scales/s'], rtol=1e-12)


def test_attention_reference(golden):
    for name, n, kv in (('attn_dense_a', 100, 300), ('attn_dense_b', 128, 128)):
        q, k, v, _ = synth.make_qkv(n, kv, 4, 2, D, seed=41 + n)
        out = O.attention_ref(f32(q), f32(k), f32(v), kv - n)
        np.testing.assert_allclose(out, golden[f'{name}/out'], rtol=1e-4, atol=2e-5)
    n, kv = 256, 1024
    q, k, v, _ = synth.make_qkv(n, kv, 4, 2, D, seed=51)
    masks = unpack_mask(golden, 'attn_sparse/masks')
    out = O.attention_ref(f32(q), f32(k), f32(v), kv - n, masks, q_block=64, kv_block=64)
    np.testing.assert_allclose(out, golden['attn_sparse/out'], rtol=1e-4, atol=2e-5)


def test_threaded_attention_matches_golden(golden):
    """attention_ref_threaded (the CPU baseline's attention, PyTorch on all host threads) gives the
    reference's outputs like attention_ref, dense and block-masked, including a chunk starting inside
    a query block (q_front) and a mask narrower than the keys."""
    for name, n, kv in (('attn_dense_a', 100, 300), ('attn_dense_b', 128, 128)):
        q, k, v, _ = synth.make_qkv(n, kv, 4, 2, D, seed=41 + n)
        out = O.attention_ref_threaded(f32(q), f32(k), f32(v), kv - n)
        np.testing.assert_allclose(out, golden[f'{name}/out'], rtol=1e-4, atol=2e-5)
    n, kv = 256, 1024
    q, k, v, _ = synth.make_qkv(n, kv, 4, 2, D, seed=51)
    masks = unpack_mask(golden, 'attn_sparse/masks')
    out = O.attention_ref_threaded(f32(q), f32(k), f32(v), kv - n, masks, q_block=64, kv_block=64)
    np.testing.assert_allclose(out, golden['attn_sparse/out'], rtol=1e-4, atol=2e-5)
    rng = np.random.default_rng(3)
    q, k, v, _ = synth.make_qkv(300, 1500, 4, 2, D, seed=9)
    m = rng.random((4, 4, 23)) < 0.5                     # 23 blocks of 64 < 1500 keys: the rest masked
    m[:, :, 0] = True
    a = O.attention_ref(f32(q), f32(k), f32(v), 1200, m, q_block=128, kv_block=64, q_front=77)
    b = O.attention_ref_threaded(f32(q), f32(k), f32(v), 1200, m, q_block=128, kv_block=64, q_front=77)
    np.testing.assert_allclose(b, a, rtol=1e-5, atol=1e-6)


def test_fp8_reference_operands(golden):
    n, kv = 128, 512
    q, k, v, _ = synth.make_qkv(n, kv, 4, 2, D, seed=61)
    sq, sk, sv = golden['attn_fp8/scales']
    for t, s, key in ((q, sq, 'q8'), (k, sk, 'k8'), (v, sv, 'v8')):
        bits, scale = O.quantize_per_tensor(f32(t))
        assert scale == pytest.approx(s, rel=0, abs=0)
        np.testing.assert_array_equal(bits, golden[f'attn_fp8/{key}'])
    deq = [O.bf16_round(O.e4m3_decode(golden[f'attn_fp8/{x}']) * np.float32(s))
           for x, s in (('q8', sq), ('k8', sk), ('v8', sv))]
    out = O.attention_ref(*deq, kv - n)
    np.testing.assert_allclose(out, golden['attn_fp8/out'], rtol=1e-4, atol=2e-5)


def test_fp8_kernel_model_close_to_reference(golden):
    """The P-rounding model of the FP8 kernel stays within the FP8 tolerance of the fp32 reference."""
    sq, sk, sv = golden['attn_fp8/scales']
    n, kv = 128, 512
    out = O.attention_fp8_kernel_model(golden['attn_fp8/q8'], golden['attn_fp8/k8'], golden['attn_fp8/v8'],
                                       sq, sk, sv, kv - n)
    ref = golden['attn_fp8/out']
    rel = np.linalg.norm(out - ref) / np.linalg.norm(ref)
    assert rel < 3e-2, rel


def test_quantisation_bits(golden):
    q, k, v, _ = synth.make_qkv(256, 256, 4, 2, D, seed=71, strength='strong')
    for i, s in enumerate((0.0123, 0.5 / 448.0, 7.1 / 448.0)):
        x = q if i != 1 else k
        bits = O.quantize_glue(f32(x), np.float32(1.0 / s))
        ref = golden[f'quant/glue{i}']
        np.testing.assert_array_equal(bits, ref)
    bits, s = O.quantize_per_tensor(f32(v))
    assert s == golden['quant/pt_scale']
    np.testing.assert_array_equal(bits, golden['quant/pt_bits'])
    vt = np.arange(2 * 3 * 64, dtype=np.int16).reshape(2, 3, 64)
    np.testing.assert_array_equal(O.permute_vt_keys(vt), golden['quant/perm'])
    assert list(golden['quant/VT_KEY_PERM']) == O.VT_KEY_PERM


def test_e4m3_roundtrip_all_codes():
    codes = np.arange(256, dtype=np.uint8)
    vals = O.e4m3_decode(codes)
    finite = ~np.isnan(vals)
    back = O.e4m3_encode(vals[finite])
    # +0 and -0 both decode to 0; compare values not codes for the zeros
    np.testing.assert_array_equal(O.e4m3_decode(back), vals[finite])
    t = torch.from_numpy(vals[finite]).to(torch.float8_e4m3fn).view(torch.uint8).numpy()
    np.testing.assert_array_equal(t[vals[finite] != 0], back[vals[finite] != 0])
