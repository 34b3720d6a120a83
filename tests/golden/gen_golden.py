"""Generate the golden vectors that pin the oracle to the reference.

Runs the reference's own PyTorch code (accion-intelligence/Qwen38-sparse-attn, imported from a
local checkout given by --reference) on CPU, on seeded inputs from `tests/synth.py`, and writes
`tests/golden/golden.npz`.  Only outputs and input fingerprints are stored; the tests regenerate
the inputs from the same seeds and check the fingerprints first.

    python tests/golden/gen_golden.py --reference <path to the reference checkout>

The reference is never needed at test time.
"""
from __future__ import annotations

import argparse
import importlib
import zlib
import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parent))
import synth  # noqa: E402

H, HK, D = 8, 2, 128

# (name, block, kv_len, q_start, n, strength, hot)
SEL_CASES = [
    ('sel_b128_unit', 128, 4096, 3072, 1024, 'unit', 3),
    ('sel_b128_strong', 128, 4096, 3072, 1024, 'strong', 3),
    ('sel_b128_unaligned', 128, 4000, 3000, 1000, 'strong', 3),
    ('sel_b64_unit', 64, 4096, 3072, 1024, 'unit', 3),
    ('sel_b64_strong', 64, 4096, 3072, 1024, 'strong', 3),
    ('sel_b64_unaligned', 64, 4000, 3000, 1000, 'strong', 3),
    ('sel_b64_tail', 64, 3000, 2000, 1000, 'strong', 3),
]
CACHE_SEQS = {
    'kc_b64': (64, [(0, 1000), (1000, 1500), (2500, 1596)]),
    'kc_b128': (128, [(0, 1000), (1000, 1500), (2500, 1596)]),
}


def _bf(t):
    return t.to(torch.bfloat16)


def gen_selection(ksp, out):
    for name, block, kv, q_start, n, strength, hot in SEL_CASES:
        ksp.BLOCK = block
        q, k, v, _ = synth.make_qkv(n, kv, H, HK, D, block=block, q_start=q_start, seed=zlib.crc32(name.encode()) % 1000,
                                    strength=strength, hot=hot)
        out[f'{name}/fp_q'] = np.float64(synth.checksum(q))
        out[f'{name}/fp_k'] = np.float64(synth.checksum(k))
        ksp._KMEAN_CACHE.clear()
        km = ksp._cached_block_means('golden', 1, k[q_start:q_start + n], q_start, q_start + n, key_all=k)
        out[f'{name}/km'] = km.numpy().astype(np.float32)
        sp = ksp.SparsePrefill(H, HK, D, 'cpu', tau=0.95, min_kv=0, min_q=0, kernel='sm120')
        front = q_start % block
        end = (-(front + n)) % block
        qp = torch.cat([q.new_zeros(front, H, D), q, q.new_zeros(end, H, D)])
        qs = q_start - front
        masks = sp.block_masks(qp, None, qs, valid=(front, n), union=False, km=km)
        out[f'{name}/masks'] = np.packbits(masks.numpy(), axis=-1)
        out[f'{name}/masks_shape'] = np.array(masks.shape)
        um = sp.block_masks(qp, None, qs, valid=(front, n), union=True, km=km)
        out[f'{name}/umasks'] = np.packbits(um.numpy(), axis=-1)
        out[f'{name}/umasks_shape'] = np.array(um.shape)
        if block == 64:
            # FP8 driver selection (sparse_prefill.py:199-225): 128-row padding, km padded, pair union
            BM = 128
            front8 = q_start % BM
            end8 = (-(front8 + n)) % BM
            q8p = torch.cat([q.new_zeros(front8, H, D), q, q.new_zeros(end8, H, D)])
            M = q8p.shape[0]
            MB = M // block
            qs8 = q_start - front8
            kk = k[:q_start + n]
            need = max(-(-kk.shape[0] // block) * block, qs8 + M)
            kmp = km
            if kmp.shape[1] < need // block:
                kmp = torch.nn.functional.pad(kmp, (0, 0, 0, need // block - kmp.shape[1]))
            m8 = sp.block_masks(q8p, None, qs8, valid=(front8, n), union=False, km=kmp)
            m8 = m8.view(H, MB // 2, 2, -1).any(2)
            counts = m8.sum(2).to(torch.int32).flatten()
            lists = torch.argsort((~m8).to(torch.int8), dim=-1, stable=True).to(torch.int32).reshape(H * (MB // 2), -1)
            out[f'{name}/fp8_counts'] = counts.numpy()
            out[f'{name}/fp8_lists'] = lists.numpy()
            out[f'{name}/fp8_masks'] = np.packbits(m8.numpy(), axis=-1)
            out[f'{name}/fp8_masks_shape'] = np.array(m8.shape)


def gen_cache(ksp, out):
    for name, (block, seq) in CACHE_SEQS.items():
        ksp.BLOCK = block
        ksp._KMEAN_CACHE.clear()
        kv = seq[-1][0] + seq[-1][1]
        _, k, _, _ = synth.make_qkv(16, kv, H, HK, D, block=block, seed=11, strength='strong', with_v=False)
        out[f'{name}/fp_k'] = np.float64(synth.checksum(k))
        for i, (q_start, n) in enumerate(seq):
            km = ksp._cached_block_means('L', 7, k[q_start:q_start + n], q_start, q_start + n)
            out[f'{name}/step{i}'] = km.numpy().astype(np.float32)
            out[f'{name}/last_kv{i}'] = np.int64(ksp._KMEAN_CACHE[('L', 7)]['last_kv'])
    # stale first page: request A fills page 3, request B reuses it after a short first chunk
    ksp.BLOCK = 64
    ksp._KMEAN_CACHE.clear()
    _, kA, _, _ = synth.make_qkv(16, 4096, H, HK, D, block=64, seed=21, with_v=False)
    _, kB, _, _ = synth.make_qkv(16, 2048, H, HK, D, block=64, seed=22, with_v=False)
    kB = _bf(kB.float() * 3.0)
    for q_start, n in ((0, 2048), (2048, 2048)):
        ksp._cached_block_means('L2', 3, kA[q_start:q_start + n], q_start, q_start + n)
    km = ksp._cached_block_means('L2', 3, kB[500:2048], 500, 2048, key_all=kB[:2048])
    out['stale/km'] = km.numpy().astype(np.float32)
    nxt = synth.make_qkv(16, 64, H, HK, D, block=64, seed=23, with_v=False)[1]
    km2 = ksp._cached_block_means('L2', 3, nxt, 2048, 2112)
    out['stale/km2'] = km2.numpy().astype(np.float32)
    out['stale/last_kv'] = np.int64(ksp._KMEAN_CACHE[('L2', 3)]['last_kv'])
    # rebuild with an unaligned boundary (q_start % BLOCK != 0 on a fresh entry)
    ksp._KMEAN_CACHE.clear()
    km3 = ksp._cached_block_means('L3', 5, kA[1000:2000], 1000, 2000, key_all=kA[:2000])
    out['rebuild_unaligned/km'] = km3.numpy().astype(np.float32)


def gen_scales(ksp, out):
    ksp._SCALE_CACHE.clear()
    q, k, v, _ = synth.make_qkv(512, 2048, H, HK, D, block=64, seed=31)
    s0 = ksp._cached_scales('L', 3, q, k[:1536], v[:1536], 1024)
    s1 = ksp._cached_scales('L', 3, q, k[:2048], v[:2048] * 2, 1536)           # continuity: reused
    s2 = ksp._cached_scales('L', 3, q * 4, k, v, 1000)                          # discontinuity: fresh
    out['scales/s'] = np.array([s0, s1, s2], dtype=np.float64)


def gen_attention(tfa, ksp, out):
    # dense causal, unaligned shapes (tests/test_fa_bf16.py:79-86 style, small)
    for name, n, kv in (('attn_dense_a', 100, 300), ('attn_dense_b', 128, 128)):
        q, k, v, _ = synth.make_qkv(n, kv, 4, 2, D, seed=41 + n)
        ref = tfa.reference(q, k, v, kv - n)
        out[f'{name}/out'] = ref.numpy().astype(np.float32)
    # block-sparse with random per-head masks (tests/test_fa_bf16.py:87-99 style)
    torch.manual_seed(5)
    n, kv = 256, 1024
    q, k, v, _ = synth.make_qkv(n, kv, 4, 2, D, seed=51)
    masks = tfa.random_masks(n, kv, kv - n, 4, 0.3, 'cpu')
    out['attn_sparse/masks'] = np.packbits(masks.numpy(), axis=-1)
    out['attn_sparse/masks_shape'] = np.array(masks.shape)
    out['attn_sparse/out'] = tfa.reference(q, k, v, kv - n, masks).numpy().astype(np.float32)
    # FP8: reference on the same e4m3-rounded operands (tests/test_fa_fp8.py:8-11)
    from sm120_attn.kernels.kai_fa_fp8 import quantize_e4m3
    n, kv = 128, 512
    q, k, v, _ = synth.make_qkv(n, kv, 4, 2, D, seed=61)
    q8, sq = quantize_e4m3(q)
    k8, sk = quantize_e4m3(k)
    v8, sv = quantize_e4m3(v)
    out['attn_fp8/q8'] = q8.view(torch.uint8).numpy()
    out['attn_fp8/k8'] = k8.view(torch.uint8).numpy()
    out['attn_fp8/v8'] = v8.view(torch.uint8).numpy()
    out['attn_fp8/scales'] = np.array([sq, sk, sv], dtype=np.float64)
    deq = [(t.float() * s).to(torch.bfloat16) for t, s in ((q8, sq), (k8, sk), (v8, sv))]
    out['attn_fp8/out'] = tfa.reference(*deq, kv - n).numpy().astype(np.float32)


def gen_quant(ksp, out):
    from sm120_attn.kernels.kai_fa_fp8 import permute_vt_keys, VT_KEY_PERM, quantize_e4m3
    q, k, v, _ = synth.make_qkv(256, 256, 4, 2, D, seed=71, strength='strong')
    for i, s in enumerate((0.0123, 0.5 / 448.0, 7.1 / 448.0)):
        x = q if i != 1 else k
        out[f'quant/glue{i}'] = (x * (1.0 / s)).to(torch.float8_e4m3fn).view(torch.uint8).numpy()
    x8, s = quantize_e4m3(v)
    out['quant/pt_bits'] = x8.view(torch.uint8).numpy()
    out['quant/pt_scale'] = np.float64(s)
    vt = torch.arange(2 * 3 * 64, dtype=torch.int16).reshape(2, 3, 64)
    out['quant/perm'] = permute_vt_keys(vt).numpy()
    out['quant/VT_KEY_PERM'] = np.array(VT_KEY_PERM)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument('--reference', required=True, help='path of the reference checkout (read only)')
    ap.add_argument('--out', default=str(HERE / 'golden.npz'))
    args = ap.parse_args()
    sys.path.insert(0, args.reference)
    sys.path.insert(0, str(Path(args.reference) / 'tests'))
    torch.set_num_threads(8)
    ksp = importlib.import_module('sm120_attn.sparse_prefill')
    tfa = importlib.import_module('test_fa_bf16')          # its `reference` and `random_masks`
    out = {}
    gen_selection(ksp, out)
    gen_cache(ksp, out)
    gen_scales(ksp, out)
    gen_attention(tfa, ksp, out)
    gen_quant(ksp, out)
    ksp.BLOCK = 64
    np.savez_compressed(args.out, **out)
    print(f'wrote {args.out}: {len(out)} arrays')


if __name__ == '__main__':
    main()
