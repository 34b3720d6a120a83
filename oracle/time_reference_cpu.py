"""Times the reference's own CPU path beside this repository's restatement of it (test infrastructure).

The GPU host has no reference checkout, so bench.py's CPU baseline (`cpu_baseline`, `--impl reference`)
times the restatement in oracle/ (numpy selection, fp32 attention on all host threads).  This script,
run where the reference checkout exists, times
the reference's own PyTorch path on the same bounded sample -- `SparsePrefill.block_masks` (selection,
sm120_attn/sparse_prefill.py:42-85) over the whole configs[1] chunk of one KV-head group, then
`reference()` (masked fp32 attention, sparse_prefill.py:262-279) of the last query blocks -- and the
oracle on the identical sample, and prints both rates (executed-block TFLOPS, the benchmark's metric)
with the agreement of their masks.

    python oracle/time_reference_cpu.py --reference PATH [--strength unit|strong] [--rows 256]
"""
from __future__ import annotations

import argparse
import sys
import time
from pathlib import Path

import numpy as np
import torch

ROOT = Path(__file__).resolve().parent.parent
sys.path.insert(0, str(ROOT))
sys.path.insert(0, str(ROOT / 'tests'))

import oracle as O  # noqa: E402
import synth  # noqa: E402

H, HK, D = 8, 1, 128                      # one KV-head group of configs[1] (64 / 8 heads)
N_Q, KV, BLOCK, TAU = 8192, 65536, 128, 0.95
Q_START = KV - N_Q


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument('--reference', required=True, help='checkout of the reference repository')
    ap.add_argument('--strength', default='unit', choices=['unit', 'strong'])
    ap.add_argument('--rows', type=int, default=256)
    args = ap.parse_args()
    sys.path.insert(0, args.reference)
    import sm120_attn.sparse_prefill as ref                 # the reference package, not this repository's
    assert Path(ref.__file__).resolve().is_relative_to(Path(args.reference).resolve()), ref.__file__
    ref.BLOCK = BLOCK
    q, k, v, _ = synth.make_qkv(N_Q, KV, H, HK, D, block=BLOCK, q_start=Q_START, seed=1000, strength=args.strength,
                                hot=6)
    qf, kf, vf = (t.float() for t in (q, k, v))
    n_blocks = N_Q // BLOCK
    sample = list(range(n_blocks - 1, n_blocks - 1 - args.rows // BLOCK, -1))

    # the reference: selection over the whole chunk, then masked fp32 attention of the sampled blocks
    sp = ref.SparsePrefill(H, HK, D, 'cpu', tau=TAU, min_kv=0, min_q=0)
    t0 = time.perf_counter()
    masks_ref = sp.block_masks(qf, kf, Q_START)             # [Hk, MB, NB] (union over the group)
    t_sel_ref = time.perf_counter() - t0
    heads_ref = sp.block_masks(qf, kf, Q_START, union=False)   # [H, MB, NB], for the mask comparison
    kh, vh = kf.transpose(0, 1).contiguous(), vf.transpose(0, 1).contiguous()
    t_attn_ref, flops = 0.0, 0.0
    for m in sample:
        r0 = m * BLOCK
        t0 = time.perf_counter()
        ref.reference(qf[r0:r0 + BLOCK], kh, vh, Q_START + r0, masks=masks_ref[:, m:m + 1])
        t_attn_ref += time.perf_counter() - t0
        flops += 4.0 * D * BLOCK * BLOCK * float(heads_ref[:, m].sum())
    rows = len(sample) * BLOCK
    tf_ref = flops / (t_attn_ref + t_sel_ref * rows / N_Q) / 1e12

    # the oracle (the CPU baseline bench.py times on the GPU host), same sample
    qn, kn, vn = qf.numpy(), kf.numpy(), vf.numpy()
    t0 = time.perf_counter()
    kc = O.KMeanCacheOracle(BLOCK)
    kc.update('t', 0, kn[:Q_START], 0, Q_START)
    km = kc.update('t', 0, kn[Q_START:], Q_START, KV)
    qm = O.q_block_means(qn, Q_START, BLOCK)
    masks_o = O.select_masks(qm, km, Q_START, BLOCK, H, HK, TAU)
    t_sel_o = time.perf_counter() - t0
    t_attn = {}
    for fn in (O.attention_ref, O.attention_ref_threaded):
        t_attn[fn.__name__] = 0.0
        for m in sample:
            r0 = m * BLOCK
            t0 = time.perf_counter()
            fn(qn[r0:r0 + BLOCK], kn, vn, Q_START + r0, masks_o[:, m:m + 1], q_block=BLOCK, kv_block=BLOCK)
            t_attn[fn.__name__] += time.perf_counter() - t0
    same = np.array_equal(heads_ref.numpy(), masks_o)
    print(f'threads {torch.get_num_threads()}; sample: selection of the whole chunk (1 KV head x {H} query heads) '
          f'+ attention of the last {rows} query rows; {args.strength} injection')
    print(f'reference (block_masks + reference(), PyTorch fp32): selection {t_sel_ref:.2f} s, attention '
          f'{t_attn_ref:.2f} s -> {tf_ref:.6f} TFLOPS')
    for name, t in t_attn.items():
        tf_o = flops / (t + t_sel_o * rows / N_Q) / 1e12
        print(f'oracle, selection (numpy) + {name:24s}: selection {t_sel_o:.2f} s, attention {t:.2f} s -> '
              f'{tf_o:.6f} TFLOPS ({tf_o / tf_ref:.3f} of the reference)')
    print(f'per-head masks identical to the reference\'s: {same}')


if __name__ == '__main__':
    main()
