"""Split walks of the FP8 attention kernel (sa_attn_fwd_fp8_split) on the GPU.

The units of the partial last wave (here: the last units of the launch order, chosen by the test) whose
walk is long enough are cut into contiguous step ranges run as separate CTAs and merged; the others
run whole.  Checks: against the fp32 oracle on the same e4m3 operands
(rel-L2 3e-2, the FP8 bar), against the oracle's P-rounding model of the split walk (rel-L2 1e-2, the
bar of the unsplit kernel against its model), against the unsplit kernel (rel-L2 4e-2: two independent
e4m3 roundings of P, each against its own running max), and unsplit units bit for bit equal to the
unsplit kernel's rows; dense and
list walks of 64- and 128-key blocks, a chunk starting inside a tile, rows with empty lists.  At the
per-rank shape of an 8-GPU strong split (8 query heads, 1 KV head, configs[1] chunk) the automatic
choice splits, and the glue's output stays within the bar of the unsplit run.
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

import oracle as O
from test_gpu_kernels import _deq, _fp8_case, _lists_from_masks, f32, rel_l2

pytestmark = pytest.mark.gpu
DEV = torch.device('cuda')


def _mixed_masks(H, n_tiles, NB, q_offset, kv_block, seed):
    """Per (head, tile): a nearly dense row (long walk) or a sparse one, plus sink and causal diagonal;
    one row left empty."""
    rng = np.random.default_rng(seed)
    dens = np.where(rng.random((H, n_tiles, 1)) < 0.5, 0.95, 0.1)
    m = rng.random((H, n_tiles, NB)) < dens
    for t in range(n_tiles):
        lo, hi = q_offset + t * 128, q_offset + t * 128 + 127
        for b in range(NB):
            if b * kv_block > hi:
                m[:, t, b] = False
            elif (b + 1) * kv_block - 1 >= lo:
                m[:, t, b] = True
        m[:, t, 0] = True
    m[1, 0, :] = False                                   # no visible key: zeros
    return m


def _run(q8, k8, v8, scales, kv, q_front, q_offset, counts, lists, kv_block, splits, tail_units=-1):
    from sm120_attn import ops
    n, H, D = q8.shape
    out = torch.full((n, H, D), float('nan'), dtype=torch.bfloat16, device=DEV)
    sq, sk, sv = (torch.from_numpy(np.asarray(s, np.float32)).to(DEV) for s in scales)
    ops.attn_fp8(torch.from_numpy(q8).to(DEV), torch.from_numpy(k8).to(DEV), torch.from_numpy(v8).to(DEV), out, kv,
                 q_front, q_offset, counts, lists, kv_block, sq, sk, sv, D ** -0.5, splits=splits,
                 tail_units=tail_units)
    ops.check_status(DEV)
    return f32(out)


@pytest.mark.parametrize('splits', [2, 3, 4])
@pytest.mark.parametrize('mode', ['dense', 'lists64', 'lists128'])
def test_attn_fp8_split(mode, splits):
    H, Hk, n, kv, q_front = 8, 2, 640, 9000, 40
    _, (q8, k8, v8), scales = _fp8_case(n, kv, H, Hk, seed=splits * 10 + len(mode), per_head=True)
    q_pos0 = kv - n
    q_offset = q_pos0 - q_front
    n_tiles = -(-(q_front + n) // 128)
    counts = lists = masks = None
    kv_block = 64
    if mode != 'dense':
        kv_block = 64 if mode == 'lists64' else 128
        masks = _mixed_masks(H, n_tiles, -(-kv // kv_block), q_offset, kv_block, seed=splits)
        counts, lists = _lists_from_masks(masks)
    units = H * n_tiles
    tail = units - 12                               # the last `tail` units of the launch order split
    out = _run(q8, k8, v8, scales, kv, q_front, q_offset, counts, lists, kv_block, splits, tail)
    whole = _run(q8, k8, v8, scales, kv, q_front, q_offset, counts, lists, kv_block, 1)
    ref = O.attention_ref(_deq(q8, scales[0]), _deq(k8, scales[1]), _deq(v8, scales[2]), q_pos0, masks,
                          q_block=128, kv_block=kv_block, q_front=q_front)
    ref = np.nan_to_num(ref)                             # a row with no visible key is 0 (kai_fa_fp8.py:259-264)
    model = O.attention_fp8_kernel_model(q8, k8, v8, *scales, q_pos0, None if counts is None else counts.cpu().numpy(),
                                         None if lists is None else lists.cpu().numpy(), q_block=128,
                                         kv_block=kv_block, q_front=q_front, splits=splits,
                                         split_min_steps=32 * splits,
                                         split_units=lambda h, t: h * n_tiles + (n_tiles - 1 - t) >= units - tail)
    assert not np.isnan(out).any()
    assert rel_l2(out, model) < 1e-2, rel_l2(out, model)
    assert rel_l2(out, ref) < 3e-2, rel_l2(out, ref)
    assert rel_l2(out, whole) < 4e-2, rel_l2(out, whole)
    # units below the split threshold (32 steps per range) run whole: bit-identical rows
    c = counts.cpu().numpy().reshape(H, n_tiles) if counts is not None else None
    n_split = 0
    for h in range(H):
        for t in range(n_tiles):
            if c is None:
                steps = -(-min(q_offset + (t + 1) * 128, kv) // 64)
            else:
                steps = int(c[h, t]) * (kv_block // 64)
            rows = slice(max(t * 128 - q_front, 0), min((t + 1) * 128 - q_front, n))
            if steps < 32 * splits or h * n_tiles + (n_tiles - 1 - t) < units - tail:
                np.testing.assert_array_equal(out[rows, h], whole[rows, h])
            else:
                n_split += 1
    assert n_split > 0
    if mode != 'dense':
        rows = slice(0, 128 - q_front)
        assert np.all(out[rows, 1] == 0)                 # the empty row


def test_attn_fp8_split_rejects_small_workspace():
    from sm120_attn import _native as N
    from sm120_attn import ops
    q8 = torch.zeros(256, 4, 128, dtype=torch.uint8, device=DEV)
    k8 = torch.zeros(1024, 2, 128, dtype=torch.uint8, device=DEV)
    out = torch.empty(256, 4, 128, dtype=torch.bfloat16, device=DEV)
    one = torch.ones(1, device=DEV)
    need = int(N.lib().sa_attn_split_workspace_bytes(256, 0, 4, 2, 8))
    assert need == 8 * 2 * (128 * 128 + 256) * 4 + 32       # partials + one arrival counter per tail unit
    ws = torch.empty(need - 16, dtype=torch.uint8, device=DEV)
    with pytest.raises(N.NativeError):
        N.call('sa_attn_fwd_fp8_split', ops._p(q8), q8.stride(0), q8.stride(1), ops._p(k8), k8.stride(0),
               k8.stride(1), ops._p(k8), k8.stride(0), k8.stride(1), ops._p(out), out.stride(0), out.stride(1), 256, 4,
               2, 128, 1024, 0, 768, None, None, 0, 128, 64, ops._p(one), 0, ops._p(one), 0, ops._p(one), 0, 0.1,
               None, 2, 8, ops._p(ws), need - 16, ops._stream(DEV))


def test_auto_split_at_eight_gpu_rank_shape(monkeypatch):
    """configs[1] chunk with one KV head and its 8 query heads (the per-rank work of an 8-GPU strong
    split): 512 units for 296 resident CTAs, so the automatic choice splits; the glue's output stays
    within the bar of two independent e4m3 roundings of the unsplit run, and the selection is unchanged."""
    import sm120_attn.sparse_prefill as ksp
    import synth
    from sm120_attn import ops
    monkeypatch.setattr(ksp, 'BLOCK', 128)
    n, kv, H, Hk, D = 8192, 65536, 8, 1, 128
    q, k, v, _ = synth.make_qkv(n, kv, H, Hk, D, block=128, q_start=kv - n, seed=1007, strength='unit', hot=6,
                                device=DEV)
    props = torch.cuda.get_device_properties(DEV)
    k_auto = ops.attn_splits(n, (kv - n) % 128, H, DEV)
    if props.multi_processor_count * 2 <= (n // 128) * H:
        assert k_auto > 1
    outs, sel = {}, {}
    for env in ('auto', '1'):
        monkeypatch.setenv('SA_ATTN_SPLITS', env)
        ksp._KMEAN_CACHE.clear()
        ksp._SCALE_CACHE.clear()
        sp = ksp.SparsePrefill(H, Hk, D, DEV, tau=0.95, min_kv=0, min_q=0, kernel='sm120fp8')
        km = ksp._cached_block_means('split', 0, k, 0, kv)
        scales = ksp._cached_scales('split', 0, q[:n], k, v, 0)
        outs[env] = sp.forward_sm120fp8(q, k, v, kv - n, km=km, scales=scales)
        sel[env] = (sp.last_counts.clone(), sp.last_lists.clone())
        ops.check_status(DEV)
    torch.cuda.synchronize()
    counts = sel['auto'][0]
    assert torch.equal(counts, sel['1'][0])
    held = torch.arange(sel['auto'][1].shape[1], device=DEV)[None, :] < counts[:, None]
    assert torch.equal(sel['auto'][1][held], sel['1'][1][held])
    a, b = outs['auto'].float(), outs['1'].float()
    assert not torch.isnan(a).any()
    assert float((a - b).norm() / b.norm()) < 4e-2
