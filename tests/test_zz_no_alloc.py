"""sa_select_static (selection on the library's built-in scratch buffer) against sa_select.

Collected last on purpose: it must pass in a fresh process (first call sets the buffer up) and
after every other test has used the library.  Both entry points run the same kernels, so their
counts, lists and masks must be identical, on each of two consecutive calls.
"""
import ctypes

import numpy as np
import pytest
import torch

DEV = torch.device('cuda') if torch.cuda.is_available() else None


def _p(t):
    return ctypes.c_void_p(t.data_ptr() if t is not None else 0)


def _static(qm, km, H, Hk, nb_total, qblk0, scale, tau, mode, counts, lists, masks):
    from sm120_attn import _native as N
    MB, _, D = qm.shape
    N.call('sa_select_static', _p(qm), qm.stride(0), qm.stride(1), _p(km), km.stride(0), km.stride(1), km.shape[1],
           H, Hk, D, MB, nb_total, qblk0, ctypes.c_float(scale), ctypes.c_float(tau), mode, _p(counts), _p(lists),
           lists.stride(0), _p(masks), ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))


@pytest.mark.gpu
@pytest.mark.parametrize('mode_name,MB,nb_total,qblk0', [('PER_HEAD', 64, 512, 448), ('PAIR_UNION', 32, 300, 270),
                                                         ('KV_UNION', 16, 96, 80), ('PER_HEAD', 64, 1500, 1440)])
def test_static_scratch_select_matches_workspace_select(mode_name, MB, nb_total, qblk0):
    from sm120_attn import _native as N, ops
    mode = getattr(N, 'SA_SELECT_' + mode_name)
    H, Hk, D, tau, scale = 64, 8, 128, 0.95, 128 ** -0.5
    g = torch.Generator(device=DEV)
    g.manual_seed(MB + nb_total)
    qm = torch.randn(MB, H, D, device=DEV, generator=g)
    km = torch.randn(Hk, nb_total - 7, D, device=DEV, generator=g)        # last blocks zero-padded
    rows = {'PER_HEAD': H * MB, 'PAIR_UNION': H * MB // 2, 'KV_UNION': Hk * MB}[mode_name]
    ref = [torch.full((rows,), -1, dtype=torch.int32, device=DEV),
           torch.full((rows, nb_total), -1, dtype=torch.int32, device=DEV),
           torch.full((rows, nb_total), 7, dtype=torch.uint8, device=DEV)]
    ops.select(qm, km, H, Hk, nb_total, qblk0, scale, tau, mode, counts=ref[0], lists=ref[1], masks=ref[2])
    torch.cuda.synchronize()
    for _ in range(2):                                                    # two calls in a row
        out = [torch.full_like(t, -1 if t.dtype == torch.int32 else 7) for t in ref]
        _static(qm, km, H, Hk, nb_total, qblk0, scale, tau, mode, *out)
        torch.cuda.synchronize()
        np.testing.assert_array_equal(out[0].cpu().numpy(), ref[0].cpu().numpy())
        np.testing.assert_array_equal(out[2].cpu().numpy(), ref[2].cpu().numpy())
        c = ref[0].cpu().numpy()
        lo, lr = out[1].cpu().numpy(), ref[1].cpu().numpy()
        for r in range(rows):
            np.testing.assert_array_equal(lo[r, :c[r]], lr[r, :c[r]])
    ops.check_status(DEV)


@pytest.mark.gpu
def test_static_scratch_refuses_sizes_beyond_its_buffer():
    from sm120_attn import _native as N
    H, Hk, D, MB, nb_total = 64, 8, 128, 128, 4096          # 134 MB of logits > 40 MiB
    qm = torch.zeros(MB, H, D, device=DEV)
    km = torch.zeros(Hk, nb_total, D, device=DEV)
    counts = torch.zeros(H * MB, dtype=torch.int32, device=DEV)
    lists = torch.zeros(H * MB, nb_total, dtype=torch.int32, device=DEV)
    with pytest.raises(N.NativeError, match='static buffer'):
        _static(qm, km, H, Hk, nb_total, 0, 0.1, 0.95, N.SA_SELECT_PER_HEAD, counts, lists, None)
