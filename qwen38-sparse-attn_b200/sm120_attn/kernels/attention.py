"""Drivers of the B200 attention kernels with the reference's call signatures.

`attention_sm120` (BF16), `attention_sm120_fp8` and `attention_sm120_fp8_tma` (FP8) keep the
arguments, defaults, list semantics and return values of sm120_attn/kernels/kai_fa_bf16.py:1206-1243,
kai_fa_fp8.py:331-375 and kai_fa_fp8_tma.py:447-490.  Behind them is one tcgen05 kernel
(sa_attn_fwd_fp8 / sa_attn_fwd_bf16); the reference's tuning switches (m_block, n_block,
num_threads, s_pipeline, pingpong, prefetch) are validated and otherwise have no effect, except
that m_block / n_block give the row and key granularity of caller-supplied block lists.

The kernel reads V in its natural [kv, Hk, D] layout.  The reference's FP8 drivers take `prequant`
V as V^T with its key order permuted inside each 32-key block (VT_KEY_PERM, for its mma.sync
register layout); these drivers undo the permutation and the transpose for `prequant` inputs so
callers can pass exactly what they passed before.
"""
from __future__ import annotations

import torch

from .. import ops
from .._native import SA_QUANT_DIV

# Key order inside each 32-key block of the reference's permuted V^T (kai_fa_fp8.py:303-306).  It is
# part of the `prequant` interface, so it is kept identical.
VT_KEY_PERM = [16 * (s >> 4) + 8 * ((s & 3) >> 1) + 2 * ((s >> 2) & 3) + ((s & 3) & 1) for s in range(32)]
_VT_INV = [VT_KEY_PERM.index(i) for i in range(32)]
_VT_PERM: dict = {}
_VT_UNPERM: dict = {}


def vt_key_index(kv_len, device):
    """Gather index that permutes the key axis of a (padded) V^T; kv_len % 32 == 0 (kai_fa_fp8.py:309-318)."""
    key = (kv_len, str(device))
    idx = _VT_PERM.get(key)
    if idx is None:
        base = torch.arange(0, kv_len, 32, device=device, dtype=torch.int64)
        perm = torch.tensor(VT_KEY_PERM, device=device, dtype=torch.int64)
        idx = (base[:, None] + perm[None, :]).reshape(-1)
        _VT_PERM[key] = idx
    return idx


def permute_vt_keys(vT8):
    """vT8 [Hk, D, kv] (kv % 32 == 0) -> same layout with keys permuted per 32-key block."""
    return vT8.index_select(2, vt_key_index(vT8.shape[2], vT8.device))


def _unpermute_vt_keys(vT8):
    key = (vT8.shape[2], str(vT8.device))
    idx = _VT_UNPERM.get(key)
    if idx is None:
        base = torch.arange(0, vT8.shape[2], 32, device=vT8.device, dtype=torch.int64)
        inv = torch.tensor(_VT_INV, device=vT8.device, dtype=torch.int64)
        idx = (base[:, None] + inv[None, :]).reshape(-1)
        _VT_UNPERM[key] = idx
    return vT8.index_select(2, idx)


def _scalar(x, device):
    if torch.is_tensor(x):
        return x.to(device=device, dtype=torch.float32).reshape(-1)
    return torch.full((1,), float(x), dtype=torch.float32, device=device)


def quantize_e4m3(x):
    """Per-tensor e4m3 quantisation: (x8, scale) with scale = amax/448 (kai_fa_fp8.py:325-328).

    One device sync (the scale is returned as a Python float, like the reference).
    """
    if x.dtype != torch.bfloat16:
        raise TypeError('quantize_e4m3: bf16 input expected')
    x3 = x.reshape(x.shape[0], -1, x.shape[-1]) if x.dim() != 3 else x
    x3 = x3 if x3.stride(-1) == 1 else x3.contiguous()
    amax = ops.absmax(x3, per_head=False).clamp_min_(1e-6)
    scale_t = amax / 448.0
    out = torch.empty(x3.shape, dtype=torch.float8_e4m3fn, device=x.device)
    ops.quantize(x3, scale_t, SA_QUANT_DIV, out.view(torch.uint8))
    return out.view(x.shape), float(scale_t.item())


def _quantize(x, scale: float):
    out = torch.empty(x.shape, dtype=torch.uint8, device=x.device)
    ops.quantize(x, _scalar(scale, x.device), SA_QUANT_DIV, out)
    return out


def _lists_args(counts, lists):
    if counts is None:
        return None, None
    if lists is None:
        raise ValueError('counts given without lists')
    counts = counts.to(torch.int32).contiguous()
    lists = lists.to(torch.int32)
    if lists.dim() == 1:
        lists = lists.view(counts.numel(), -1)
    if lists.stride(1) != 1:
        lists = lists.contiguous()
    return counts, lists


def attention_sm120(q, k, v, q_offset=None, *, causal=True, m_block=64, n_block=64, num_threads=128, out=None,
                    counts=None, lists=None):
    """Dense causal attention, or block-sparse when (counts, lists) are given: for row r = head * MB + m_block,
    lists[r, :counts[r]] is the ascending list of allowed n_blocks (diagonal block last).

    q [n, H, D], k/v [kv_len, Hk, D] bf16 (NHD); returns bf16 [n, H, D].
    """
    n, H, D = q.shape
    kv_len, Hk, _ = k.shape
    if q_offset is None:
        q_offset = kv_len - n
    if not (q.dtype == torch.bfloat16 and k.dtype == torch.bfloat16 and v.dtype == torch.bfloat16):
        raise TypeError('attention_sm120: bf16 q, k, v expected')
    if m_block not in (64, 128) or n_block not in (64, 128) or num_threads <= 0:
        raise ValueError('configuration not implementable')
    if out is None:
        out = torch.empty_like(q)
    if not causal:
        q_offset = max(q_offset, kv_len)              # every key visible to every row
    v = v if v.stride(-1) == 1 else v.contiguous()
    counts, lists = _lists_args(counts, lists)
    ops.attn_bf16(q, k, v, out, kv_len, 0, q_offset, counts, lists, n_block, D ** -0.5, q_block=m_block)
    return out


def attention_sm120_fp8(q, k, v, q_offset=None, *, causal=True, out=None, counts=None, lists=None, prequant=None,
                        m_block=128):
    """q [n,H,D], k/v [kv,Hk,D] bf16 (quantised here, per tensor) or prequant=(q8, sq, k8, sk, vT8, sv) with
    q8 [n,H,D], k8 [kv,Hk,D], vT8 [Hk,D,kv] in e4m3 and kv a multiple of 64 (zero padded); vT8's key axis
    permuted with permute_vt_keys().  Lists are per 128-row query block over 64-key blocks."""
    n, H, D = q.shape
    kv_len = k.shape[0]
    if q_offset is None:
        q_offset = kv_len - n
    if m_block not in (64, 128):
        raise ValueError('fp8 kernel supports m_block 64 or 128')
    if prequant is None:
        q8, sq = quantize_e4m3(q)
        k8, sk = quantize_e4m3(k)
        _, sv = None, None
        v3 = v if v.stride(-1) == 1 else v.contiguous()
        amax = ops.absmax(v3, per_head=False).clamp_min_(1e-6)
        sv = float((amax / 448.0).item())
        v8 = _quantize(v3, sv)
        kv_keys = kv_len
    else:
        q8, sq, k8, sk, vT8, sv = prequant
        kv_keys = k8.shape[0]
        v8 = _unpermute_vt_keys(vT8)[:, :, :kv_keys].permute(2, 0, 1).contiguous()
    if not causal:
        q_offset = max(q_offset, kv_keys)
    if out is None:
        out = torch.empty(n, H, D, dtype=torch.bfloat16, device=q.device)
    counts, lists = _lists_args(counts, lists)
    dev = q.device
    ops.attn_fp8(q8.view(torch.uint8), k8.view(torch.uint8), v8.view(torch.uint8), out, kv_keys, 0, q_offset,
                 counts, lists, 64, _scalar(sq, dev), _scalar(sk, dev), _scalar(sv, dev), D ** -0.5, q_block=m_block)
    return out


def attention_sm120_fp8_tma(q, k, v, q_offset=None, *, causal=True, out=None, counts=None, lists=None, prequant=None,
                            m_block=128, s_pipeline=False, pingpong=False, prefetch=False):
    """Same contract as attention_sm120_fp8 (kai_fa_fp8_tma.py:447-490); one kernel serves both pipelines."""
    for name, val in (('s_pipeline', s_pipeline), ('pingpong', pingpong), ('prefetch', prefetch)):
        if not isinstance(val, bool):
            raise TypeError(f'{name} must be a bool')
    return attention_sm120_fp8(q, k, v, q_offset, causal=causal, out=out, counts=counts, lists=lists,
                               prequant=prequant, m_block=m_block)
