"""Tensor-level wrappers over the C-ABI entry points (device pointers, element strides, current stream).

Every function here launches CUDA work from `_lib/libsa_b200.so` on
`torch.cuda.current_stream()`; inputs must already be CUDA tensors.  There is no other path.
"""
from __future__ import annotations

import ctypes

import torch

from . import _native as N

_STATUS: dict = {}


def _p(t):
    return ctypes.c_void_p(t.data_ptr()) if t is not None else ctypes.c_void_p(0)


def _stream(dev):
    return ctypes.c_void_p(torch.cuda.current_stream(dev).cuda_stream)


def _need_cuda(name, *ts):
    for t in ts:
        if t is not None and not t.is_cuda:
            raise ValueError(f'{name}: tensors must be on a CUDA device (no CPU path), got {t.device}')


def status_word(device) -> torch.Tensor:
    dev = torch.device(device)
    idx = dev.index if dev.index is not None else torch.cuda.current_device()
    t = _STATUS.get(idx)
    if t is None:
        t = torch.zeros(1, dtype=torch.int32, device=torch.device('cuda', idx))
        _STATUS[idx] = t
    return t


def read_status(device) -> int:
    """Fetch and clear the device status word (synchronises the current stream)."""
    t = status_word(device)
    val = ctypes.c_int32(0)
    N.call('sa_read_status', _p(t), ctypes.byref(val), _stream(t.device))
    return int(val.value)


def check_status(device) -> None:
    v = read_status(device)
    if v:
        raise N.NativeError('device status', N.SA_ERR_DEVICE, f'kernel status bits 0x{v:x}')


def block_means(x, pos0: int, block: int, out, out_block0: int, q8=None, inv_scale=None, fixed_divisor: int = 0):
    """Block means of x [n, heads, D] bf16 (absolute row positions pos0..) into out viewed as
    [heads, blocks, D] fp32 (block index b written at b - out_block0); optional fused e4m3 q8."""
    _need_cuda('block_means', x, out, q8, inv_scale)
    assert x.dtype == torch.bfloat16 and out.dtype == torch.float32 and x.dim() == 3 and out.dim() == 3
    assert x.stride(2) == 1 and out.stride(2) == 1
    n, heads, D = x.shape
    iss = 0
    if q8 is not None:
        assert q8.stride(2) == 1 and inv_scale is not None and inv_scale.dtype == torch.float32
        iss = 0 if inv_scale.numel() == 1 else 1
    N.call('sa_block_means_bf16', _p(x), x.stride(0), x.stride(1), n, heads, D, pos0, block, _p(out),
           out.stride(0), out.stride(1), out_block0, _p(q8), q8.stride(0) if q8 is not None else 0,
           q8.stride(1) if q8 is not None else 0, _p(inv_scale), iss, int(fixed_divisor), _stream(x.device))


def select_workspace_bytes(num_heads: int, MB: int, nb_total: int) -> int:
    return int(N.lib().sa_select_workspace_bytes(num_heads, MB, nb_total))


def select(qm, km, num_heads: int, num_kv_heads: int, nb_total: int, qblk0: int, scale: float, tau: float,
           mode: int, counts=None, lists=None, masks=None, workspace=None):
    """Block selection (see sa_select).  qm [MB, H, D] fp32, km [Hk, NBk, D] fp32.

    workspace: optional uint8 device tensor of at least select_workspace_bytes(...) bytes; by
    default one is taken from torch's caching allocator for the call."""
    _need_cuda('select', qm, km, counts, lists, masks)
    assert qm.dtype == torch.float32 and km.dtype == torch.float32 and qm.stride(2) == 1 and km.stride(2) == 1
    MB, H, D = qm.shape
    need = select_workspace_bytes(num_heads, MB, nb_total)
    if workspace is None:
        workspace = torch.empty(need, dtype=torch.uint8, device=qm.device)
    _need_cuda('select', workspace)
    N.call('sa_select', _p(qm), qm.stride(0), qm.stride(1), _p(km), km.stride(0), km.stride(1), km.shape[1],
           num_heads, num_kv_heads, D, MB, nb_total, qblk0, float(scale), float(tau), mode, _p(counts), _p(lists),
           lists.stride(0) if lists is not None else 0, _p(masks), _p(workspace), workspace.numel(),
           _stream(qm.device))


def quantize(x, scale, mode: int, out, transpose: bool = False, rows_pad: int = 0):
    """e4m3 quantisation of x [rows, heads, D] bf16 into out (uint8 / float8_e4m3fn storage)."""
    _need_cuda('quantize', x, scale, out)
    rows, heads, D = x.shape
    ss = 0 if scale.numel() == 1 else 1
    if transpose:
        # out [heads, D, rows_pad]
        N.call('sa_quantize_e4m3', _p(x), x.stride(0), x.stride(1), rows, heads, D, _p(scale), ss, mode, _p(out),
               out.stride(1), out.stride(0), 1, rows_pad, _stream(x.device))
    else:
        N.call('sa_quantize_e4m3', _p(x), x.stride(0), x.stride(1), rows, heads, D, _p(scale), ss, mode, _p(out),
               out.stride(0), out.stride(1), 0, 0, _stream(x.device))


def absmax(x, per_head: bool, out=None):
    _need_cuda('absmax', x, out)
    rows, heads, D = x.shape
    if out is None:
        out = torch.empty(heads if per_head else 1, dtype=torch.float32, device=x.device)
    N.call('sa_absmax_bf16', _p(x), x.stride(0), x.stride(1), rows, heads, D, 1 if per_head else 0, _p(out),
           _stream(x.device))
    return out


def attn_fp8(q8, k8, v8, out, kv_len: int, q_front: int, q_offset: int, counts, lists, kv_block: int,
             q_scale, k_scale, v_scale, softmax_scale: float, q_block: int = 128):
    """Block-sparse (counts/lists) or dense causal FP8 attention; see sa_attn_fwd_fp8.

    q8 [n, H, D], k8 / v8 [kv, Hk, D] e4m3 bytes (last dim contiguous), out [n, H, D] bf16."""
    _need_cuda('attn_fp8', q8, k8, v8, out, counts, lists, q_scale, k_scale, v_scale)
    n, H, D = q8.shape
    Hk = k8.shape[1]
    st = status_word(q8.device)
    N.call('sa_attn_fwd_fp8', _p(q8), q8.stride(0), q8.stride(1), _p(k8), k8.stride(0), k8.stride(1), _p(v8),
           v8.stride(0), v8.stride(1), _p(out), out.stride(0), out.stride(1), n, H, Hk, D, kv_len, q_front,
           q_offset, _p(counts), _p(lists), lists.stride(0) if lists is not None else 0, q_block, kv_block,
           _p(q_scale), 0 if q_scale.numel() == 1 else 1, _p(k_scale), 0 if k_scale.numel() == 1 else 1,
           _p(v_scale), 0 if v_scale.numel() == 1 else 1, float(softmax_scale), _p(st), _stream(q8.device))


def attn_bf16(q, k, v, out, kv_len: int, q_front: int, q_offset: int, counts, lists, kv_block: int,
              softmax_scale: float, q_block: int = 128):
    """Block-sparse (counts/lists) or dense causal BF16 attention; see sa_attn_fwd_bf16.

    q [n, H, D], k / v [kv, Hk, D] bf16 (last dim contiguous), out [n, H, D] bf16."""
    _need_cuda('attn_bf16', q, k, v, out, counts, lists)
    n, H, D = q.shape
    Hk = k.shape[1]
    st = status_word(q.device)
    N.call('sa_attn_fwd_bf16', _p(q), q.stride(0), q.stride(1), _p(k), k.stride(0), k.stride(1), _p(v),
           v.stride(0), v.stride(1), _p(out), out.stride(0), out.stride(1), n, H, Hk, D, kv_len, q_front,
           q_offset, _p(counts), _p(lists), lists.stride(0) if lists is not None else 0, q_block, kv_block,
           float(softmax_scale), _p(st), _stream(q.device))
