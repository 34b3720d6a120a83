"""Tensor-level wrappers over the C-ABI entry points (device pointers, element strides, current stream).

Every function here launches CUDA work from `_lib/libsa_b200.so` on
`torch.cuda.current_stream()`; inputs must already be CUDA tensors.  There is no other path.
"""
from __future__ import annotations

import ctypes
import os

import torch

from . import _native as N

_STATUS: dict = {}



def attn_schedule(fp8: bool = True):
    """(keys per online-softmax step, paired tiles) of the attention kernel this process launches.

    P is rounded (e4m3) against the running row maximum of each step, so numerical models of the
    kernel follow this granularity.  The default one-tile kernel takes 64-key steps.  The paired-tile
    kernel (FP8, SA_ATTN_KERNEL=pair; the library reads the same variable once per process) walks
    two query tiles that share a KV head together, 128 keys per step: two query heads (h, h ^ 1) of
    one tile when the GQA group size is even, else tiles (t, t ^ 1) of one head.  BF16 always uses
    the one-tile kernel."""
    paired = fp8 and os.environ.get('SA_ATTN_KERNEL', '') == 'pair'
    return (128 if paired else 64), paired


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


def select_q_supported(num_heads: int, num_kv_heads: int, head_dim: int, nb_total: int, mode: int) -> bool:
    """Whether sa_select_q (the one-pass pooling + selection kernel) serves these sizes: head_dim 128,
    at most 16 query heads per KV head, rows of at most 1024 key blocks, and the unit's logits
    (query blocks of the unit x heads per KV head x padded key blocks) within 16384 floats."""
    g = num_heads // num_kv_heads
    npl = -(-nb_total // 32)
    rows = (2 if mode == N.SA_SELECT_PAIR_UNION else 1) * g
    return head_dim == 128 and g <= 16 and npl <= 32 and rows * npl * 32 <= 16384


def select_q(q, q_start: int, block: int, qblk0: int, MB: int, km, num_heads: int, num_kv_heads: int,
             nb_total: int, scale: float, tau: float, mode: int, counts=None, lists=None, masks=None, q8=None,
             inv_scale=None):
    """Block selection straight from the query rows (see sa_select_q): q [n, H, D] bf16 at absolute
    positions q_start.., pooled per `block` rows into query blocks qblk0 .. qblk0+MB-1, scored against
    km [Hk, NBk, D] fp32; optional fused e4m3 q8 [n, H, D] = e4m3(bf16(q * inv_scale))."""
    _need_cuda('select_q', q, km, counts, lists, masks, q8, inv_scale)
    assert q.dtype == torch.bfloat16 and q.stride(2) == 1 and km.dtype == torch.float32 and km.stride(2) == 1
    n, H, D = q.shape
    iss = 0
    if q8 is not None:
        assert q8.stride(2) == 1 and inv_scale is not None and inv_scale.dtype == torch.float32
        iss = 0 if inv_scale.numel() == 1 else 1
    N.call('sa_select_q', _p(q), q.stride(0), q.stride(1), n, q_start, block, qblk0, MB, _p(km), km.stride(0),
           km.stride(1), km.shape[1], num_heads, num_kv_heads, D, nb_total, float(scale), float(tau), mode,
           _p(counts), _p(lists), lists.stride(0) if lists is not None else 0, _p(masks), _p(q8),
           q8.stride(0) if q8 is not None else 0, q8.stride(1) if q8 is not None else 0, _p(inv_scale), iss,
           _p(status_word(q.device)), _stream(q.device))


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


def _paged(name, cache, table):
    """Strides of a paged cache [num_pages, page, heads, D] bf16 and its int32 page table row."""
    if cache.dtype != torch.bfloat16 or cache.dim() != 4 or cache.stride(3) != 1:
        raise ValueError(f'{name}: cache must be bf16 [num_pages, page, heads, head_dim] with unit last stride')
    if table.dtype != torch.int32 or table.dim() != 1 or table.stride(0) != 1:
        raise ValueError(f'{name}: page table must be a contiguous int32 vector')
    return cache.stride(0), cache.stride(1), cache.stride(2)


def block_means_paged(cache, table, pos0: int, n: int, block: int, out, out_block0: int):
    """Block means of the keys at positions pos0 .. pos0+n-1 of a paged cache (page table row
    `table`) into out [heads, blocks, D] fp32; see sa_block_means_paged_bf16."""
    _need_cuda('block_means_paged', cache, table, out)
    ps, rs, hs = _paged('block_means_paged', cache, table)
    heads, D = cache.shape[2], cache.shape[3]
    assert out.dtype == torch.float32 and out.dim() == 3 and out.stride(2) == 1
    N.call('sa_block_means_paged_bf16', _p(cache), ps, rs, hs, _p(table), cache.shape[1], n, heads, D, pos0, block,
           _p(out), out.stride(0), out.stride(1), out_block0, _stream(cache.device))


def absmax_paged(cache, table, row0: int, rows: int, per_head: bool, out=None):
    """absmax over positions row0 .. row0+rows-1 of a paged cache; see sa_absmax_paged_bf16."""
    _need_cuda('absmax_paged', cache, table, out)
    ps, rs, hs = _paged('absmax_paged', cache, table)
    heads, D = cache.shape[2], cache.shape[3]
    if out is None:
        out = torch.empty(heads if per_head else 1, dtype=torch.float32, device=cache.device)
    N.call('sa_absmax_paged_bf16', _p(cache), ps, rs, hs, _p(table), cache.shape[1], row0, rows, heads, D,
           1 if per_head else 0, _p(out), _stream(cache.device))
    return out


def quantize_paged(cache, table, row0: int, scale, mode: int, out):
    """e4m3 of positions row0 .. row0+len(out)-1 of a paged cache into out [rows, heads, D] (row r =
    position row0 + r); see sa_quantize_paged_e4m3."""
    _need_cuda('quantize_paged', cache, table, scale, out)
    ps, rs, hs = _paged('quantize_paged', cache, table)
    heads, D = cache.shape[2], cache.shape[3]
    ss = 0 if scale.numel() == 1 else 1
    N.call('sa_quantize_paged_e4m3', _p(cache), ps, rs, hs, _p(table), cache.shape[1], row0, out.shape[0], heads, D,
           _p(scale), ss, mode, _p(out), out.stride(0), out.stride(1), _stream(cache.device))


def absmax(x, per_head: bool, out=None):
    _need_cuda('absmax', x, out)
    rows, heads, D = x.shape
    if out is None:
        out = torch.empty(heads if per_head else 1, dtype=torch.float32, device=x.device)
    N.call('sa_absmax_bf16', _p(x), x.stride(0), x.stride(1), rows, heads, D, 1 if per_head else 0, _p(out),
           _stream(x.device))
    return out


_SPLITS: dict = {}


def attn_splits(n: int, q_front: int, num_heads: int, device) -> int:
    """Split count for an FP8 attention launch: SA_ATTN_SPLITS (an integer; 0 or 1 = never split) or,
    unset / `auto`, sa_attn_split_count's choice for the current GPU (cached per shape and device)."""
    env = os.environ.get('SA_ATTN_SPLITS', 'auto').strip().lower()
    if env not in ('', 'auto'):
        return max(1, int(env))
    key = (n, q_front, num_heads, torch.device(device).index)
    if key not in _SPLITS:
        _SPLITS[key] = int(N.lib().sa_attn_split_count(n, q_front, num_heads))
    return _SPLITS[key]


def attn_fp8(q8, k8, v8, out, kv_len: int, q_front: int, q_offset: int, counts, lists, kv_block: int,
             q_scale, k_scale, v_scale, softmax_scale: float, q_block: int = 128, splits=None,
             tail_units: int = -1):
    """Block-sparse (counts/lists) or dense causal FP8 attention; see sa_attn_fwd_fp8.

    q8 [n, H, D], k8 / v8 [kv, Hk, D] e4m3 bytes (last dim contiguous), out [n, H, D] bf16.
    splits: step ranges per walk of the split units (sa_attn_fwd_fp8_split, with a workspace from
    torch's caching allocator); None = attn_splits' choice.  tail_units: how many units (the last of
    the launch order) are split; -1 = the partial last wave of this GPU."""
    _need_cuda('attn_fp8', q8, k8, v8, out, counts, lists, q_scale, k_scale, v_scale)
    n, H, D = q8.shape
    Hk = k8.shape[1]
    st = status_word(q8.device)
    k = attn_splits(n, q_front, H, q8.device) if splits is None else max(1, int(splits))
    if k > 1 and q_block == 128:
        nbytes = int(N.lib().sa_attn_split_workspace_bytes(n, q_front, H, k, int(tail_units)))
        ws = torch.empty(max(nbytes, 16), dtype=torch.uint8, device=q8.device)
        N.call('sa_attn_fwd_fp8_split', _p(q8), q8.stride(0), q8.stride(1), _p(k8), k8.stride(0), k8.stride(1),
               _p(v8), v8.stride(0), v8.stride(1), _p(out), out.stride(0), out.stride(1), n, H, Hk, D, kv_len,
               q_front, q_offset, _p(counts), _p(lists), lists.stride(0) if lists is not None else 0, q_block,
               kv_block, _p(q_scale), 0 if q_scale.numel() == 1 else 1, _p(k_scale), 0 if k_scale.numel() == 1 else 1,
               _p(v_scale), 0 if v_scale.numel() == 1 else 1, float(softmax_scale), _p(st), k, int(tail_units),
               _p(ws), nbytes, _stream(q8.device))
        return
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


def attn_bf16_paged(q, k_cache, v_cache, table, out, kv_len: int, q_front: int, q_offset: int, counts, lists,
                    kv_block: int, softmax_scale: float, q_block: int = 128):
    """attn_bf16 with K and V read in place from paged caches [num_pages, page, Hk, D] through the
    request's page table row (int32); see sa_attn_fwd_bf16_paged."""
    _need_cuda('attn_bf16_paged', q, k_cache, v_cache, table, out, counts, lists)
    ps, rs, hs = _paged('attn_bf16_paged', k_cache, table)
    if v_cache.stride() != k_cache.stride() or v_cache.shape != k_cache.shape:
        raise ValueError('attn_bf16_paged: k_cache and v_cache must have the same shape and strides')
    n, H, D = q.shape
    num_pages, page, Hk = k_cache.shape[0], k_cache.shape[1], k_cache.shape[2]
    st = status_word(q.device)
    N.call('sa_attn_fwd_bf16_paged', _p(q), q.stride(0), q.stride(1), _p(k_cache), _p(v_cache), ps, rs, hs, _p(table),
           page, num_pages, _p(out), out.stride(0), out.stride(1), n, H, Hk, D, kv_len, q_front, q_offset, _p(counts),
           _p(lists), lists.stride(0) if lists is not None else 0, q_block, kv_block, float(softmax_scale), _p(st),
           _stream(q.device))


def paged_attention_supported(page: int) -> bool:
    """Page sizes sa_attn_fwd_bf16_paged reads in place."""
    return page in (8, 16, 32) or (page > 0 and page % 64 == 0)


# ---------------------------------------------------------------- end-to-end prefill harness kernels

def _rows2d(name, t):
    if t.dim() != 2 or t.stride(1) != 1 or t.dtype != torch.bfloat16:
        raise ValueError(f'{name}: expected a bf16 [rows, cols] tensor with unit column stride')


def add_rmsnorm(h, weight, x_out, eps: float, delta=None):
    """h <- h + delta (when given); x_out <- rmsnorm(h) * weight (fp32 arithmetic); see sa_add_rmsnorm_bf16."""
    _need_cuda('add_rmsnorm', h, weight, x_out, delta)
    for name, t in (('h', h), ('x_out', x_out)) + ((('delta', delta),) if delta is not None else ()):
        _rows2d(f'add_rmsnorm {name}', t)
    rows, hidden = h.shape
    if x_out.shape != h.shape or (delta is not None and delta.shape != h.shape) or weight.shape != (hidden,):
        raise ValueError('add_rmsnorm: shape mismatch')
    N.call('sa_add_rmsnorm_bf16', _p(delta), delta.stride(0) if delta is not None else 0, _p(h), h.stride(0),
           _p(weight), _p(x_out), x_out.stride(0), rows, hidden, ctypes.c_float(eps), _stream(h.device))


def rope_qkv(qkv, num_heads: int, num_kv_heads: int, head_dim: int, cos_sin, pos0: int, q_out, k_out, v_out,
             km=None, block: int = 0, km_block0: int = 0):
    """Rotary embedding of the q and k heads of qkv [rows, (H + 2 Hk) D] at positions pos0..; q to
    q_out [rows, H, D], k and v to k_out / v_out [rows, Hk, D] (e.g. cache rows); see sa_rope_qkv_bf16.
    With km ([Hk, blocks, D] fp32) the block means of the rotated keys (blocks of `block` rows, block
    b at km[:, b - km_block0]) are written in the same pass (sa_rope_qkv_means_bf16)."""
    _need_cuda('rope_qkv', qkv, cos_sin, q_out, k_out, v_out)
    _rows2d('rope_qkv qkv', qkv)
    rows = qkv.shape[0]
    if qkv.shape[1] != (num_heads + 2 * num_kv_heads) * head_dim:
        raise ValueError('rope_qkv: qkv width does not match the head counts')
    for t, hh in ((q_out, num_heads), (k_out, num_kv_heads), (v_out, num_kv_heads)):
        if t.dtype != torch.bfloat16 or t.dim() != 3 or t.shape[0] < rows or t.shape[1:] != (hh, head_dim) or \
                t.stride(2) != 1 or t.stride(1) != head_dim:
            raise ValueError('rope_qkv: outputs must be bf16 [rows, heads, head_dim] with contiguous heads')
    if q_out.stride(0) != num_heads * head_dim:
        raise ValueError('rope_qkv: q_out must be contiguous')
    if cos_sin.dtype != torch.float32 or cos_sin.dim() != 2 or cos_sin.shape[1] != head_dim or not cos_sin.is_contiguous():
        raise ValueError('rope_qkv: cos_sin must be a contiguous fp32 [max_pos, head_dim] table')
    if km is None:
        N.call('sa_rope_qkv_bf16', _p(qkv), qkv.stride(0), rows, num_heads, num_kv_heads, head_dim, _p(cos_sin), pos0,
               cos_sin.shape[0], _p(q_out), _p(k_out), k_out.stride(0), _p(v_out), v_out.stride(0),
               _stream(qkv.device))
        return
    _need_cuda('rope_qkv', km)
    if km.dtype != torch.float32 or km.dim() != 3 or km.shape[0] != num_kv_heads or km.shape[2] != head_dim or \
            km.stride(2) != 1:
        raise ValueError('rope_qkv: km must be fp32 [num_kv_heads, blocks, head_dim]')
    if block <= 0 or -(-(pos0 + rows) // block) - km_block0 > km.shape[1]:
        raise ValueError('rope_qkv: km holds too few blocks')
    N.call('sa_rope_qkv_means_bf16', _p(qkv), qkv.stride(0), rows, num_heads, num_kv_heads, head_dim, _p(cos_sin),
           pos0, cos_sin.shape[0], _p(q_out), _p(k_out), k_out.stride(0), _p(v_out), v_out.stride(0), block, _p(km),
           km.stride(0), km.stride(1), km_block0, _stream(qkv.device))


def silu_mul(gate_up, out):
    """out = silu(gate_up[:, :I]) * gate_up[:, I:] with I = out.shape[1]; see sa_silu_mul_bf16."""
    _need_cuda('silu_mul', gate_up, out)
    _rows2d('silu_mul gate_up', gate_up)
    _rows2d('silu_mul out', out)
    rows, inter = out.shape
    if gate_up.shape != (rows, 2 * inter):
        raise ValueError('silu_mul: gate_up must be [rows, 2 * inter]')
    N.call('sa_silu_mul_bf16', _p(gate_up), gate_up.stride(0), rows, inter, _p(out), out.stride(0),
           _stream(out.device))
