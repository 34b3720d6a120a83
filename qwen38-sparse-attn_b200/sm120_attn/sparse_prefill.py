"""Dynamic block-sparse causal prefill attention for long contexts (B200 implementation).

Drop-in replacement of accion-intelligence/Qwen38-sparse-attn `sm120_attn/sparse_prefill.py`: the same
module globals, classes, functions, knobs and cache dictionaries, with the selection math, pooling,
quantisation and attention running in the CUDA kernels of `_lib/libsa_b200.so`:

* per full-attention layer and prefill chunk, the keys of the chunk are mean-pooled into the
  per-request block-mean cache (kernel a, `_cached_block_means`);
* the queries of the chunk are mean-pooled per block (kernel a; fused with the e4m3 quantisation
  of q on the FP8 path) and scored against the cached key means; per query head and query
  block the smallest block set reaching attention mass tau is kept, plus the sink and the
  diagonal block (kernel b, `SparsePrefill.block_masks`);
* the selected blocks are walked by the block-sparse attention kernel (kernel c).

`BLOCK` (64, as in the reference; 128 via SM120_SPARSE_BLOCK) is the selection block.  The FP8
path uses 128-row query blocks: with BLOCK 64 they are the union of two 64-row masks over 64-key
blocks (sparse_prefill.py:223), with BLOCK 128 they are the 128-row masks over 128-key blocks.
Decode and short chunks never enter this module's kernels (`try_sparse_forward` returns False).
"""
from __future__ import annotations

import json
import math
import os
import time
import weakref
from pathlib import Path
from typing import Callable, NamedTuple

import torch

from . import ops
from ._native import SA_QUANT_MUL_BF16, SA_SELECT_KV_UNION, SA_SELECT_PAIR_UNION, SA_SELECT_PER_HEAD

BLOCK = int(os.environ.get('SM120_SPARSE_BLOCK', '64'))

_KERNEL_ALIASES = {'sm120fp8': 'sm120fp8', 'fp8': 'sm120fp8', 'sm120': 'sm120', 'bf16': 'sm120'}


def _cdiv(a, b):
    return -(-a // b)


class SparsePrefill:
    def __init__(self, num_heads: int, num_kv_heads: int, head_dim: int, device,
                 tau: float = 0.95, min_kv: int = 8192, min_q: int = 1024,
                 workspace_bytes: int = 256 << 20, kernel: str = 'sm120fp8', fp8_pipeline: str = 'tma'):
        if kernel not in _KERNEL_ALIASES:
            raise ValueError(f'kernel {kernel!r}: expected sm120fp8 | sm120 (fp8 | bf16); the FlashInfer path is retired')
        if fp8_pipeline not in ('tma', 'cpasync'):
            raise ValueError(f'fp8_pipeline {fp8_pipeline!r}: expected tma | cpasync')
        self.kernel = _KERNEL_ALIASES[kernel]
        self.fp8_pipeline = fp8_pipeline     # accepted for compatibility: one TMA/tcgen05 kernel serves both
        # shape: query heads H, KV heads Hk (GQA group g = H / Hk), head_dim D, softmax scale D^-1/2
        self.H = num_heads
        self.Hk = num_kv_heads
        self.D = head_dim
        self.g, self.scale = self.H // self.Hk, 1.0 / math.sqrt(head_dim)
        # selection threshold and the eligibility limits of the hook
        self.tau = tau
        self.min_q, self.min_kv = min_q, min_kv
        self.wrapper = None                  # the retired FlashInfer planner's slot (always None)
        # counters of the reference's stats dictionary; the *_ms entries grow only with timing=True
        self.stats = dict.fromkeys(('calls', 'blocks_total', 'blocks_kept'), 0)
        self.stats.update(dict.fromkeys(('plan_ms', 'run_ms', 'select_ms'), 0.0))
        self._kept_acc = None                # device tensor: kept blocks summed over calls
        self.timing = False
        # Optional list: when set, every forward appends (start, end) CUDA events recorded on the
        # launching stream around the attention kernel (profiling without host syncs).
        self.kernel_events = None

    def _attn_events(self):
        if self.kernel_events is None:
            return None, None
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        self.kernel_events.append((s, e))
        return s, e

    def eligible(self, q_len: int, kv_len: int) -> bool:
        """Long enough for the sparse path: at least min_q queries over at least min_kv keys."""
        return not (q_len < self.min_q or kv_len < self.min_kv)

    # -------------------------------------------------------------------------------------------
    # selection
    # -------------------------------------------------------------------------------------------
    def _km_from_keys(self, k, nb, kv_rows=None):
        """Block means [Hk, nb, D] of NHD keys k over nb BLOCK-row blocks; rows missing from k count as
        zeros (the reference zero-pads k before `.mean`, sparse_prefill.py:166-168, :216-218)."""
        km = torch.empty(self.Hk, nb, self.D, dtype=torch.float32, device=k.device)
        rows = min(k.shape[0], nb * BLOCK) if kv_rows is None else kv_rows
        if rows < nb * BLOCK:
            km.zero_()
        if rows > 0:
            ops.block_means(k[:rows], 0, BLOCK, km, 0, fixed_divisor=BLOCK)
        return km

    def _select(self, q, q_start, qblk0, MB, km, nb_total, mode, counts=None, lists=None, masks=None, q8=None,
                inv_scale=None):
        """Selection for the query rows q [n, H, D] at q_start.. over query blocks qblk0.. (MB of them):
        one pass over q (pool, score, select; sa_select_q) when that kernel serves the sizes, else the
        pooled means qm and sa_select.  q8 / inv_scale: fused e4m3 copy of q (FP8 path)."""
        if ops.select_q_supported(self.H, self.Hk, self.D, nb_total, mode):
            ops.select_q(q, q_start, BLOCK, qblk0, MB, km, self.H, self.Hk, nb_total, self.scale, self.tau, mode,
                         counts=counts, lists=lists, masks=masks, q8=q8, inv_scale=inv_scale)
            return
        qm = self._pool_q(q, q_start, qblk0 * BLOCK, MB, q8=q8, inv_scale=inv_scale)
        ops.select(qm, km, self.H, self.Hk, nb_total, qblk0, self.scale, self.tau, mode, counts=counts, lists=lists,
                   masks=masks)

    def _pool_q(self, q, q_start, qs, MB, q8=None, inv_scale=None):
        """Pooled query blocks qm [MB, H, D] (block m at aligned position qs + m*BLOCK) of q [n, H, D] at
        q_start; optionally writes e4m3(bf16(q * inv_scale)) into q8 in the same pass."""
        qm = torch.zeros(MB, self.H, self.D, dtype=torch.float32, device=q.device)
        if q.shape[0]:
            ops.block_means(q, q_start, BLOCK, qm.permute(1, 0, 2), qs // BLOCK, q8=q8, inv_scale=inv_scale)
        return qm

    @torch.no_grad()
    def block_masks(self, q: torch.Tensor, k, q_start: int, valid=None, union: bool = True, km=None):
        """Selected blocks of a chunk whose first query sits at absolute position q_start (a multiple of
        BLOCK; the caller pads q [n, H, D] to whole blocks, `valid` = (first row, row count) of the
        real queries).  Keys: the cached means km [Hk, NB, D], or k given head-major [Hk, N, D] or
        NHD [N, Hk, D] (N a multiple of BLOCK).  Returns a bool tensor [Hk, MB, NB] (each KV head's
        union over its query heads) or, with union=False, [H, MB, NB] (one row per query head)."""
        n = q.shape[0]
        if km is None:                                       # pool the given keys (NHD view of either layout)
            nhd = k.permute(1, 0, 2) if (k.shape[0] == self.Hk and k.shape[1] != self.Hk) else k
            km = self._km_from_keys(nhd, nhd.shape[0] // BLOCK)
        NB = km.shape[1]
        MB = _cdiv(n, BLOCK)
        assert n % BLOCK == 0 and q_start % BLOCK == 0, 'callers pad q to whole blocks'
        if valid is None:
            valid = (0, n)
        v0, nv = int(valid[0]), int(valid[1])
        rows = (self.Hk if union else self.H) * MB
        masks = torch.empty(rows, NB, dtype=torch.uint8, device=q.device)
        self._select(q[v0:v0 + nv], q_start + v0, q_start // BLOCK, MB, km, NB,
                     SA_SELECT_KV_UNION if union else SA_SELECT_PER_HEAD, masks=masks)
        return masks.view(self.Hk if union else self.H, MB, NB).bool()

    # -------------------------------------------------------------------------------------------
    # forward paths
    # -------------------------------------------------------------------------------------------
    @torch.no_grad()
    def forward(self, q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, q_start: int,
                out: torch.Tensor | None = None) -> torch.Tensor:
        """Block-sparse attention of q [n, H, D] (bf16, positions q_start..) over NHD k, v [kv_len, Hk, D]
        with the kernel this instance was made for."""
        run = self.forward_sm120fp8 if self.kernel == 'sm120fp8' else self.forward_sm120
        return run(q, k, v, q_start, out)

    def _out(self, out, n, dev):
        if out is not None and out.stride(-1) == 1 and out.stride(0) % 8 == 0 and out.stride(1) % 8 == 0 \
                and out.data_ptr() % 16 == 0:
            return out, False
        return torch.empty(n, self.H, self.D, dtype=torch.bfloat16, device=dev), out is not None

    @torch.no_grad()
    def forward_sm120(self, q, k, v, q_start, out=None, km=None, kv_pages=None):
        """BF16 kernel, one block list per query head and BLOCK-row query block.  k and v are NHD
        [T, Hk, D]; rows T > q_start + n are not read.  km: the request's cached fp32 block means
        [Hk, ceil((q_start + n) / BLOCK), D], else they are pooled here from k.  Makes no host sync.
        kv_pages: (key_cache, value_cache, table) read in place by the kernel instead of k and v (which
        may then be None; km is required): vLLM's paged caches [num_pages, page, Hk, D] and the
        request's int32 page-table row, holding at least q_start + n keys."""
        n = q.shape[0]
        kv_len = q_start + n
        if kv_pages is not None:
            if km is None:
                raise ValueError('forward_sm120: kv_pages needs km')
            if kv_pages[2].shape[0] * kv_pages[0].shape[1] < kv_len:
                raise AssertionError('the page table holds fewer keys than q_start + n')
        elif k.shape[0] < kv_len:
            raise AssertionError('k holds fewer rows than q_start + n')
        B = BLOCK
        front = q_start % B
        M = _cdiv(front + n, B) * B
        MB = M // B
        qs = q_start - front
        dev = q.device
        t0 = self._tick()
        if km is None:
            km = self._km_from_keys(k, _cdiv(kv_len, B))
        if FP8_EMULATE:
            if kv_pages is not None:
                raise ValueError('forward_sm120: FP8 emulation reads gathered k and v, not kv_pages')
            q, k, v = (_fp8_round(t, FP8_EMULATE, name) for t, name in ((q, 'q'), (k, 'k'), (v, 'v')))
        NB = km.shape[1]
        counts = torch.empty(self.H * MB, dtype=torch.int32, device=dev)
        lists = torch.empty(self.H * MB, NB, dtype=torch.int32, device=dev)
        self._select(q, q_start, qs // B, MB, km, NB, SA_SELECT_PER_HEAD, counts=counts, lists=lists)
        t1 = self._tick()
        o, copy_back = self._out(out, n, dev)
        ev0, ev1 = self._attn_events()
        if ev0 is not None:
            ev0.record()
        if kv_pages is not None:
            ops.attn_bf16_paged(q, kv_pages[0], kv_pages[1], kv_pages[2], o, kv_len, front, qs, counts, lists, B,
                                self.scale, q_block=B)
        else:
            ops.attn_bf16(q, k[:kv_len], v[:kv_len], o, kv_len, front, qs, counts, lists, B, self.scale, q_block=B)
        if ev1 is not None:
            ev1.record()
        self.last_counts, self.last_lists = counts, lists
        self._account(t0, t1, self._tick(), qs // B, MB, counts.sum())
        if out is None:
            return o
        if copy_back:
            out.copy_(o)
        return out

    @torch.no_grad()
    def forward_sm120fp8(self, q, k, v, q_start, out=None, km=None, scales=None, kv8=None, k_rows=None):
        """FP8 (e4m3) kernel over 128-row query blocks; k, v NHD [T, Hk, D] bf16, quantised here.

        scales: the request's (sq, sk, sv), each a Python float (per tensor, the reference's scales) or
        a sequence of per-head floats (H for q, Hk for k and v); the hook caches them per layer and
        request.  When absent they are taken from this call's per-tensor amax (three device syncs).  kv8: optional (k8, v8) uint8
        [kv_len, Hk, D] already quantised with these scales (`_cached_kv8`); then k and v are not
        read here and may be None (with km and scales given), k_rows then standing for k.shape[0]
        (the selection covers ceil(k_rows / BLOCK) key blocks, as with the key tensor itself).
        """
        BM = 128
        B = BLOCK
        n = q.shape[0]
        kv_len = q_start + n
        if k is None or v is None:
            if km is None or scales is None or kv8 is None:
                raise ValueError('forward_sm120fp8: k and v may be omitted only with km, scales and kv8')
            k_rows = kv_len if k_rows is None else k_rows
        else:
            k_rows = k.shape[0] if k_rows is None else k_rows
        assert k_rows >= kv_len
        front = q_start % BM
        M = _cdiv(front + n, BM) * BM
        MB = M // B
        qs = q_start - front
        dev = q.device
        need = max(_cdiv(k_rows, B) * B, qs + M)
        nb_need = need // B
        t0 = self._tick()
        if km is None:
            km = self._km_from_keys(k, _cdiv(kv_len, B))
        if scales is None:
            amax = torch.cat([ops.absmax(t if t.stride(-1) == 1 else t.contiguous(), per_head=False)
                              for t in (q, k, v)]).clamp_min_(1e-6).tolist()
            scales = tuple(a / 448.0 for a in amax)
        inv_q, inv_k, inv_v, s_q, s_k, s_v = _scale_views(dev, scales)
        q8 = torch.empty(n, self.H, self.D, dtype=torch.uint8, device=dev)
        rows = self.H * (M // BM)
        counts = torch.empty(rows, dtype=torch.int32, device=dev)
        lists = torch.empty(rows, nb_need, dtype=torch.int32, device=dev)
        self._select(q, q_start, qs // B, MB, km, nb_need, SA_SELECT_PAIR_UNION if B == 64 else SA_SELECT_PER_HEAD,
                     counts=counts, lists=lists, q8=q8, inv_scale=inv_q)
        if kv8 is not None:
            k8, v8 = kv8
            if k8.shape[0] < kv_len or v8.shape[0] < kv_len:
                raise ValueError('kv8 holds fewer rows than q_start + n')
        else:
            k8 = torch.empty(kv_len, self.Hk, self.D, dtype=torch.uint8, device=dev)
            ops.quantize(k[:kv_len], inv_k, SA_QUANT_MUL_BF16, k8)
            v8 = torch.empty(kv_len, self.Hk, self.D, dtype=torch.uint8, device=dev)
            ops.quantize(v[:kv_len], inv_v, SA_QUANT_MUL_BF16, v8)
        t1 = self._tick()
        o, copy_back = self._out(out, n, dev)
        ev0, ev1 = self._attn_events()
        if ev0 is not None:
            ev0.record()
        ops.attn_fp8(q8, k8, v8, o, kv_len, front, qs, counts, lists, B, s_q, s_k, s_v, self.scale)
        if ev1 is not None:
            ev1.record()
        self.last_counts, self.last_lists = counts, lists
        self._account(t0, t1, self._tick(), qs // B, MB, counts.sum() * (BM // B))
        if out is None:
            return o
        if copy_back:
            out.copy_(o)
        return out

    def _account(self, t0, t1, t2, qblk0, MB, kept):
        """Statistics of one call: blocks a dense causal walk would visit (per query head: every block
        before the chunk for each of its MB query blocks, plus the causal triangle), kept blocks (a
        device tensor, summed without a sync), and with timing the select / run milliseconds."""
        if self.timing:
            self.stats['select_ms'] += t1 - t0
            self.stats['run_ms'] += t2 - t1
        self.stats['calls'] += 1
        self.stats['blocks_total'] += int(self.H * (qblk0 * MB + MB * (MB + 1) // 2))
        self._kept_acc = kept if self._kept_acc is None else self._kept_acc + kept

    def kept_fraction(self):
        """Blocks kept / causal blocks over all calls so far (one device sync); None before any call."""
        total = self.stats['blocks_total']
        return None if (self._kept_acc is None or total == 0) else int(self._kept_acc.item()) / total

    def _tick(self):
        """Host milliseconds after a device sync, only with timing=True (0 otherwise)."""
        if self.timing:
            torch.cuda.synchronize()
            return time.perf_counter() * 1e3
        return 0.0


def reference(q, k, v, q_start, masks=None):
    """fp32 causal attention of q [n, H, D] (positions q_start..) over head-major k, v [Hk, N, D], with
    optional per-KV-head block masks [Hk, MB, NB]: query row i uses mask row i // BLOCK (counted from
    q[0]), key j mask column j // BLOCK (the reference's `reference`, sparse_prefill.py:262-279).  Plain
    PyTorch: a checker, not a product path."""
    n, H, D = q.shape
    Hk, N, _ = k.shape
    g = H // Hk
    dev = q.device
    rows, keys = torch.arange(n, device=dev), torch.arange(N, device=dev)
    causal = keys[None, :] <= (rows + q_start)[:, None]                 # [n, N]
    out = torch.empty(n, H, D, dtype=torch.float32, device=dev)
    for hk in range(Hk):                                                 # one GQA group at a time
        allowed = causal
        if masks is not None:
            allowed = causal & masks[hk][(rows // BLOCK)[:, None], (keys // BLOCK)[None, :]]
        heads = slice(hk * g, (hk + 1) * g)
        scores = torch.einsum('ngd,jd->gnj', q[:, heads].float(), k[hk].float()) * D ** -0.5
        probs = torch.softmax(scores.masked_fill(~allowed, float('-inf')), dim=-1)
        out[:, heads] = torch.einsum('gnj,jd->ngd', probs, v[hk].float())
    return out


# ===============================================================================================
# Serving side: knobs, one SparsePrefill per attention shape, per-request caches keyed by
# (layer, first KV page), and the prefill hook vLLM's FlashAttention backend calls.
# ===============================================================================================
_CONFIG = None
_STATE: dict = {}
FP8_EMULATE = os.environ.get('SM120_SPARSE_FP8_EMULATE', '')      # '' | 'tensor' | 'token' (numerics experiment)


def _flag(value) -> bool:
    return str(value) not in ('0', 'false', 'False')


def _flag_or_empty(value) -> bool:
    return _flag(value) and str(value) != ''


class _Knob(NamedTuple):
    name: str            # key of config() and of the JSON file
    env: str             # environment variable; it wins over the file
    default: object
    parse: Callable


# The reference's SM120_SPARSE_* knobs (sparse_prefill.py:358-381) plus the FP8 KV cache switch.
_KNOBS = (
    _Knob('enabled', 'SM120_SPARSE_ATTN', 1, _flag),
    _Knob('tau', 'SM120_SPARSE_TAU', 0.95, float),
    _Knob('min_kv', 'SM120_SPARSE_MIN_KV', 8192, int),
    _Knob('min_q', 'SM120_SPARSE_MIN_Q', 1024, int),
    _Knob('kernel', 'SM120_SPARSE_KERNEL', 'sm120fp8', str),
    _Knob('fp8_pipeline', 'SM120_SPARSE_FP8_PIPELINE', 'tma', str),
    _Knob('fp8_kv_cache', 'SM120_SPARSE_FP8_KV_CACHE', 0, _flag_or_empty),   # keep e4m3 K/V per request
    _Knob('fp8_scales', 'SM120_SPARSE_FP8_SCALES', 'tensor', str),            # 'tensor' | 'head' e4m3 scales
)


def config() -> dict:
    """The knobs, read once: environment variable, else the JSON file named by SM120_SPARSE_CONFIG
    (for launchers that do not forward the environment), else the default."""
    global _CONFIG
    if _CONFIG is None:
        path = os.environ.get('SM120_SPARSE_CONFIG')
        from_file = json.loads(Path(path).read_text()) if path else {}
        _CONFIG = {kn.name: kn.parse(os.environ[kn.env] if kn.env in os.environ else from_file.get(kn.name, kn.default))
                   for kn in _KNOBS}
        print(f'[sm120-sparse] config {_CONFIG!r}', flush=True)
    return _CONFIG


def _state(num_heads, num_kv_heads, head_dim, device):
    """The SparsePrefill serving one (heads, KV heads, head_dim, device) shape, built on first use with
    the knobs of config()."""
    shape = (num_heads, num_kv_heads, head_dim, str(device))
    sp = _STATE.get(shape)
    if sp is None:
        knobs = config()
        sp = _STATE[shape] = SparsePrefill(num_heads, num_kv_heads, head_dim, device,
                                           **{k: knobs[k] for k in ('tau', 'min_kv', 'min_q', 'kernel', 'fp8_pipeline')})
    return sp


# amax axes of the SM120_SPARSE_FP8_EMULATE rounding: one scale per tensor, or per (row, head) for
# q and k and per (head, channel) for v
_EMULATE_AXES = {'tensor': dict(q=None, k=None, v=None), 'token': dict(q=(2,), k=(2,), v=(0,))}


def _fp8_round(x, mode, which):
    """x [rows, heads, D] through float8_e4m3fn and back with amax/448 scaling (the reference's
    FP8-emulation experiment, sparse_prefill.py:334-348); `which` is 'q', 'k' or 'v'."""
    xf = x.float()
    axes = _EMULATE_AXES['tensor' if mode == 'tensor' else 'token'][which]
    magnitude = xf.abs()
    peak = magnitude.amax() if axes is None else magnitude.amax(dim=axes, keepdim=True)
    step = peak.clamp_min(1e-6) / 448.0
    return (xf / step).to(torch.float8_e4m3fn).to(torch.float32).mul_(step).to(x.dtype)


class _DebugLines:
    """Prints at most `budget` lines prefixed '[sm120-sparse]' (SM120_SPARSE_DEBUG=N)."""

    def __init__(self, budget: int):
        self.budget = budget

    def __call__(self, msg: str) -> None:
        if self.budget > 0:
            self.budget -= 1
            print(f'[sm120-sparse] {msg}', flush=True)


_debug = _DebugLines(int(os.environ.get('SM120_SPARSE_DEBUG', '0')))


def _request_entry(cache: dict, key, q_start: int, continues, make):
    """Per-request cache discipline shared by the block-mean, scale and FP8 KV caches: the entry of
    (layer, first page) is reused when `continues(entry)` says the request's previous chunk ended at
    q_start (a recycled first page of another request never does), else a fresh one from `make()`
    replaces it, the oldest entry of the cache being dropped when it holds _KMEAN_MAX_ENTRIES.
    Returns (entry, fresh)."""
    entry = cache.get(key)
    if entry is not None and q_start > 0 and continues(entry):
        return entry, False
    if len(cache) >= _KMEAN_MAX_ENTRIES:
        del cache[next(iter(cache))]
    entry = cache[key] = make()
    return entry, True


_KMEAN_CACHE: dict = {}
_KMEAN_MAX_ENTRIES = 128


class _PagedRows(NamedTuple):
    """Rows 0 .. rows-1 of a request in one of vLLM's paged caches [num_pages, page, Hk, D]: position
    l is slot l % page of page table[l // page] (the request's int32 block-table row).  Stands for
    the gathered history `cache[table].reshape(-1, Hk, D)[:rows]` and is read in place."""
    cache: torch.Tensor
    table: torch.Tensor
    rows: int

    @property
    def shape(self):
        return (self.rows, self.cache.shape[2], self.cache.shape[3])


def _km_continues(q_start):
    return lambda e: e['nb'] >= q_start // BLOCK and e.get('last_kv') == q_start


def _km_entry(layer_key, first_page, q_start, end_block, Hk, D, dev):
    """(entry, rebuilt): the block-mean entry of (layer, request) for a chunk at q_start, its km grown
    (capacity doubling, at least to end_block blocks)."""
    def fresh():
        return {'km': torch.zeros(Hk, max(4096, end_block), D, dtype=torch.float32, device=dev), 'nb': 0,
                'last_kv': 0}
    entry, rebuilt = _request_entry(_KMEAN_CACHE, (layer_key, first_page), q_start, _km_continues(q_start), fresh)
    held = entry['km'].shape[1]
    if held < end_block:
        grown = entry['km'].new_zeros(Hk, max(end_block, 2 * held), D)
        grown[:, :held] = entry['km']
        entry['km'] = grown
    return entry, rebuilt


def km_slot(layer_key, first_page, q_start, kv_len, Hk, D, dev):
    """The km tensor [Hk, capacity, D] of a request's block-mean entry prepared for the chunk of keys
    q_start .. kv_len, for the producer of those keys to write their block means into at KV-write time
    (ops.rope_qkv(..., km=)); _cached_block_means(..., written=True) then only records them.  None
    when the entry does not continue at q_start (it is rebuilt from the key history instead)."""
    entry = _KMEAN_CACHE.get((layer_key, first_page))
    if q_start > 0 and (entry is None or not _km_continues(q_start)(entry)):
        return None
    entry, _ = _km_entry(layer_key, first_page, q_start, -(-kv_len // BLOCK), Hk, D, dev)
    entry['slot'] = (q_start, kv_len)
    return entry['km']


def _cached_block_means(layer_key, first_page, key_chunk, q_start, kv_len, key_all=None, written=False, q8=None,
                        inv_scale=None):
    """fp32 block means [Hk, NB, D] of a request's keys, NB = ceil((q_start + n) / BLOCK), kept per
    (layer, request) and extended by each chunk (sparse_prefill.py:398-447).

    key_chunk [n, Hk, D] holds the keys at positions q_start..; the entry grows by the chunk's blocks.
    A request whose cached entry does not end at q_start (new request, recycled first page, skipped
    chunks) is rebuilt from key_all, its history: a tensor [>= q_start, Hk, D], or _PagedRows read in
    place (then covering the chunk too, positions 0 .. kv_len).  As in the reference, a chunk that
    starts inside a block replaces that block's mean by the mean of its own rows there; only a rebuild
    averages the block's history rows and chunk rows together.
    written: the chunk's means were written into the km_slot of this chunk by the keys' producer.
    q8 / inv_scale: e4m3 copy of the chunk's keys written in the same pass (continuing entries only).
    """
    B = BLOCK
    n, Hk, D = key_chunk.shape
    end_block = -(-(q_start + n) // B)
    if written:
        entry = _KMEAN_CACHE.get((layer_key, first_page))
        if entry is None or entry.pop('slot', None) != (q_start, kv_len):
            raise RuntimeError('block means marked written without a km_slot for this chunk')
        entry['nb'], entry['last_kv'] = end_block, kv_len
        return entry['km'][:, :end_block]
    entry, rebuilt = _km_entry(layer_key, first_page, q_start, end_block, Hk, D, key_chunk.device)
    rows, pos0 = key_chunk, q_start                  # rows whose block means are (re)computed below
    if rebuilt and q_start > 0:
        if key_all is None:
            raise RuntimeError('stale block-mean cache entry and no key history to rebuild it')
        if q8 is not None:
            raise RuntimeError('a fused e4m3 key copy needs a continuing block-mean entry')
        if isinstance(key_all, _PagedRows):
            ops.block_means_paged(key_all.cache, key_all.table, 0, q_start + n, B, entry['km'], 0)
            rows = key_chunk[:0]
        else:
            whole = q_start - q_start % B            # history rows that fill complete blocks
            if whole:
                ops.block_means(key_all[:whole], 0, B, entry['km'], 0)
            if whole < q_start:                      # the block the chunk continues: history + chunk rows
                rows, pos0 = torch.cat([key_all[whole:q_start], key_chunk], 0), whole
    if rows.shape[0]:
        ops.block_means(rows, pos0, B, entry['km'], 0, q8=q8, inv_scale=inv_scale)
    entry['nb'], entry['last_kv'] = end_block, kv_len
    return entry['km'][:, :end_block]


_SCALE_TENSORS: dict = {}


def _scale_list(x) -> tuple:
    """A scale as a tuple of floats: one for a per-tensor scale, one per head otherwise."""
    return tuple(float(a) for a in x) if isinstance(x, (tuple, list)) else (float(x),)


def _scale_views(dev, scales):
    """Device fp32 views (1/sq, 1/sk, 1/sv, sq, sk, sv) of one scale triple, each of one element
    (per-tensor scale) or one per head, kept per (device, triple).

    A host tensor copied from pageable memory makes the copy wait for the whole stream (a device
    sync every chunk); the triple is fixed per request and layer, so it is staged once through
    pinned memory and reused."""
    parts = [_scale_list(x) for x in scales]
    flat = [1.0 / a for p in parts for a in p] + [a for p in parts for a in p]
    dev = torch.device(dev)
    if dev.type != 'cuda':                                      # host-side tests with fake ops
        t = torch.tensor(flat, dtype=torch.float32, device=dev)
    else:
        key = (dev.index if dev.index is not None else torch.cuda.current_device(), tuple(parts))
        hit = _SCALE_TENSORS.get(key)
        if hit is None:
            if len(_SCALE_TENSORS) >= 4 * _KMEAN_MAX_ENTRIES:
                _SCALE_TENSORS.pop(next(iter(_SCALE_TENSORS)))
            host = torch.tensor(flat, dtype=torch.float32).pin_memory()
            hit = (host.to(dev, non_blocking=True), host)      # the pinned source lives as long as the entry
            _SCALE_TENSORS[key] = hit
        t = hit[0]
    sizes = [len(p) for p in parts] * 2
    return tuple(torch.split(t, sizes))


def _kv_scale_key(scales) -> tuple:
    """The part of a scale triple the e4m3 K/V bytes depend on (k and v scales)."""
    return _scale_list(scales[1]), _scale_list(scales[2])


_KV8_CACHE: dict = {}
# Device memory the FP8 KV cache may hold over all (layer, request) entries; the oldest entries are
# dropped past it (a dropped request is rebuilt from its K/V pages on its next chunk).
KV8_CACHE_MAX_BYTES = int(float(os.environ.get('SM120_SPARSE_FP8_KV_CACHE_GB', '16')) * (1 << 30))


def _kv8_bytes(entry) -> int:
    return entry['k8'].numel() + entry['v8'].numel()


def _kv8_evict(keep_key):
    """Drop the oldest entries (never keep_key) until the cache is within KV8_CACHE_MAX_BYTES."""
    total = sum(_kv8_bytes(e) for e in _KV8_CACHE.values())
    for key in list(_KV8_CACHE):
        if total <= KV8_CACHE_MAX_BYTES:
            break
        if key != keep_key:
            total -= _kv8_bytes(_KV8_CACHE.pop(key))


def _quantize_into(src, lo, hi, row0, inv, out8):
    """e4m3 (MUL_BF16) of key/value positions lo .. hi-1 into out8[lo:hi]; src is a tensor holding
    positions row0 .. or _PagedRows (read in place)."""
    if hi <= lo:
        return
    if isinstance(src, _PagedRows):
        ops.quantize_paged(src.cache, src.table, lo, inv, SA_QUANT_MUL_BF16, out8[lo:hi])
    else:
        ops.quantize(src[lo - row0:hi - row0], inv, SA_QUANT_MUL_BF16, out8[lo:hi])


def _kv8_entry(layer_key, first_page, q_start, kv_len, scales, Hk, D, dev):
    """(entry, lo): the FP8 KV cache entry of (layer, request) for a chunk ending at kv_len, grown to
    hold kv_len rows, with rows lo .. kv_len still to be quantised (lo = q_start for an entry that
    continues at q_start with the same scales, else 0: a fresh entry)."""
    kv_key = _kv_scale_key(scales)
    key = (layer_key, first_page)

    def fresh():
        rows = max(kv_len, 8192)
        return {'k8': torch.empty(rows, Hk, D, dtype=torch.uint8, device=dev),
                'v8': torch.empty(rows, Hk, D, dtype=torch.uint8, device=dev), 'rows': 0, 'scales': kv_key,
                'inv': _scale_views(dev, scales)[1:3]}
    entry, _ = _request_entry(_KV8_CACHE, key, q_start,
                              lambda e: e['rows'] == q_start and e['scales'] == kv_key, fresh)
    lo = entry['rows']
    if entry['k8'].shape[0] < kv_len:
        cap = max(kv_len, 2 * entry['k8'].shape[0])
        for name in ('k8', 'v8'):
            grown = torch.empty(cap, Hk, D, dtype=torch.uint8, device=dev)
            grown[:lo] = entry[name][:lo]
            entry[name] = grown
    _kv8_evict(key)
    return entry, lo


def _cached_kv8(layer_key, first_page, k, v, q_start, kv_len, scales, k_row0=0):
    """Per-(layer, request) e4m3 K and V [kv_len, Hk, D] (uint8 views), each row quantised once.

    The FP8 path quantises the whole key/value history with the request's scales on every chunk
    (sparse_prefill.py:230-233); the scales are cached per request, so rows quantised for an earlier
    chunk never change.  An entry contiguous with this chunk (its last row is q_start) and made with
    the same scales only quantises rows q_start..kv_len; otherwise it is rebuilt from k, v.  k and v
    are NHD tensors holding sequence rows k_row0 .. k_row0 + len (k_row0 > 0 only for a contiguous
    entry: a rebuild needs every row from 0), or _PagedRows read in place.  The bytes are the same as
    re-quantising the history.
    """
    kv_key = _kv_scale_key(scales)
    prior = _KV8_CACHE.get((layer_key, first_page))
    if k_row0 and not (prior is not None and q_start > 0 and prior['rows'] == q_start and prior['scales'] == kv_key):
        raise RuntimeError('stale FP8 KV cache entry and no key/value rows before %d to rebuild it' % k_row0)
    entry, lo = _kv8_entry(layer_key, first_page, q_start, kv_len, scales, k.shape[1], k.shape[2],
                           (k.cache if isinstance(k, _PagedRows) else k).device)
    if kv_len > lo:
        for src in (k, v):
            if not isinstance(src, _PagedRows) and (src.shape[0] < kv_len - k_row0 or lo < k_row0):
                raise ValueError('_cached_kv8: k/v do not hold rows %d..%d' % (lo, kv_len))
        _quantize_into(k, lo, kv_len, k_row0, entry['inv'][0], entry['k8'])
        _quantize_into(v, lo, kv_len, k_row0, entry['inv'][1], entry['v8'])
    entry['rows'] = kv_len
    return entry['k8'][:kv_len], entry['v8'][:kv_len]


def _kv8_scratch(k, v, kv_len, scales, dev):
    """e4m3 K and V of positions 0 .. kv_len-1 for one chunk (no FP8 KV cache: the whole history is
    quantised every chunk, as in the reference), read in place from the pages."""
    inv_k, inv_v = _scale_views(dev, scales)[1:3]
    out = []
    for src, inv in ((k, inv_k), (v, inv_v)):
        t = torch.empty(kv_len, src.shape[1], src.shape[2], dtype=torch.uint8, device=dev)
        _quantize_into(src, 0, kv_len, 0, inv, t)
        out.append(t)
    return tuple(out)


def _fp8_warm(layer_key, first_page, q_start) -> bool:
    """True when the block-mean, scale and FP8 KV caches of this (layer, request) all continue at
    q_start, so a chunk needs none of the key/value history (only its own rows)."""
    key = (layer_key, first_page)
    km, sc, kv = _KMEAN_CACHE.get(key), _SCALE_CACHE.get(key), _KV8_CACHE.get(key)
    return (q_start > 0 and km is not None and km.get('last_kv') == q_start and km['nb'] >= q_start // BLOCK
            and sc is not None and sc['last_kv'] == q_start and kv is not None and kv['rows'] == q_start
            and kv['scales'] == _kv_scale_key(sc['scales']))


_SCALE_CACHE: dict = {}
SCALE_MARGIN = 1.5


def _cached_scales(layer_key, first_page, q, k, v, q_start, per_head: bool = False):
    """e4m3 scales (sq, sk, sv) of a request, fixed at its first sparse chunk: amax of that chunk's q and
    of k, v (the history so far) / 448, times SCALE_MARGIN for the rows still to come
    (sparse_prefill.py:450-469).  per_head (SM120_SPARSE_FP8_SCALES=head): each of the three is a
    tuple with one scale per head (H for q, Hk for k and v) instead of one per tensor.  One host sync
    when an entry is made."""
    def fresh():
        peaks = [(ops.absmax_paged(t.cache, t.table, 0, t.rows, per_head) if isinstance(t, _PagedRows) else
                  ops.absmax(t if t.stride(-1) == 1 else t.contiguous(), per_head=per_head)).clamp_min(1e-6)
                 for t in (q, k, v)]
        if not per_head:
            return {'scales': tuple(a * SCALE_MARGIN / 448.0 for a in torch.cat(peaks).tolist()), 'last_kv': 0}
        sizes = [int(p.numel()) for p in peaks]
        host = torch.cat(peaks).tolist()
        parts, i = [], 0
        for n in sizes:
            parts.append(tuple(a * SCALE_MARGIN / 448.0 for a in host[i:i + n]))
            i += n
        return {'scales': tuple(parts), 'last_kv': 0}
    entry, _ = _request_entry(_SCALE_CACHE, (layer_key, first_page), q_start,
                              lambda e: e['last_kv'] == q_start, fresh)
    entry['last_kv'] = q_start + q.shape[0]
    return entry['scales']


_META_HOST: dict = {'ref': None, 'vals': None}


def _host_metadata(attn_metadata):
    """(query_start_loc, seq_lens, first page of each request) as host lists.  vLLM hands every
    attention layer of a step the same metadata object, so the device reads (each a stream sync)
    happen once per step, not once per layer: the lists are kept for the object last seen, held by a
    weak reference so a later object can never be mistaken for it.  Host copies the backend keeps
    (`query_start_loc_cpu`, `seq_lens_cpu`) are used when present."""
    ref = _META_HOST['ref']
    if ref is not None and ref() is attn_metadata:
        return _META_HOST['vals']
    qsl = getattr(attn_metadata, 'query_start_loc_cpu', None)
    qsl = (qsl if qsl is not None else attn_metadata.query_start_loc).tolist()
    seq_lens = getattr(attn_metadata, 'seq_lens_cpu', None)
    seq_lens = (seq_lens if seq_lens is not None else attn_metadata.seq_lens).tolist()
    first_pages = attn_metadata.block_table[:len(seq_lens), 0].tolist()
    vals = (qsl, seq_lens, first_pages)
    try:
        _META_HOST['ref'], _META_HOST['vals'] = weakref.ref(attn_metadata), vals
    except TypeError:                                   # not weak-referenceable: no reuse
        _META_HOST['ref'], _META_HOST['vals'] = None, None
    return vals


def _hook_applies(impl, attn_metadata, cfg) -> bool:
    """Checks that need no device read: the knob is on, the layer is causal full attention, the batch
    holds a chunk long enough somewhere, and no CUDA graph is being captured (decode batches are
    captured; reading the metadata there would be a device-to-host copy during capture)."""
    if not cfg['enabled']:
        return False
    window = getattr(impl, 'sliding_window', None)
    if attn_metadata.causal is not True or (window is not None and any(int(w) >= 0 for w in window)):
        _debug(f'not causal full attention (causal={attn_metadata.causal!r}, window={window!r}): dense path')
        return False
    long_enough = attn_metadata.max_query_len >= cfg['min_q'] and attn_metadata.max_seq_len >= cfg['min_kv']
    return long_enough and not torch.cuda.is_current_stream_capturing()


class _Request(NamedTuple):
    index: int           # row of the block table
    q0: int              # its rows in this batch's query / key / output tensors
    q1: int
    kv_len: int          # keys of the request after this chunk
    first_page: int      # identifies the request in the per-request caches

    @property
    def n(self) -> int:
        return self.q1 - self.q0

    @property
    def q_start(self) -> int:
        return self.kv_len - self.n


@torch.no_grad()
def try_sparse_forward(impl, query, key, key_cache, value_cache, output, attn_metadata) -> bool:
    """Prefill hook of vLLM's FlashAttention backend (sparse_prefill.py:472-535): writes the attention
    output of every request of the batch and returns True when at least one request has a chunk of
    >= min_q queries over >= min_kv keys; those run block-sparse, the others (short chunks, decode
    steps) get the backend's dense paged call.  Returns False, writing nothing, otherwise.

    query, key, output are the batch's token-major tensors (num_actual_tokens rows); the paged caches
    key_cache and value_cache are [num_blocks, page, Hk, D].
    """
    cfg = config()
    if not _hook_applies(impl, attn_metadata, cfg):
        return False
    starts, seq_lens, first_pages = _host_metadata(attn_metadata)
    requests = [_Request(r, starts[r], starts[r + 1], seq_lens[r], first_pages[r]) for r in range(len(seq_lens))]
    sparse = [rq.n >= cfg['min_q'] and rq.kv_len >= cfg['min_kv'] for rq in requests]
    if not any(sparse):
        return False
    _debug(f'{sum(sparse)} of {len(requests)} requests block-sparse; chunk lengths '
           f'{[rq.n for rq in requests]}, key lengths {[rq.kv_len for rq in requests]}')
    sp = _state(query.shape[1], key_cache.shape[2], query.shape[2], query.device)
    table = attn_metadata.block_table
    for rq, is_sparse in zip(requests, sparse):
        q_r, o_r = query[rq.q0:rq.q1], output[rq.q0:rq.q1]
        if is_sparse:
            _sparse_request(sp, cfg, id(impl), rq, q_r, key[rq.q0:rq.q1], key_cache, value_cache, o_r,
                            table[rq.index])
        else:
            _dense_request(impl, q_r, key_cache, value_cache, o_r, table[rq.index], rq.n, rq.kv_len)
    return True


def _sparse_request(sp, cfg, layer, rq, q_r, key_r, key_cache, value_cache, o_r, pages_row):
    """One long prefill chunk through the block-sparse path.  The caches of (layer, first page) carry
    the request's block means, e4m3 scales and (with fp8_kv_cache) e4m3 K/V from chunk to chunk.
    The key/value history is read in place from the pages (the reference gathers it into contiguous
    tensors on every chunk, sparse_prefill.py:521-522): by the paged block-mean, absmax and e4m3
    kernels, and by the BF16 attention kernel itself."""
    page = key_cache.shape[1]
    npages = -(-rq.kv_len // page)
    q_start, kv_len = rq.q_start, rq.kv_len
    table = pages_row[:npages]
    if table.dtype != torch.int32 or not table.is_contiguous():
        table = table.to(torch.int32).contiguous()
    k_src, v_src = _PagedRows(key_cache, table, kv_len), _PagedRows(value_cache, table, kv_len)
    per_head = cfg.get('fp8_scales') == 'head'
    if sp.kernel != 'sm120fp8':
        km = _cached_block_means(layer, rq.first_page, key_r, q_start, kv_len, key_all=k_src)
        if ops.paged_attention_supported(page) and not FP8_EMULATE:
            sp.forward_sm120(q_r, None, None, q_start, out=o_r, km=km, kv_pages=(key_cache, value_cache, table))
        else:                                  # page sizes the kernel does not read in place: gather
            pages = table.long()
            Hk, D = key_cache.shape[2], key_cache.shape[3]
            sp.forward_sm120(q_r, key_cache[pages].reshape(-1, Hk, D), value_cache[pages].reshape(-1, Hk, D), q_start,
                             out=o_r, km=km)
        return
    if cfg['fp8_kv_cache'] and _fp8_warm(layer, rq.first_page, q_start):
        # block means, scales and the e4m3 history all continue at this chunk: only the chunk's own
        # rows are read, its keys once for both their block means and their e4m3 copy
        scales = _cached_scales(layer, rq.first_page, q_r, None, None, q_start, per_head=per_head)
        entry, lo = _kv8_entry(layer, rq.first_page, q_start, kv_len, scales, key_r.shape[1], key_r.shape[2],
                               q_r.device)
        if lo != q_start:
            raise RuntimeError('FP8 KV cache entry does not continue at the chunk')
        km = _cached_block_means(layer, rq.first_page, key_r, q_start, kv_len, q8=entry['k8'][q_start:kv_len],
                                 inv_scale=entry['inv'][0])
        _quantize_into(v_src, q_start, kv_len, 0, entry['inv'][1], entry['v8'])
        entry['rows'] = kv_len
        kv8 = (entry['k8'][:kv_len], entry['v8'][:kv_len])
    else:
        km = _cached_block_means(layer, rq.first_page, key_r, q_start, kv_len, key_all=k_src)
        scales = _cached_scales(layer, rq.first_page, q_r, k_src, v_src, q_start, per_head=per_head)
        if cfg['fp8_kv_cache']:
            kv8 = _cached_kv8(layer, rq.first_page, k_src, v_src, q_start, kv_len, scales)
        else:
            kv8 = _kv8_scratch(k_src, v_src, kv_len, scales, q_r.device)
    sp.forward_sm120fp8(q_r, None, None, q_start, out=o_r, km=km, scales=scales, kv8=kv8, k_rows=npages * page)


def _dense_request(impl, query, key_cache, value_cache, output, bt_row, n, kv_len):
    """Dense paged attention for one request of a mixed batch through the call the backend itself makes
    (vLLM's flash_attn_varlen_func; sparse_prefill.py:538-550)."""
    from vllm.vllm_flash_attn import flash_attn_varlen_func
    dev = query.device
    window = getattr(impl, 'sliding_window', None)
    args = dict(q=query, k=key_cache, v=value_cache, out=output,
                cu_seqlens_q=torch.tensor([0, n], dtype=torch.int32, device=dev), max_seqlen_q=n,
                seqused_k=torch.tensor([kv_len], dtype=torch.int32, device=dev), max_seqlen_k=kv_len,
                softmax_scale=impl.scale, causal=True, alibi_slopes=getattr(impl, 'alibi_slopes', None),
                window_size=list(window) if window is not None else None, block_table=bt_row.unsqueeze(0),
                softcap=getattr(impl, 'logits_soft_cap', 0.0), fa_version=getattr(impl, 'vllm_flash_attn_version', 2))
    flash_attn_varlen_func(**args)
