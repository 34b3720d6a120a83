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
import os
import weakref

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
        self.H, self.Hk, self.D = num_heads, num_kv_heads, head_dim
        self.g = num_heads // num_kv_heads
        self.tau, self.min_kv, self.min_q = tau, min_kv, min_q
        self.scale = head_dim ** -0.5
        self.wrapper = None
        self.stats = {'calls': 0, 'blocks_total': 0, 'blocks_kept': 0, 'plan_ms': 0.0, 'run_ms': 0.0, 'select_ms': 0.0}
        self._kept_acc = None
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
        return q_len >= self.min_q and kv_len >= self.min_kv

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

    def _pool_q(self, q, q_start, qs, MB, q8=None, inv_scale=None):
        """Pooled query blocks qm [MB, H, D] (block m at aligned position qs + m*BLOCK) of q [n, H, D] at
        q_start; optionally writes e4m3(bf16(q * inv_scale)) into q8 in the same pass."""
        qm = torch.zeros(MB, self.H, self.D, dtype=torch.float32, device=q.device)
        if q.shape[0]:
            ops.block_means(q, q_start, BLOCK, qm.permute(1, 0, 2), qs // BLOCK, q8=q8, inv_scale=inv_scale)
        return qm

    @torch.no_grad()
    def block_masks(self, q: torch.Tensor, k, q_start: int, valid=None, union: bool = True, km=None):
        """q [n, H, D]; k [Hk, N, D] (head-major) or [N, Hk, D] (NHD) with N a multiple of BLOCK;
        q_start = absolute position of q[0]. Returns bool masks [Hk, MB, NB] (union over the query
        heads of each KV head) or [H, MB, NB] per query head when union=False.
        """
        n = q.shape[0]
        if km is not None:                                   # cached block means [Hk, NB, D] (fp32)
            NB = km.shape[1]
        else:
            head_major = k.shape[0] == self.Hk and k.shape[1] != self.Hk
            kn = k.permute(1, 0, 2) if head_major else k     # NHD view
            NB = kn.shape[0] // BLOCK
            km = self._km_from_keys(kn, NB)
        MB = _cdiv(n, BLOCK)
        assert n % BLOCK == 0 and q_start % BLOCK == 0, 'callers pad q to whole blocks'
        if valid is None:
            valid = (0, n)
        v0, nv = int(valid[0]), int(valid[1])
        qm = torch.zeros(MB, self.H, self.D, dtype=torch.float32, device=q.device)
        if nv > 0:
            ops.block_means(q[v0:v0 + nv], q_start + v0, BLOCK, qm.permute(1, 0, 2), q_start // BLOCK)
        rows = (self.Hk if union else self.H) * MB
        masks = torch.empty(rows, NB, dtype=torch.uint8, device=q.device)
        ops.select(qm, km, self.H, self.Hk, NB, q_start // BLOCK, self.scale, self.tau,
                   SA_SELECT_KV_UNION if union else SA_SELECT_PER_HEAD, masks=masks)
        return masks.view(self.Hk if union else self.H, MB, NB).bool()

    # -------------------------------------------------------------------------------------------
    # forward paths
    # -------------------------------------------------------------------------------------------
    @torch.no_grad()
    def forward(self, q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, q_start: int,
                out: torch.Tensor | None = None) -> torch.Tensor:
        """q [n, H, D] bf16 at absolute positions q_start..; k, v [kv_len, Hk, D] (NHD)."""
        if self.kernel == 'sm120':
            return self.forward_sm120(q, k, v, q_start, out)
        return self.forward_sm120fp8(q, k, v, q_start, out)

    def _out(self, out, n, dev):
        if out is not None and out.stride(-1) == 1 and out.stride(0) % 8 == 0 and out.stride(1) % 8 == 0 \
                and out.data_ptr() % 16 == 0:
            return out, False
        return torch.empty(n, self.H, self.D, dtype=torch.bfloat16, device=dev), out is not None

    @torch.no_grad()
    def forward_sm120(self, q, k, v, q_start, out=None, km=None):
        """Per-query-head block-sparse attention, BF16 kernel.

        k, v: NHD [T, Hk, D] with T >= q_start + n (rows beyond the sequence are ignored);
        km: optional cached block means [Hk, ceil((q_start+n)/BLOCK), D] (fp32). No host syncs.
        """
        n = q.shape[0]
        kv_len = q_start + n
        assert k.shape[0] >= kv_len
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
            q, k, v = _fp8_round(q, FP8_EMULATE, 'q'), _fp8_round(k, FP8_EMULATE, 'k'), _fp8_round(v, FP8_EMULATE, 'v')
        NB = km.shape[1]
        qm = self._pool_q(q, q_start, qs, MB)
        counts = torch.empty(self.H * MB, dtype=torch.int32, device=dev)
        lists = torch.empty(self.H * MB, NB, dtype=torch.int32, device=dev)
        ops.select(qm, km, self.H, self.Hk, NB, qs // B, self.scale, self.tau, SA_SELECT_PER_HEAD,
                   counts=counts, lists=lists)
        t1 = self._tick()
        o, copy_back = self._out(out, n, dev)
        ev0, ev1 = self._attn_events()
        if ev0 is not None:
            ev0.record()
        ops.attn_bf16(q, k[:kv_len], v[:kv_len], o, kv_len, front, qs, counts, lists, B, self.scale, q_block=B)
        if ev1 is not None:
            ev1.record()
        self.last_counts, self.last_lists = counts, lists
        t2 = self._tick()
        if self.timing:
            self.stats['select_ms'] += t1 - t0
            self.stats['run_ms'] += t2 - t1
        self.stats['calls'] += 1
        self.stats['blocks_total'] += int(self.H * ((qs // B) * MB + MB * (MB + 1) // 2))
        self._kept_acc = counts.sum() if self._kept_acc is None else self._kept_acc + counts.sum()
        if out is None:
            return o
        if copy_back:
            out.copy_(o)
        return out

    @torch.no_grad()
    def forward_sm120fp8(self, q, k, v, q_start, out=None, km=None, scales=None, kv8=None, k_rows=None):
        """FP8 (e4m3) path, 128-row query blocks; k, v NHD [T, Hk, D] bf16, quantised here.

        scales: (sq, sk, sv) python floats (per-request, per-layer, cached by the caller); without
        them per-call amax scales are used (three device syncs).  kv8: optional (k8, v8) uint8
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
        sq, sk, sv = scales
        st = _scale_tensor(dev, sq, sk, sv)
        inv, sc = st[0:3], st[3:6]
        q8 = torch.empty(n, self.H, self.D, dtype=torch.uint8, device=dev)
        qm = self._pool_q(q, q_start, qs, MB, q8=q8, inv_scale=inv[0:1])
        rows = self.H * (M // BM)
        counts = torch.empty(rows, dtype=torch.int32, device=dev)
        lists = torch.empty(rows, nb_need, dtype=torch.int32, device=dev)
        ops.select(qm, km, self.H, self.Hk, nb_need, qs // B, self.scale, self.tau,
                   SA_SELECT_PAIR_UNION if B == 64 else SA_SELECT_PER_HEAD, counts=counts, lists=lists)
        if kv8 is not None:
            k8, v8 = kv8
            if k8.shape[0] < kv_len or v8.shape[0] < kv_len:
                raise ValueError('kv8 holds fewer rows than q_start + n')
        else:
            k8 = torch.empty(kv_len, self.Hk, self.D, dtype=torch.uint8, device=dev)
            ops.quantize(k[:kv_len], inv[1:2], SA_QUANT_MUL_BF16, k8)
            v8 = torch.empty(kv_len, self.Hk, self.D, dtype=torch.uint8, device=dev)
            ops.quantize(v[:kv_len], inv[2:3], SA_QUANT_MUL_BF16, v8)
        t1 = self._tick()
        o, copy_back = self._out(out, n, dev)
        ev0, ev1 = self._attn_events()
        if ev0 is not None:
            ev0.record()
        ops.attn_fp8(q8, k8, v8, o, kv_len, front, qs, counts, lists, B, sc[0:1], sc[1:2], sc[2:3], self.scale)
        if ev1 is not None:
            ev1.record()
        self.last_counts, self.last_lists = counts, lists
        t2 = self._tick()
        if self.timing:
            self.stats['select_ms'] += t1 - t0
            self.stats['run_ms'] += t2 - t1
        self.stats['calls'] += 1
        self.stats['blocks_total'] += int(self.H * ((qs // B) * MB + MB * (MB + 1) // 2))
        kept = counts.sum() * (BM // B)
        self._kept_acc = kept if self._kept_acc is None else self._kept_acc + kept
        if out is None:
            return o
        if copy_back:
            out.copy_(o)
        return out

    def kept_fraction(self):
        """Blocks kept / causal blocks over all calls so far (one device sync)."""
        if self._kept_acc is None or not self.stats['blocks_total']:
            return None
        return int(self._kept_acc.item()) / self.stats['blocks_total']

    def _tick(self):
        if not self.timing:
            return 0.0
        torch.cuda.synchronize()
        import time
        return time.time() * 1000.0


def reference(q, k, v, q_start, masks=None):
    """fp32 reference: causal attention of q [n,H,D] (positions q_start..) over k,v [Hk,N,D], optional
    per-KV-head block masks [Hk, MB, NB] (sparse_prefill.py:262-279).  Plain PyTorch: a checker, not a
    product path."""
    n, H, D = q.shape
    Hk, N, _ = k.shape
    g = H // Hk
    pos_q = q_start + torch.arange(n, device=q.device)
    pos_k = torch.arange(N, device=q.device)
    allowed = pos_k[None, :] <= pos_q[:, None]
    outs = []
    for h in range(H):
        s = (q[:, h].float() @ k[h // g].float().T) * D ** -0.5
        mask = allowed.clone()
        if masks is not None:
            bm = masks[h // g]
            mask &= bm.repeat_interleave(BLOCK, 0)[:n].repeat_interleave(BLOCK, 1)[:, :N]
        s.masked_fill_(~mask, float('-inf'))
        outs.append(torch.softmax(s, -1) @ v[h // g].float())
    return torch.stack(outs, 1)


# ---------------------------------------------------------------------------
# vLLM glue: dynamic block-sparse path for long prefill chunks in the
# FlashAttention backend. Enabled by SM120_SPARSE_ATTN (default on);
# SM120_SPARSE_TAU, SM120_SPARSE_MIN_KV, SM120_SPARSE_MIN_Q tune it.
# ---------------------------------------------------------------------------
_CONFIG = None
_STATE: dict = {}
FP8_EMULATE = os.environ.get('SM120_SPARSE_FP8_EMULATE', '')      # '' | 'tensor' | 'token' (experiment switch)


def _fp8_round(x, mode, which):
    """Round a [rows, heads, D] bf16 tensor through float8_e4m3fn with amax scaling (sparse_prefill.py:334-348).

    mode 'tensor': one scale per tensor; mode 'token': per (row, head) scales for q/k and per
    (head, channel) scales for v.  Numerics experiment only.
    """
    xf = x.float()
    if mode == 'tensor':
        amax = xf.abs().amax().clamp_min(1e-6)
    elif which == 'v':
        amax = xf.abs().amax(dim=0, keepdim=True).clamp_min(1e-6)
    else:
        amax = xf.abs().amax(dim=2, keepdim=True).clamp_min(1e-6)
    scale = amax / 448.0
    return ((xf / scale).to(torch.float8_e4m3fn).float() * scale).to(x.dtype)


_DEBUG_LEFT = [int(os.environ.get('SM120_SPARSE_DEBUG', '0'))]


def _debug(msg):
    if _DEBUG_LEFT[0] > 0:
        _DEBUG_LEFT[0] -= 1
        print('[sm120-sparse] ' + msg, flush=True)


def config():
    """SM120_SPARSE_* environment variables, with optional defaults from the JSON file named by
    SM120_SPARSE_CONFIG (sparse_prefill.py:358-381)."""
    global _CONFIG
    if _CONFIG is None:
        file_cfg = {}
        path = os.environ.get('SM120_SPARSE_CONFIG')
        if path:
            with open(path) as f:
                file_cfg = json.load(f)

        def pick(env, key, default, cast):
            if env in os.environ:
                return cast(os.environ[env])
            return cast(file_cfg.get(key, default))
        _CONFIG = {
            'enabled': pick('SM120_SPARSE_ATTN', 'enabled', 1, lambda v: str(v) not in ('0', 'false', 'False')),
            'tau': pick('SM120_SPARSE_TAU', 'tau', 0.95, float),
            'min_kv': pick('SM120_SPARSE_MIN_KV', 'min_kv', 8192, int),
            'min_q': pick('SM120_SPARSE_MIN_Q', 'min_q', 1024, int),
            'kernel': pick('SM120_SPARSE_KERNEL', 'kernel', 'sm120fp8', str),
            'fp8_pipeline': pick('SM120_SPARSE_FP8_PIPELINE', 'fp8_pipeline', 'tma', str),
            # new: keep e4m3 K/V per (layer, request) and quantise each chunk's rows once
            'fp8_kv_cache': pick('SM120_SPARSE_FP8_KV_CACHE', 'fp8_kv_cache', 0,
                                 lambda v: str(v) not in ('0', 'false', 'False', '')),
        }
        print('[sm120-sparse] config %r' % (_CONFIG,), flush=True)
    return _CONFIG


def _state(num_heads, num_kv_heads, head_dim, device):
    key = (num_heads, num_kv_heads, head_dim, str(device))
    if key not in _STATE:
        cfg = config()
        _STATE[key] = SparsePrefill(num_heads, num_kv_heads, head_dim, device, tau=cfg['tau'],
                                    min_kv=cfg['min_kv'], min_q=cfg['min_q'], kernel=cfg['kernel'],
                                    fp8_pipeline=cfg['fp8_pipeline'])
    return _STATE[key]


_KMEAN_CACHE: dict = {}
_KMEAN_MAX_ENTRIES = 128


def _cached_block_means(layer_key, first_page, key_chunk, q_start, kv_len, key_all=None):
    """Maintain per-(layer, request) K block means [Hk, NB, D] (fp32), updated from the chunk's keys
    (sparse_prefill.py:398-447).

    A request is identified by its first physical page. An entry is only trusted when it was built
    contiguously by this request (its last chunk ended exactly at q_start); otherwise it is rebuilt
    from the full key history `key_all` [kv_len, Hk, D].  Chunk boundaries unaligned to BLOCK make
    the boundary block's mean use only the rows of the current chunk.
    """
    B = BLOCK
    n, Hk, D = key_chunk.shape
    cache_key = (layer_key, first_page)
    entry = _KMEAN_CACHE.get(cache_key)
    b0, b1 = q_start // B, -(-(q_start + n) // B)
    if entry is None or q_start == 0 or entry['nb'] < b0 or entry.get('last_kv') != q_start:
        if len(_KMEAN_CACHE) >= _KMEAN_MAX_ENTRIES:
            _KMEAN_CACHE.pop(next(iter(_KMEAN_CACHE)))
        cap = max(4096, b1)
        entry = {'km': torch.zeros(Hk, cap, D, dtype=torch.float32, device=key_chunk.device), 'nb': 0, 'last_kv': 0}
        _KMEAN_CACHE[cache_key] = entry
        if q_start > 0:
            if key_all is None:
                raise RuntimeError('stale block-mean cache entry and no key history to rebuild it')
            hist = key_all[:q_start]
            full, rem = q_start // B, q_start % B
            if full:
                ops.block_means(hist[:full * B], 0, B, entry['km'], 0)
            if rem:   # partial block: completed below from `front` rows of the chunk
                ops.block_means(hist[full * B:], full * B, B, entry['km'], 0)
            entry['nb'] = full + (1 if rem else 0)
            if rem:
                key_chunk = torch.cat([hist[full * B:], key_chunk], 0)
                q_start, n = full * B, n + rem
                b0 = full
    if entry['km'].shape[1] < b1:
        grown = torch.zeros(Hk, max(b1, 2 * entry['km'].shape[1]), D, dtype=torch.float32, device=key_chunk.device)
        grown[:, :entry['km'].shape[1]] = entry['km']
        entry['km'] = grown
    if n:
        ops.block_means(key_chunk, q_start, B, entry['km'], 0)
    entry['nb'] = b1
    entry['last_kv'] = kv_len
    return entry['km'][:, :b1]


_SCALE_TENSORS: dict = {}


def _scale_tensor(dev, sq, sk, sv):
    """Device fp32 [1/sq, 1/sk, 1/sv, sq, sk, sv] for one scale triple, kept per (device, triple).

    A host tensor copied from pageable memory makes the copy wait for the whole stream (a device
    sync every chunk); the triple is fixed per request and layer, so it is staged once through
    pinned memory and reused."""
    dev = torch.device(dev)
    if dev.type != 'cuda':                                      # host-side tests with fake ops
        return torch.tensor([1.0 / sq, 1.0 / sk, 1.0 / sv, sq, sk, sv], dtype=torch.float32, device=dev)
    key = (dev.index if dev.index is not None else torch.cuda.current_device(), float(sq), float(sk), float(sv))
    hit = _SCALE_TENSORS.get(key)
    if hit is None:
        if len(_SCALE_TENSORS) >= 4 * _KMEAN_MAX_ENTRIES:
            _SCALE_TENSORS.pop(next(iter(_SCALE_TENSORS)))
        host = torch.tensor([1.0 / sq, 1.0 / sk, 1.0 / sv, sq, sk, sv], dtype=torch.float32).pin_memory()
        hit = (host.to(dev, non_blocking=True), host)          # the pinned source lives as long as the entry
        _SCALE_TENSORS[key] = hit
    return hit[0]


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


def _cached_kv8(layer_key, first_page, k, v, q_start, kv_len, scales, k_row0=0):
    """Per-(layer, request) e4m3 K and V [kv_len, Hk, D] (uint8 views), each row quantised once.

    The FP8 path quantises the whole key/value history with the request's scales on every chunk
    (sparse_prefill.py:230-233); the scales are cached per request, so rows quantised for an earlier
    chunk never change.  An entry contiguous with this chunk (its last row is q_start) and made with
    the same scales only quantises rows q_start..kv_len; otherwise it is rebuilt from k, v (NHD).
    k and v hold sequence rows k_row0 .. k_row0 + len (k_row0 > 0 only for a contiguous entry: a
    rebuild needs every row from 0).  The bytes are the same as re-quantising the history.
    """
    sk, sv = float(scales[1]), float(scales[2])
    key = (layer_key, first_page)
    entry = _KV8_CACHE.get(key)
    Hk, D = k.shape[1], k.shape[2]
    dev = k.device
    if entry is None or q_start == 0 or entry['rows'] != q_start or entry['scales'] != (sk, sv):
        if k_row0:
            raise RuntimeError('stale FP8 KV cache entry and no key/value rows before %d to rebuild it' % k_row0)
        if len(_KV8_CACHE) >= _KMEAN_MAX_ENTRIES:
            _KV8_CACHE.pop(next(iter(_KV8_CACHE)))
        cap = max(kv_len, 8192)
        entry = {'k8': torch.empty(cap, Hk, D, dtype=torch.uint8, device=dev),
                 'v8': torch.empty(cap, Hk, D, dtype=torch.uint8, device=dev), 'rows': 0, 'scales': (sk, sv),
                 'inv': _scale_tensor(dev, scales[0], sk, sv)[1:3]}
        _KV8_CACHE[key] = entry
    lo = entry['rows']
    if entry['k8'].shape[0] < kv_len:
        cap = max(kv_len, 2 * entry['k8'].shape[0])
        for name in ('k8', 'v8'):
            grown = torch.empty(cap, Hk, D, dtype=torch.uint8, device=dev)
            grown[:lo] = entry[name][:lo]
            entry[name] = grown
    _kv8_evict(key)
    if kv_len > lo:
        if k.shape[0] < kv_len - k_row0 or v.shape[0] < kv_len - k_row0 or lo < k_row0:
            raise ValueError('_cached_kv8: k/v do not hold rows %d..%d' % (lo, kv_len))
        ops.quantize(k[lo - k_row0:kv_len - k_row0], entry['inv'][0:1], SA_QUANT_MUL_BF16, entry['k8'][lo:kv_len])
        ops.quantize(v[lo - k_row0:kv_len - k_row0], entry['inv'][1:2], SA_QUANT_MUL_BF16, entry['v8'][lo:kv_len])
    entry['rows'] = kv_len
    return entry['k8'][:kv_len], entry['v8'][:kv_len]


def _fp8_warm(layer_key, first_page, q_start) -> bool:
    """True when the block-mean, scale and FP8 KV caches of this (layer, request) all continue at
    q_start, so a chunk needs none of the key/value history (only its own rows)."""
    key = (layer_key, first_page)
    km, sc, kv = _KMEAN_CACHE.get(key), _SCALE_CACHE.get(key), _KV8_CACHE.get(key)
    return (q_start > 0 and km is not None and km.get('last_kv') == q_start and km['nb'] >= q_start // BLOCK
            and sc is not None and sc['last_kv'] == q_start and kv is not None and kv['rows'] == q_start
            and kv['scales'] == (float(sc['scales'][1]), float(sc['scales'][2])))


_SCALE_CACHE: dict = {}
SCALE_MARGIN = 1.5


def _cached_scales(layer_key, first_page, q, k, v, q_start):
    """Per-(layer, request) e4m3 scales (amax/448 x margin) from the request's first sparse chunk
    (sparse_prefill.py:450-469); one host sync when an entry is (re)built."""
    key = (layer_key, first_page)
    entry = _SCALE_CACHE.get(key)
    if q_start == 0 or entry is None or entry['last_kv'] != q_start:
        if len(_SCALE_CACHE) >= _KMEAN_MAX_ENTRIES:
            _SCALE_CACHE.pop(next(iter(_SCALE_CACHE)))
        amax = torch.cat([ops.absmax(t if t.stride(-1) == 1 else t.contiguous(), per_head=False)
                          for t in (q, k, v)]).clamp_min(1e-6).tolist()
        entry = {'scales': tuple(a * SCALE_MARGIN / 448.0 for a in amax), 'last_kv': 0}
        _SCALE_CACHE[key] = entry
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


@torch.no_grad()
def try_sparse_forward(impl, query, key, key_cache, value_cache, output, attn_metadata) -> bool:
    """Block-sparse attention for the long prefill chunks of this batch; other requests in the
    same batch (short chunks, decode steps) get a per-request dense FlashAttention call
    (sparse_prefill.py:472-535).

    query/key/output: this batch's [num_actual_tokens, ...] tensors; key_cache/value_cache:
    [num_blocks, page, Hk, D]. Returns False (nothing written) when no request qualifies.
    """
    cfg = config()
    if not cfg['enabled']:
        return False
    window = getattr(impl, 'sliding_window', None)
    windowed = window is not None and any(int(w) >= 0 for w in window)   # full attention is (-1, -1)
    if attn_metadata.causal is not True or windowed:
        _debug('fallback: causal=%r window=%r' % (attn_metadata.causal, window))
        return False
    # Host-side checks first: no device-to-host copies during CUDA graph capture and no sync for
    # batches that cannot qualify.
    if attn_metadata.max_query_len < cfg['min_q'] or attn_metadata.max_seq_len < cfg['min_kv']:
        return False
    if torch.cuda.is_current_stream_capturing():
        return False
    qsl, seq_lens, first_pages = _host_metadata(attn_metadata)
    nreq = len(seq_lens)
    eligible = [r for r in range(nreq) if qsl[r + 1] - qsl[r] >= cfg['min_q'] and seq_lens[r] >= cfg['min_kv']]
    if not eligible:
        return False
    _debug('sparse path: %d/%d requests, q_lens=%s kv_lens=%s' % (
        len(eligible), nreq, [qsl[i + 1] - qsl[i] for i in range(nreq)], seq_lens))
    H, D = query.shape[1], query.shape[2]
    Hk = key_cache.shape[2]
    sp = _state(H, Hk, D, query.device)
    page = key_cache.shape[1]
    bt = attn_metadata.block_table
    for r in range(nreq):
        kv_len = seq_lens[r]
        n = qsl[r + 1] - qsl[r]
        q_r = query[qsl[r]:qsl[r + 1]]
        o_r = output[qsl[r]:qsl[r + 1]]
        if r not in eligible:
            _dense_request(impl, q_r, key_cache, value_cache, o_r, bt[r], n, kv_len)
            continue
        npages = -(-kv_len // page)
        q_start = kv_len - n
        if sp.kernel == 'sm120fp8' and cfg['fp8_kv_cache'] and _fp8_warm(id(impl), first_pages[r], q_start):
            # Block means, scales and the e4m3 history are cached: only this chunk's pages are read
            # (the reference gathers the whole history every chunk, sparse_prefill.py:521-522).
            p0 = q_start // page
            pages = bt[r, p0:npages].long()
            kc = key_cache[pages].reshape(-1, Hk, D)
            vc = value_cache[pages].reshape(-1, Hk, D)
            km = _cached_block_means(id(impl), first_pages[r], key[qsl[r]:qsl[r + 1]], q_start, kv_len)
            scales = _cached_scales(id(impl), first_pages[r], q_r, None, None, q_start)
            kv8 = _cached_kv8(id(impl), first_pages[r], kc, vc, q_start, kv_len, scales, k_row0=p0 * page)
            sp.forward_sm120fp8(q_r, None, None, q_start, out=o_r, km=km, scales=scales, kv8=kv8,
                                k_rows=npages * page)
            continue
        pages = bt[r, :npages].long()
        k = key_cache[pages].reshape(npages * page, Hk, D)    # one gather copy, NHD
        v = value_cache[pages].reshape(npages * page, Hk, D)
        km = _cached_block_means(id(impl), first_pages[r], key[qsl[r]:qsl[r + 1]], kv_len - n, kv_len, key_all=k)
        if sp.kernel == 'sm120fp8':
            scales = _cached_scales(id(impl), first_pages[r], q_r, k[:kv_len], v[:kv_len], kv_len - n)
            kv8 = (_cached_kv8(id(impl), first_pages[r], k, v, kv_len - n, kv_len, scales)
                   if cfg['fp8_kv_cache'] else None)
            sp.forward_sm120fp8(q_r, k, v, kv_len - n, out=o_r, km=km, scales=scales, kv8=kv8)
        else:
            sp.forward_sm120(q_r, k, v, kv_len - n, out=o_r, km=km)
    return True


def _dense_request(impl, query, key_cache, value_cache, output, bt_row, n, kv_len):
    """Dense paged FlashAttention for one request of a mixed batch: the backend's own call
    (sparse_prefill.py:538-550)."""
    from vllm.vllm_flash_attn import flash_attn_varlen_func
    dev = query.device
    cu = torch.tensor([0, n], dtype=torch.int32, device=dev)
    su = torch.tensor([kv_len], dtype=torch.int32, device=dev)
    window = getattr(impl, 'sliding_window', None)
    flash_attn_varlen_func(q=query, k=key_cache, v=value_cache, out=output, cu_seqlens_q=cu, max_seqlen_q=n,
                           seqused_k=su, max_seqlen_k=kv_len, softmax_scale=impl.scale, causal=True,
                           alibi_slopes=getattr(impl, 'alibi_slopes', None),
                           window_size=list(window) if window is not None else None,
                           block_table=bt_row.unsqueeze(0), softcap=getattr(impl, 'logits_soft_cap', 0.0),
                           fa_version=getattr(impl, 'vllm_flash_attn_version', 2))
