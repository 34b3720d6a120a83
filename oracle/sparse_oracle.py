"""numpy restatement of the reference's block-sparse prefill algorithm (TEST INFRASTRUCTURE ONLY).

Every function names the reference file:line it follows (paths inside
accion-intelligence/Qwen38-sparse-attn).  Arithmetic mirrors the reference's
PyTorch CPU semantics where they matter for bit-level parity:

* block sums accumulate in float32, row by row, then divide by the valid-row
  count (sparse_prefill.py:60-63, :437-444);
* the tau cumulative sum accumulates in float64 and is rounded to float32
  before the `< tau` test, because ATen's CPU cumsum uses a double accumulator
  for float tensors (sparse_prefill.py:75-76);
* the glue quantises in bf16 arithmetic: e4m3(bf16(f32(x) * f32(1/s)))
  (sparse_prefill.py:230-233);
* torch's float -> float8_e4m3fn cast rounds to nearest-even and is
  non-saturating: |x| in (448, 464] -> 448, |x| > 464 -> NaN.

Never imported by the product package; see `oracle/__init__.py`.
"""
from __future__ import annotations

import math

import numpy as np

__all__ = [
    'bf16_round', 'bf16_bits', 'bf16_from_bits', 'e4m3_encode', 'e4m3_decode', 'e4m3_round',
    'VT_KEY_PERM', 'vt_key_index', 'permute_vt_keys',
    'block_means', 'q_block_means', 'KMeanCacheOracle', 'ScaleCacheOracle',
    'select_masks', 'pair_union', 'masks_to_lists', 'compare_masks',
    'quantize_glue', 'quantize_per_tensor', 'attention_ref', 'attention_ref_threaded', 'attention_fp8_kernel_model',
    'causal_blocks', 'causal_flops',
]

F32 = np.float32


# ---------------------------------------------------------------------------------------------
# Number formats
# ---------------------------------------------------------------------------------------------
def bf16_bits(x) -> np.ndarray:
    """float32 -> bf16 bit patterns (uint16), round to nearest even; NaN stays NaN (the bf16 arithmetic of
    `q * (1.0 / sq)` before the e4m3 cast, sparse_prefill.py:230-233)."""
    b = np.ascontiguousarray(x, dtype=F32).view(np.uint32).astype(np.uint64)
    nan = np.isnan(np.asarray(x, dtype=F32))
    r = ((b + 0x7FFF + ((b >> 16) & 1)) >> 16).astype(np.uint16)
    r[nan] = 0x7FC0
    return r


def bf16_from_bits(u) -> np.ndarray:
    return (np.asarray(u, dtype=np.uint16).astype(np.uint32) << 16).view(F32)


def bf16_round(x) -> np.ndarray:
    return bf16_from_bits(bf16_bits(x))


def e4m3_round(x) -> np.ndarray:
    """Values of float8_e4m3fn(x) with torch's cast semantics (RNE, |x| > 464 -> NaN), the cast of
    sparse_prefill.py:230-233 and kernels/kai_fa_fp8.py:327."""
    x = np.asarray(x, dtype=np.float64)
    a = np.abs(x)
    out = np.empty_like(a)
    sub = a < 2.0 ** -6
    out[sub] = np.rint(a[sub] * 2.0 ** 9) * 2.0 ** -9                  # subnormals: step 2^-9
    nz = ~sub
    if np.any(nz):
        m, e = np.frexp(a[nz])                                        # a = m * 2^e, m in [0.5, 1)
        q = np.rint(m * 16.0) / 16.0                                  # 1 + 3 mantissa bits
        out[nz] = np.ldexp(q, e)
    out = np.where(a > 464.0, np.nan, np.minimum(out, 448.0))
    out = np.where(np.isnan(a), np.nan, out)
    return (np.sign(x) * out).astype(F32)


def e4m3_encode(x) -> np.ndarray:
    """float -> e4m3fn bit patterns (uint8), same rounding as `e4m3_round`; NaN -> 0x7F | sign."""
    x = np.asarray(x, dtype=np.float64)
    v = e4m3_round(x).astype(np.float64)
    sign = np.signbit(np.where(np.isnan(v), x, v)).astype(np.uint8) << 7     # NaN keeps the sign of x
    a = np.abs(v)
    bits = np.zeros(a.shape, dtype=np.uint8)
    nan = np.isnan(a)
    sub = (a < 2.0 ** -6) & ~nan
    bits[sub] = np.rint(a[sub] * 2.0 ** 9).astype(np.uint8)
    nrm = ~sub & ~nan
    if np.any(nrm):
        m, e = np.frexp(a[nrm])                                       # a = (2m) * 2^(e-1)
        exp_field = (e - 1 + 7).astype(np.int64)
        man = np.rint((2.0 * m - 1.0) * 8.0).astype(np.int64)
        bits[nrm] = ((exp_field << 3) | man).astype(np.uint8)
    bits[nan] = 0x7F
    return bits | sign


def e4m3_decode(u) -> np.ndarray:
    u = np.asarray(u, dtype=np.uint8)
    s = np.where(u & 0x80, -1.0, 1.0)
    e = (u >> 3) & 0xF
    m = (u & 7).astype(np.float64)
    val = np.where(e == 0, m * 2.0 ** -9, (1.0 + m / 8.0) * np.exp2(e.astype(np.float64) - 7))
    val = np.where((u & 0x7F) == 0x7F, np.nan, val)
    return (s * val).astype(F32)


# Key order inside each 32-key block of the reference's permuted V^T (kai_fa_fp8.py:303-306).
VT_KEY_PERM = [16 * (s >> 4) + 8 * ((s & 3) >> 1) + 2 * ((s >> 2) & 3) + ((s & 3) & 1) for s in range(32)]


def vt_key_index(kv_len: int) -> np.ndarray:
    """kai_fa_fp8.py:309-318: gather index permuting the key axis of V^T; kv_len % 32 == 0."""
    base = np.arange(0, kv_len, 32, dtype=np.int64)
    return (base[:, None] + np.asarray(VT_KEY_PERM, dtype=np.int64)[None, :]).reshape(-1)


def permute_vt_keys(vt: np.ndarray) -> np.ndarray:
    """kai_fa_fp8.py:321-322: vT [Hk, D, kv] -> keys permuted per 32-key block."""
    return np.take(vt, vt_key_index(vt.shape[2]), axis=2)


# ---------------------------------------------------------------------------------------------
# Block summaries (kernel a)
# ---------------------------------------------------------------------------------------------
def _seq_block_sum(x: np.ndarray, rows: list) -> np.ndarray:
    acc = np.zeros(x.shape[1:], dtype=F32)
    for r in rows:
        acc += x[r]
    return acc


def block_means(x: np.ndarray, pos0: int, block: int):
    """Means of the rows of x [n, heads, D] (absolute positions pos0..pos0+n-1) per `block`-row block.

    Block b covers positions [b*block, (b+1)*block); only rows present in x count (a partial
    boundary block is the mean of the rows this chunk holds - the quirk of
    sparse_prefill.py:437-444).  Returns (b0, means [heads, b1-b0, D] float32).
    """
    x = np.asarray(x, dtype=F32)
    n = x.shape[0]
    b0 = pos0 // block
    b1 = -(-(pos0 + n) // block)
    out = np.zeros((x.shape[1], b1 - b0, x.shape[2]), dtype=F32)
    for b in range(b0, b1):
        lo = max(pos0, b * block) - pos0
        hi = min(pos0 + n, (b + 1) * block) - pos0
        s = _seq_block_sum(x, range(lo, hi))
        out[:, b - b0] = s / F32(max(hi - lo, 1))
    return b0, out


def q_block_means(q: np.ndarray, q_start: int, block: int) -> np.ndarray:
    """Pooled query blocks of `block_masks` (sparse_prefill.py:58-63) for q [n, H, D] at q_start.

    The reference pads q with `front = q_start % block` zero rows and passes valid=(front, n);
    block m covers aligned positions (q_start - front) + [m*block, (m+1)*block).  Returns
    qm [MB, H, D] with MB = ceil((front + n) / block).
    """
    _, means = block_means(q, q_start, block)
    return np.ascontiguousarray(means.transpose(1, 0, 2))


class KMeanCacheOracle:
    """`_cached_block_means` (sparse_prefill.py:394-447) with its dict bookkeeping, in numpy."""

    def __init__(self, block: int, max_entries: int = 128):
        self.block = block
        self.max_entries = max_entries
        self.entries: dict = {}

    def update(self, layer_key, first_page, key_chunk, q_start, kv_len, key_all=None):
        B = self.block
        key_chunk = np.asarray(key_chunk, dtype=F32)
        n, Hk, D = key_chunk.shape
        ck = (layer_key, first_page)
        entry = self.entries.get(ck)
        b0, b1 = q_start // B, -(-(q_start + n) // B)
        if entry is None or q_start == 0 or entry['nb'] < b0 or entry.get('last_kv') != q_start:
            if len(self.entries) >= self.max_entries:
                self.entries.pop(next(iter(self.entries)))
            cap = max(4096, b1)
            entry = {'km': np.zeros((Hk, cap, D), dtype=F32), 'nb': 0, 'last_kv': 0}
            self.entries[ck] = entry
            if q_start > 0:
                if key_all is None:
                    raise RuntimeError('stale block-mean cache entry and no key history to rebuild it')
                hist = np.asarray(key_all, dtype=F32)[:q_start]
                full, rem = q_start // B, q_start % B
                if full:
                    _, m = block_means(hist[:full * B], 0, B)
                    entry['km'][:, :full] = m
                if rem:
                    entry['km'][:, full] = _seq_block_sum(hist, range(full * B, q_start)) / F32(rem)
                entry['nb'] = full + (1 if rem else 0)
                if rem:
                    key_chunk = np.concatenate([hist[full * B:], key_chunk], 0)
                    q_start, n = full * B, n + rem
                    b0 = full
        if entry['km'].shape[1] < b1:
            grown = np.zeros((Hk, max(b1, 2 * entry['km'].shape[1]), D), dtype=F32)
            grown[:, :entry['km'].shape[1]] = entry['km']
            entry['km'] = grown
        _, m = block_means(key_chunk, q_start, B)
        entry['km'][:, b0:b1] = m
        entry['nb'] = b1
        entry['last_kv'] = kv_len
        return entry['km'][:, :b1]


class ScaleCacheOracle:
    """`_cached_scales` (sparse_prefill.py:450-469): amax * 1.5 / 448 from the first sparse chunk."""

    MARGIN = 1.5

    def __init__(self, max_entries: int = 128):
        self.max_entries = max_entries
        self.entries: dict = {}

    def update(self, layer_key, first_page, q, k, v, q_start):
        key = (layer_key, first_page)
        entry = self.entries.get(key)
        if q_start == 0 or entry is None or entry['last_kv'] != q_start:
            if len(self.entries) >= self.max_entries:
                self.entries.pop(next(iter(self.entries)))
            amax = [max(float(np.abs(np.asarray(t, dtype=F32)).max()), float(F32(1e-6))) for t in (q, k, v)]
            entry = {'scales': tuple(a * self.MARGIN / 448.0 for a in amax), 'last_kv': 0}
            self.entries[key] = entry
        entry['last_kv'] = q_start + q.shape[0]
        return entry['scales']


# ---------------------------------------------------------------------------------------------
# Selection (kernel b)
# ---------------------------------------------------------------------------------------------
def select_masks(qm, km, qs: int, block: int, num_heads: int, num_kv_heads: int, tau: float,
                 union: bool = False, nb_total: int | None = None, return_aux: bool = False):
    """`SparsePrefill.block_masks` (sparse_prefill.py:41-85) given pooled q and cached km.

    qm [MB, H, D] float32, km [Hk, NBk, D] float32, qs = aligned absolute start of q block 0.
    nb_total: number of key blocks scored (the FP8 driver zero-pads km up to it,
    sparse_prefill.py:219-221); defaults to NBk.  Returns bool masks [H, MB, NB] (union=False) or
    [Hk, MB, NB]; with return_aux also the float32 probs [Hk, MB, g, NB], the stable descending order,
    the float32 cumsum and `keep`.
    """
    qm = np.asarray(qm, dtype=F32)
    km = np.asarray(km, dtype=F32)
    MB, H, D = qm.shape
    Hk = num_kv_heads
    g = num_heads // num_kv_heads
    NBk = km.shape[1]
    NB = NBk if nb_total is None else nb_total
    kmf = np.zeros((Hk, NB, D), dtype=F32)
    kmf[:, :min(NB, NBk)] = km[:, :min(NB, NBk)]
    gi = qs // block + np.arange(MB)
    j = np.arange(NB)
    future = j[None, :] > gi[:, None]                                          # [MB, NB]
    qg = qm.reshape(MB, Hk, g, D)
    logits = np.einsum('mhgd,hnd->hmgn', qg, kmf).astype(F32) * F32(D ** -0.5)
    logits = np.where(future[None, :, None, :], F32(-np.inf), logits).astype(F32)
    mx = logits.max(-1, keepdims=True)
    e = np.exp(logits - mx).astype(F32)
    probs = (e / e.sum(-1, keepdims=True, dtype=F32)).astype(F32)
    order = np.argsort(-probs, axis=-1, kind='stable')                         # descending, ties by index
    srt = np.take_along_axis(probs, order, -1)
    csum = np.cumsum(srt.astype(np.float64), axis=-1).astype(F32)
    keep = (csum < F32(tau)).sum(-1, keepdims=True) + 1
    sel_sorted = j[None, None, None, :] < keep
    sel = np.zeros_like(sel_sorted)
    np.put_along_axis(sel, order, sel_sorted, -1)
    if union:
        masks = sel.any(2)
    else:
        masks = sel.transpose(0, 2, 1, 3).reshape(num_heads, MB, NB)
    masks = masks.copy()
    masks[:, np.arange(MB), np.minimum(gi, NB - 1)] |= (gi < NB)[None, :]
    masks[:, :, 0] = True
    masks &= ~future[None]
    if return_aux:
        return masks, {'probs': probs, 'order': order, 'csum': csum, 'keep': keep[..., 0], 'gi': gi}
    return masks


def pair_union(masks: np.ndarray) -> np.ndarray:
    """128-row masks from 64-row masks (sparse_prefill.py:223; tests/test_fa_bf16.py:50-56)."""
    H, MB, NB = masks.shape
    if MB % 2:
        masks = np.concatenate([masks, np.zeros((H, 1, NB), dtype=bool)], 1)
    return masks.reshape(H, -1, 2, NB).any(2)


def masks_to_lists(masks: np.ndarray):
    """counts [R] int32 and lists [R, NB] int32 (selected blocks first, ascending; sparse_prefill.py:224-225)."""
    R = masks.shape[0] * masks.shape[1]
    m = masks.reshape(R, -1)
    counts = m.sum(1).astype(np.int32)
    lists = np.argsort(~m, axis=1, kind='stable').astype(np.int32)
    return counts, lists


def compare_masks(test: np.ndarray, ref: np.ndarray, aux: dict, tau: float, num_kv_heads: int,
                  pair: bool = False, tol: float = 1e-4, tie_rtol: float = 1e-5, report: dict | None = None):
    """Mask parity with the tau-boundary exemption.

    test/ref: per-query-head masks [H, MB', NB] (MB' = MB/2 when `pair`).  A mismatching block is
    exempt when, in the oracle's sorted order of a contributing (head, q-block) row, its cumulative
    mass (inclusive or exclusive) lies within `tol` of tau (the exemption the parity bar states), or
    its probability ties (relative `tie_rtol`) the probability at the keep boundary - torch.sort is
    not stable, so the reference does not define which of equal-probability blocks it keeps.
    Returns (mismatches, unexplained).  When `report` is a dict it receives how many mismatches each
    exemption absorbed: 'tau_band' (checked first) and 'tie' (only blocks outside the tau band), plus
    'mismatches' and 'unexplained' counts, so that the second exemption cannot hide a real error
    unnoticed.
    """
    probs, order, keep = aux['probs'], aux['order'], aux['keep']
    Hk, MB, g, NB = probs.shape
    csum64 = np.cumsum(np.take_along_axis(probs, order, -1).astype(np.float64), axis=-1)
    pos = np.empty_like(order)
    np.put_along_axis(pos, order, np.arange(NB)[None, None, None, :].repeat(Hk, 0).repeat(MB, 1).repeat(g, 2), -1)
    bad = np.argwhere(test != ref)
    unexplained = []
    n_band = n_tie = 0
    for h, mm, jj in bad:
        hk, i = divmod(int(h), g)
        rows = [m for m in ((2 * mm, 2 * mm + 1) if pair else (mm,)) if m < MB]
        band = tie = False
        for m in rows:
            p = pos[hk, m, i, jj]
            inc = csum64[hk, m, i, p]
            exc = inc - float(probs[hk, m, i, jj])
            band = band or abs(inc - tau) < tol or abs(exc - tau) < tol
        if not band:
            for m in rows:
                kb = int(keep[hk, m, i])
                edge = [float(probs[hk, m, i, order[hk, m, i, t]]) for t in (kb - 1, kb) if 0 <= t < NB]
                pj = float(probs[hk, m, i, jj])
                tie = tie or any(abs(pj - e) <= tie_rtol * max(e, 1e-30) for e in edge)
        n_band += band
        n_tie += tie
        if not (band or tie):
            unexplained.append((int(h), int(mm), int(jj)))
    if report is not None:
        report.update({'mismatches': int(len(bad)), 'tau_band': int(n_band), 'tie': int(n_tie),
                       'unexplained': len(unexplained)})
    return len(bad), unexplained


# ---------------------------------------------------------------------------------------------
# Quantisation and attention (kernel c)
# ---------------------------------------------------------------------------------------------
def quantize_glue(x_bf16_vals: np.ndarray, inv_scale) -> np.ndarray:
    """sparse_prefill.py:230-233: e4m3(bf16(f32(x) * f32(1/s))) -> uint8 bit patterns.

    inv_scale: scalar or per-head array broadcast over axis 1 of x [rows, heads, D].
    """
    x = np.asarray(x_bf16_vals, dtype=F32)
    inv = np.asarray(inv_scale, dtype=F32)
    if inv.ndim == 1:
        inv = inv[None, :, None]
    return e4m3_encode(bf16_round((x * inv).astype(F32)))


def quantize_per_tensor(x_vals: np.ndarray):
    """kai_fa_fp8.py:325-328 `quantize_e4m3`: amax/448 per tensor, fp32 division. Returns (u8, scale)."""
    x = np.asarray(x_vals, dtype=F32)
    amax = max(float(np.abs(x).max()), float(F32(1e-6)))
    scale = float(F32(F32(amax) / F32(448.0)))
    return e4m3_encode((x / F32(scale)).astype(F32)), scale


def _expand_block_mask(masks_h: np.ndarray, n: int, N: int, q_block: int, kv_block: int, q_front: int):
    rows = (np.arange(n) + q_front) // q_block
    cols = np.arange(N) // kv_block
    MBr, NBc = masks_h.shape
    m = np.zeros((n, N), dtype=bool)
    rv = rows < MBr
    cv = cols < NBc
    m[np.ix_(rv, cv)] = masks_h[np.ix_(rows[rv], cols[cv])]
    return m


def attention_ref(q, k, v, q_pos0: int, masks=None, q_block: int = 64, kv_block: int = 64, q_front: int = 0,
                  scale: float | None = None):
    """fp32 masked causal attention (tests/test_fa_bf16.py:17-33; sparse_prefill.py:262-279).

    q [n, H, D] at absolute positions q_pos0.., k/v [N, Hk, D] (NHD), per-query-head masks
    [H, MBr, NBc]: row i uses mask row (i + q_front) // q_block, key j uses block j // kv_block.
    """
    q = np.asarray(q, dtype=F32)
    k = np.asarray(k, dtype=F32)
    v = np.asarray(v, dtype=F32)
    n, H, D = q.shape
    N, Hk, _ = k.shape
    g = H // Hk
    sc = F32(D ** -0.5 if scale is None else scale)
    allowed = np.arange(N)[None, :] <= (q_pos0 + np.arange(n))[:, None]
    out = np.empty((n, H, D), dtype=F32)
    for h in range(H):
        s = (q[:, h] @ k[:, h // g].T).astype(F32) * sc
        m = allowed if masks is None else allowed & _expand_block_mask(masks[h], n, N, q_block, kv_block, q_front)
        s = np.where(m, s, F32(-np.inf))
        mx = s.max(-1, keepdims=True)
        e = np.exp(s - mx)
        p = e / e.sum(-1, keepdims=True)
        out[:, h] = (p @ v[:, h // g]).astype(F32)
    return out


def attention_ref_threaded(q, k, v, q_pos0: int, masks=None, q_block: int = 64, kv_block: int = 64, q_front: int = 0,
                           scale: float | None = None):
    """attention_ref with the same fp32 arithmetic run through PyTorch on the host cores (all intra-op
    threads), as the reference's own CPU path runs (`reference()`, sparse_prefill.py:262-279: per
    head, fp32 scores, masked fill, softmax, P.V).  The CPU baseline of the benchmark times this so
    that the restatement runs at the reference's own CPU speed (numpy's elementwise passes are single
    threaded).  Same arguments and result as attention_ref."""
    import torch
    qt = torch.from_numpy(np.ascontiguousarray(q, dtype=F32))
    kt = torch.from_numpy(np.ascontiguousarray(k, dtype=F32))
    vt = torch.from_numpy(np.ascontiguousarray(v, dtype=F32))
    n, H, D = qt.shape
    N, Hk, _ = kt.shape
    g = H // Hk
    sc = float(F32(D ** -0.5 if scale is None else scale))
    allowed = torch.arange(N)[None, :] <= (q_pos0 + torch.arange(n))[:, None]
    rows = (torch.arange(n) + q_front) // q_block                 # mask row of each query row
    out = torch.empty((n, H, D), dtype=torch.float32)
    for h in range(H):
        s_ = (qt[:, h] @ kt[:, h // g].T) * sc
        if masks is None:
            m = allowed
        else:
            mh = torch.from_numpy(np.ascontiguousarray(masks[h], dtype=bool))[rows]          # [n, NBc]
            nbc = mh.shape[1]
            full = mh[:, :, None].expand(n, nbc, kv_block).reshape(n, nbc * kv_block)     # key j -> j // kv_block
            if full.shape[1] < N:
                full = torch.cat([full, full.new_zeros(n, N - full.shape[1])], 1)
            m = allowed & full[:, :N]
        s_.masked_fill_(~m, float('-inf'))
        out[:, h] = torch.softmax(s_, -1) @ vt[:, h // g]
    return out.numpy()


def attention_fp8_kernel_model(q8, k8, v8, sq, sk, sv, q_pos0: int, counts=None, lists=None,
                               q_block: int = 128, kv_block: int = 64, q_front: int = 0, tile: int = 128,
                               key_tile: int = 64, group: int = 1, partner_of=None, splits: int = 1,
                               split_min_steps: int = 0, split_units=None):
    """Numerical model of the block-sparse FP8 forward (kai_fa_fp8.py:248-292, kai_fa_fp8_tma.py:256-272).

    Walks each (head, 128-row tile)'s block list from the last entry to the first in `key_tile`-key
    steps (a 128-key block is split, upper half first); every `group` consecutive steps form one key
    tile of the online softmax (the CUDA FP8 kernel takes one 64-key step per tile; a kernel taking
    two steps per tile, not necessarily adjacent keys, is modelled by group=2).  Online softmax in
    the exp2 domain,
    P scaled by 448 and rounded to e4m3 before the PV product, the row sum over unrounded P, and
    `O * (sv / 448) / rowsum` (0 for an empty row).  The order and granularity of the walk set where
    P is rounded, so they follow the CUDA kernel.  `partner_of(h, t)` -> (h2, t2) or None models a
    kernel that walks two query tiles together: the steps are formed from the union of both tiles'
    64-key blocks (descending, `group` per step), and each tile takes the keys of its own blocks in
    every step that holds any (the partner's blocks are masked out for it).  `splits` > 1 models the
    split walks of sa_attn_fwd_fp8_split: a walk of a split unit (`split_units(h, t)` true, all units
    when it is None) of at least split_min_steps steps is cut into
    `splits` contiguous step ranges, each run from a fresh online-softmax state, and the ranges are
    combined with weights 2^(m_s - max m) on their unnormalised outputs and row sums.
    Inputs are e4m3 bit patterns q8 [n, H, D],
    k8 [N, Hk, D], v8 [N, Hk, D]; per-head scale arrays or scalars.  Dense when counts is None.
    Returns fp32 [n, H, D].
    """
    qv, kv, vv = (e4m3_decode(t).astype(np.float64) for t in (q8, k8, v8))
    n, H, D = qv.shape
    N, Hk, _ = kv.shape
    g = H // Hk
    sq = np.broadcast_to(np.asarray(sq, dtype=np.float64), (H,))
    sk = np.broadcast_to(np.asarray(sk, dtype=np.float64), (Hk,))
    sv = np.broadcast_to(np.asarray(sv, dtype=np.float64), (Hk,))
    n_tiles = -(-(q_front + n) // tile)
    qpos0 = q_pos0 - q_front                                 # absolute position of virtual row 0
    out = np.zeros((n, H, D), dtype=F32)
    log2e = 1.4426950408889634
    for h in range(H):
        hk = h // g
        c = float(F32(D ** -0.5 * sq[h] * sk[hk] * log2e))
        for t in range(n_tiles):
            r0 = t * tile - q_front
            rows = np.arange(r0, r0 + tile)
            valid_rows = (rows >= 0) & (rows < n)
            qpos = qpos0 + t * tile + np.arange(tile)
            qt = np.zeros((tile, D))
            qt[valid_rows] = qv[rows[valid_rows], h]
            def own_starts(hh, tt):
                if counts is None:
                    nkeys = min(qpos0 + (tt + 1) * tile, N)
                    return list(range(0, nkeys, key_tile))[::-1]
                r = hh * (-(-(q_front + n) // q_block)) + (tt * tile) // q_block
                out_s = []
                for b in [int(x) for x in lists[r, :counts[r]]][::-1]:
                    out_s += list(range(b * kv_block, (b + 1) * kv_block, key_tile))[::-1]
                return out_s
            starts = own_starts(h, t)
            mate = partner_of(h, t) if partner_of is not None else None
            if mate is None:
                steps = [starts[gi:gi + group] for gi in range(0, len(starts), group)]
            else:
                union = sorted(set(starts) | set(own_starts(*mate)), reverse=True)
                mine = set(starts)
                steps = [[k0 for k0 in union[gi:gi + group] if k0 in mine] for gi in range(0, len(union), group)]
                steps = [st for st in steps if st]
            def run(range_steps):
                m = np.full(tile, -np.inf)
                l = np.zeros(tile)
                o = np.zeros((tile, D))
                for step in range_steps:
                    keys = np.concatenate([np.arange(k0, k0 + key_tile) for k0 in step])
                    kk = np.zeros((len(keys), D))
                    vk = np.zeros((len(keys), D))
                    inr = keys < N
                    kk[inr] = kv[keys[inr], hk]
                    vk[inr] = vv[keys[inr], hk]
                    sc = (qt @ kk.T) * c
                    sc = np.where(keys[None, :] <= qpos[:, None], sc, -np.inf)
                    mn = np.maximum(m, sc.max(1))
                    ms = np.where(np.isneginf(mn), 0.0, mn)
                    alpha = np.where(np.isneginf(m), 0.0, np.exp2(m - ms))
                    p = np.exp2(sc - ms[:, None])
                    l = l * alpha + p.sum(1)
                    p8 = e4m3_round(p * 448.0).astype(np.float64)
                    o = o * alpha[:, None] + p8 @ vk
                    m = mn
                return m, l, o
            if splits > 1 and len(steps) >= split_min_steps and (split_units is None or split_units(h, t)):
                parts = [run(steps[len(steps) * s_ // splits:len(steps) * (s_ + 1) // splits]) for s_ in range(splits)]
                with np.errstate(invalid='ignore'):
                    M = np.max([pm for pm, _, _ in parts], axis=0)
                    ws = [np.where(pl > 0, np.exp2(pm - np.where(np.isneginf(M), 0.0, M)), 0.0) for pm, pl, _ in parts]
                l = sum(w * pl for w, (_, pl, _) in zip(ws, parts))
                o = sum(w[:, None] * np.where(pl[:, None] > 0, po, 0.0) for w, (_, pl, po) in zip(ws, parts))
            else:
                _, l, o = run(steps)
            bad = (l == 0) | np.isnan(l)
            inv = np.where(bad, 0.0, sv[hk] / 448.0 / np.where(bad, 1.0, l))
            res = o * inv[:, None]
            out[rows[valid_rows], h] = res[valid_rows]
    return out


def causal_blocks(qs: int, MB: int, block: int) -> int:
    """Number of causal (head-independent) blocks for MB query blocks starting at aligned qs: the
    per-head term of the `blocks_total` statistic (sparse_prefill.py:182, :242)."""
    return int((qs // block) * MB + MB * (MB + 1) // 2)


def causal_flops(num_heads: int, head_dim: int, n: int, kv: int) -> float:
    """Dense causal attention FLOPs of the reference's benchmarks (tests/test_fa_bf16.py:105)."""
    return 4.0 * num_heads * head_dim * n * (kv - n + (n + 1) / 2)


def _selftest():  # pragma: no cover - quick manual check
    x = np.array([440., 448., 449., 464., 465., 2 ** -10, 0.75 * 2 ** -9, -3.3], dtype=F32)
    print(e4m3_round(x), e4m3_decode(e4m3_encode(x)))
    print(math.isclose(float(bf16_round(np.array([1.00390625], F32))[0]), 1.0))


if __name__ == '__main__':  # pragma: no cover
    _selftest()
