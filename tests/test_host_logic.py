"""Host-side logic of the drop-in `sm120_attn.sparse_prefill` on CPU: knobs, eligibility gates, and the
bookkeeping of the block-mean and scale caches (sparse_prefill.py:358-469, :472-499).

The CUDA entry points are replaced, inside these tests only, by oracle-backed fakes that write into CPU
tensors; the product itself has no CPU path.
"""
from __future__ import annotations

import json
import types

import numpy as np
import pytest
import torch

import oracle as O
import synth


@pytest.fixture
def ksp(monkeypatch):
    import sm120_attn.sparse_prefill as m
    from sm120_attn import ops

    def fake_block_means(x, pos0, block, out, out_block0, q8=None, inv_scale=None, fixed_divisor=0):
        b0, means = O.block_means(x.float().numpy(), pos0, block)
        if fixed_divisor:
            n = x.shape[0]
            for i in range(means.shape[1]):
                b = b0 + i
                rows = min(pos0 + n, (b + 1) * block) - max(pos0, b * block)
                means[:, i] *= np.float32(rows) / np.float32(fixed_divisor)
        out[:, b0 - out_block0:b0 - out_block0 + means.shape[1]] = torch.from_numpy(means)

    def fake_absmax(x, per_head, out=None):
        a = x.float().abs()
        return a.amax(dim=(0, 2)) if per_head else a.amax().reshape(1)

    def gathered(cache, table):
        return cache[table.long()].reshape(-1, cache.shape[2], cache.shape[3])

    def fake_block_means_paged(cache, table, pos0, n, block, out, out_block0):
        fake_block_means(gathered(cache, table)[pos0:pos0 + n], pos0, block, out, out_block0)

    def fake_absmax_paged(cache, table, row0, rows, per_head, out=None):
        return fake_absmax(gathered(cache, table)[row0:row0 + rows], per_head)

    monkeypatch.setattr(ops, 'block_means', fake_block_means)
    monkeypatch.setattr(ops, 'absmax', fake_absmax)
    monkeypatch.setattr(ops, 'block_means_paged', fake_block_means_paged)
    monkeypatch.setattr(ops, 'absmax_paged', fake_absmax_paged)
    m._KMEAN_CACHE.clear()
    m._SCALE_CACHE.clear()
    m._KV8_CACHE.clear()
    old_block = m.BLOCK
    yield m
    m.BLOCK = old_block
    m._KMEAN_CACHE.clear()
    m._SCALE_CACHE.clear()
    m._KV8_CACHE.clear()


def test_config_env_and_json(monkeypatch, tmp_path, capsys):
    import sm120_attn.sparse_prefill as m
    cfg = tmp_path / 'cfg.json'
    cfg.write_text(json.dumps({'tau': 0.9, 'min_kv': 4096, 'kernel': 'sm120', 'enabled': 'false'}))
    monkeypatch.setenv('SM120_SPARSE_CONFIG', str(cfg))
    monkeypatch.setenv('SM120_SPARSE_TAU', '0.85')
    for k in ('SM120_SPARSE_ATTN', 'SM120_SPARSE_MIN_KV', 'SM120_SPARSE_MIN_Q', 'SM120_SPARSE_KERNEL',
              'SM120_SPARSE_FP8_PIPELINE'):
        monkeypatch.delenv(k, raising=False)
    monkeypatch.setattr(m, '_CONFIG', None)
    c = m.config()
    assert c == {'enabled': False, 'tau': 0.85, 'min_kv': 4096, 'min_q': 1024, 'kernel': 'sm120', 'fp8_pipeline': 'tma',
                 'fp8_kv_cache': False, 'fp8_scales': 'tensor'}
    assert 'config' in capsys.readouterr().out
    assert m.config() is c                                           # cached
    monkeypatch.setattr(m, '_CONFIG', None)
    monkeypatch.delenv('SM120_SPARSE_CONFIG')
    monkeypatch.delenv('SM120_SPARSE_TAU')
    c = m.config()
    assert c['enabled'] is True and c['tau'] == 0.95 and c['min_kv'] == 8192 and c['kernel'] == 'sm120fp8'
    monkeypatch.setattr(m, '_CONFIG', None)


def test_kernel_knob_validation():
    import sm120_attn.sparse_prefill as m
    assert m.SparsePrefill(8, 2, 128, 'cpu', kernel='fp8').kernel == 'sm120fp8'
    assert m.SparsePrefill(8, 2, 128, 'cpu', kernel='bf16').kernel == 'sm120'
    with pytest.raises(ValueError):
        m.SparsePrefill(8, 2, 128, 'cpu', kernel='flashinfer')
    with pytest.raises(ValueError):
        m.SparsePrefill(8, 2, 128, 'cpu', fp8_pipeline='other')
    sp = m.SparsePrefill(8, 2, 128, 'cpu', min_kv=100, min_q=10)
    assert sp.eligible(10, 100) and not sp.eligible(9, 100) and not sp.eligible(10, 99)
    assert sp.kept_fraction() is None
    assert sp.stats == {'calls': 0, 'blocks_total': 0, 'blocks_kept': 0, 'plan_ms': 0.0, 'run_ms': 0.0, 'select_ms': 0.0}


def _meta(qlens, kvlens, page=16, causal=True):
    qsl = np.concatenate([[0], np.cumsum(qlens)]).astype(np.int32)
    npages = [-(-k // page) for k in kvlens]
    bt = torch.zeros(len(qlens), max(npages), dtype=torch.int32)
    nxt = 0
    for r, p in enumerate(npages):
        bt[r, :p] = torch.arange(nxt, nxt + p)
        nxt += p
    return types.SimpleNamespace(causal=causal, max_query_len=int(max(qlens)), max_seq_len=int(max(kvlens)),
                                 query_start_loc=torch.from_numpy(qsl), seq_lens=torch.tensor(kvlens, dtype=torch.int32),
                                 block_table=bt)


@pytest.mark.parametrize('case', ['disabled', 'noncausal', 'window', 'short_q', 'short_kv', 'no_eligible'])
def test_try_sparse_forward_gates(monkeypatch, case):
    import sm120_attn.sparse_prefill as m
    monkeypatch.setattr(m, '_CONFIG', {'enabled': case != 'disabled', 'tau': 0.95, 'min_kv': 8192, 'min_q': 1024,
                                       'kernel': 'sm120fp8', 'fp8_pipeline': 'tma', 'fp8_kv_cache': False})
    monkeypatch.setattr(torch.cuda, 'is_current_stream_capturing', lambda: False)
    impl = types.SimpleNamespace(sliding_window=(-1, -1) if case != 'window' else (128, 0), scale=0.1)
    if case == 'short_q':
        meta = _meta([512], [16384])
    elif case == 'short_kv':
        meta = _meta([2048], [4096])
    elif case == 'no_eligible':
        meta = _meta([2048, 1], [4096, 20000])           # max lengths pass, no single request qualifies
    else:
        meta = _meta([2048], [16384], causal=(case != 'noncausal'))
    q = torch.zeros(int(meta.query_start_loc[-1]), 8, 128)
    assert m.try_sparse_forward(impl, q, q, None, None, q, meta) is False


def test_cached_block_means_bookkeeping(ksp):
    B = 64
    ksp.BLOCK = B
    _, k, _, _ = synth.make_qkv(16, 3000, 8, 2, 128, block=B, seed=3, with_v=False)
    kc = O.KMeanCacheOracle(B)
    for q_start, n in ((0, 1000), (1000, 1500), (2500, 500)):
        km = ksp._cached_block_means('L', 5, k[q_start:q_start + n], q_start, q_start + n)
        ref = kc.update('L', 5, k[q_start:q_start + n].float().numpy(), q_start, q_start + n)
        np.testing.assert_allclose(km.numpy(), ref, rtol=1e-6, atol=1e-7)
        assert ksp._KMEAN_CACHE[('L', 5)]['last_kv'] == q_start + n
    # discontinuity without history -> RuntimeError; with history -> rebuild
    with pytest.raises(RuntimeError):
        ksp._cached_block_means('L', 5, k[100:200], 100, 200)
    km = ksp._cached_block_means('L', 6, k[1000:2000], 1000, 2000, key_all=k[:2000])
    ref = O.KMeanCacheOracle(B).update('L', 6, k[1000:2000].float().numpy(), 1000, 2000, key_all=k[:2000].float().numpy())
    np.testing.assert_allclose(km.numpy(), ref, rtol=1e-6, atol=1e-7)


def test_cached_block_means_eviction_and_growth(ksp):
    ksp.BLOCK = 64
    _, k, _, _ = synth.make_qkv(16, 256, 8, 2, 128, seed=4, with_v=False)
    for page in range(ksp._KMEAN_MAX_ENTRIES + 3):
        ksp._cached_block_means('E', page, k[:64], 0, 64)
    assert len(ksp._KMEAN_CACHE) == ksp._KMEAN_MAX_ENTRIES
    assert ('E', 0) not in ksp._KMEAN_CACHE and ('E', 2) not in ksp._KMEAN_CACHE and ('E', 3) in ksp._KMEAN_CACHE
    e = ksp._KMEAN_CACHE[('E', 3)]
    cap = e['km'].shape[1]
    e['last_kv'] = cap * 64                                          # pretend the request reached the capacity
    e['nb'] = cap
    ksp._cached_block_means('E', 3, k[:128], cap * 64, cap * 64 + 128)
    assert ksp._KMEAN_CACHE[('E', 3)]['km'].shape[1] == 2 * cap


def test_cached_scales_bookkeeping(ksp):
    q, k, v, _ = synth.make_qkv(512, 2048, 8, 2, 128, block=64, seed=31)
    sc = O.ScaleCacheOracle()
    s0 = ksp._cached_scales('L', 3, q, k[:1536], v[:1536], 1024)
    s1 = ksp._cached_scales('L', 3, q, k[:2048], v[:2048] * 2, 1536)      # continuity: reused
    s2 = ksp._cached_scales('L', 3, q * 4, k, v, 1000)                     # discontinuity: fresh
    r0 = sc.update('L', 3, q.float().numpy(), k[:1536].float().numpy(), v[:1536].float().numpy(), 1024)
    r1 = sc.update('L', 3, q.float().numpy(), k[:2048].float().numpy(), (v[:2048] * 2).float().numpy(), 1536)
    r2 = sc.update('L', 3, (q * 4).float().numpy(), k.float().numpy(), v.float().numpy(), 1000)
    np.testing.assert_allclose(np.array([s0, s1, s2]), np.array([r0, r1, r2]), rtol=1e-12)
    assert s0 == s1 and s2 != s1
    assert ksp._SCALE_CACHE[('L', 3)]['last_kv'] == 1000 + 512


def test_cached_scales_per_head(ksp):
    """SM120_SPARSE_FP8_SCALES=head: one scale per query head and per KV head, fixed at the request's
    first chunk like the per-tensor ones; the FP8 KV cache keys on them."""
    q, k, v, _ = synth.make_qkv(512, 2048, 8, 2, 128, seed=6, strength='strong')
    sq, sk, sv = ksp._cached_scales('H', 1, q, k[:1536], v[:1536], 1024, per_head=True)
    margin = ksp.SCALE_MARGIN / 448.0
    np.testing.assert_allclose(sq, np.abs(q.float().numpy()).max(axis=(0, 2)) * margin, rtol=1e-6)
    np.testing.assert_allclose(sk, np.abs(k[:1536].float().numpy()).max(axis=(0, 2)) * margin, rtol=1e-6)
    assert len(sq) == 8 and len(sk) == len(sv) == 2
    assert ksp._cached_scales('H', 1, q, None, None, 1536, per_head=True) == (sq, sk, sv)   # continued
    views = ksp._scale_views('cpu', (sq, sk, sv))
    assert [t.numel() for t in views] == [8, 2, 2, 8, 2, 2]
    np.testing.assert_allclose(views[4].numpy(), sk, rtol=1e-6)
    assert ksp._kv_scale_key((sq, sk, sv)) == (tuple(sk), tuple(sv))
    assert ksp._kv_scale_key((0.1, 0.2, 0.3)) == ((0.2,), (0.3,))


def test_cached_kv8_quantises_each_row_once(ksp, monkeypatch):
    """The FP8 KV cache quantises only a contiguous chunk's own rows; scale changes, gaps and q_start 0
    rebuild it from the full history."""
    from sm120_attn import ops
    calls = []

    def fake_quantize(x, scale, mode, out, transpose=False, rows_pad=0):
        calls.append((x.shape[0], round(float(scale.reshape(-1)[0]), 3)))
        out.copy_((x.float() * scale.reshape(1, 1, 1)).round().clamp(-100, 100).to(torch.int8).view(torch.uint8))

    monkeypatch.setattr(ops, 'quantize', fake_quantize)
    ksp._KV8_CACHE.clear()
    Hk, D = 2, 8
    k = torch.randn(10000, Hk, D).to(torch.bfloat16)
    v = torch.randn(10000, Hk, D).to(torch.bfloat16)
    sc = (0.1, 0.02, 0.03)
    k8, v8 = ksp._cached_kv8('L', 3, k, v, 0, 1000, sc)
    assert k8.shape == (1000, Hk, D) and calls == [(1000, 50.0), (1000, 33.333)]
    calls.clear()
    k8b, v8b = ksp._cached_kv8('L', 3, k, v, 1000, 2500, sc)            # contiguous: only the new rows
    assert calls == [(1500, 50.0), (1500, 33.333)] and k8b.shape[0] == 2500
    assert torch.equal(k8b[:1000], k8)                                   # earlier rows unchanged
    calls.clear()
    ksp._cached_kv8('L', 3, k, v, 3000, 4000, sc)                        # gap: rebuilt from row 0
    assert calls == [(4000, 50.0), (4000, 33.333)]
    calls.clear()
    ksp._cached_kv8('L', 3, k, v, 4000, 4500, (0.1, 0.04, 0.03))         # other scales: rebuilt
    assert calls == [(4500, 25.0), (4500, 33.333)]
    calls.clear()
    k8c, _ = ksp._cached_kv8('L', 3, k, v, 4500, 5000, (0.1, 0.04, 0.03))   # contiguous again
    assert calls == [(500, 25.0), (500, 33.333)] and k8c.shape[0] == 5000
    calls.clear()
    k8d, _ = ksp._cached_kv8('L', 3, k, v, 5000, 10000, (0.1, 0.04, 0.03))  # past the 8192-row capacity
    assert calls == [(5000, 25.0), (5000, 33.333)] and k8d.shape[0] == 10000
    assert torch.equal(k8d[:5000], k8c)                                  # rows kept across the regrowth
    ksp._KV8_CACHE.clear()


def test_fp8_warm_and_chunk_rows(ksp, monkeypatch):
    """_fp8_warm is true only when the block-mean, scale and FP8 KV caches all continue at q_start;
    a warm FP8 KV entry accepts just the chunk's rows (k_row0 > 0) and a stale one refuses them."""
    from sm120_attn import ops
    calls = []

    def fake_quantize(x, scale, mode, out, transpose=False, rows_pad=0):
        calls.append(x.shape[0])
        out.copy_((x.float() * scale.reshape(1, 1, 1)).round().clamp(-100, 100).to(torch.int8).view(torch.uint8))

    monkeypatch.setattr(ops, 'quantize', fake_quantize)
    ksp.BLOCK = 64
    g = torch.Generator().manual_seed(0)
    k = torch.randn(4000, 2, 8, generator=g).to(torch.bfloat16)
    v = torch.randn(4000, 2, 8, generator=g).to(torch.bfloat16)
    q = torch.randn(1000, 4, 8, generator=g).to(torch.bfloat16)
    assert not ksp._fp8_warm('W', 1, 1000)
    ksp._cached_block_means('W', 1, k[:1000], 0, 1000)
    sc = ksp._cached_scales('W', 1, q, k[:1000], v[:1000], 0)
    assert not ksp._fp8_warm('W', 1, 1000)                              # no FP8 KV entry yet
    k8, _ = ksp._cached_kv8('W', 1, k, v, 0, 1000, sc)
    assert ksp._fp8_warm('W', 1, 1000)
    assert not ksp._fp8_warm('W', 1, 1200) and not ksp._fp8_warm('W', 1, 0) and not ksp._fp8_warm('W', 2, 1000)
    calls.clear()
    k8b, v8b = ksp._cached_kv8('W', 1, k[992:2000], v[992:2000], 1000, 2000, sc, k_row0=992)
    assert calls == [1000, 1000] and k8b.shape[0] == 2000 and torch.equal(k8b[:1000], k8)
    full, _ = ksp._cached_kv8('X', 1, k, v, 0, 2000, sc)                 # the same rows quantised in one go
    assert torch.equal(full, k8b)
    with pytest.raises(RuntimeError):                                    # gap: a rebuild needs rows from 0
        ksp._cached_kv8('W', 1, k[2992:], v[2992:], 3000, 3500, sc, k_row0=2992)


def test_kv8_cache_byte_cap(ksp, monkeypatch):
    """The FP8 KV cache drops its oldest entries past KV8_CACHE_MAX_BYTES (never the one in use); a
    dropped request is rebuilt from its rows on its next chunk."""
    from sm120_attn import ops
    monkeypatch.setattr(ops, 'quantize', lambda x, scale, mode, out, transpose=False, rows_pad=0: out.zero_())
    k = torch.zeros(9000, 2, 8, dtype=torch.bfloat16)
    sc = (0.1, 0.02, 0.03)
    per_entry = 2 * 8192 * 2 * 8                                # k8 + v8 at the minimum capacity
    monkeypatch.setattr(ksp, 'KV8_CACHE_MAX_BYTES', 2 * per_entry)
    for layer in ('L0', 'L1', 'L2'):
        ksp._cached_kv8(layer, 1, k, k, 0, 1000, sc)
    assert list(k_[0] for k_ in ksp._KV8_CACHE) == ['L1', 'L2']  # the oldest went first
    ksp._cached_kv8('L1', 1, k, k, 1000, 9000, sc)              # grows past the cap: others dropped
    assert list(k_[0] for k_ in ksp._KV8_CACHE) == ['L1']
    assert ksp._KV8_CACHE[('L1', 1)]['rows'] == 9000
    ksp._KV8_CACHE.clear()


def test_cached_block_means_random_sequences(ksp):
    """Property test: any sequence of chunks of one (layer, request) - contiguous appends, restarts at
    0 and gaps that force a rebuild from the history, at block 64 and 128, chunk boundaries anywhere -
    gives the same block-mean cache as the oracle's restatement of the reference."""
    from hypothesis import given, settings, strategies as st

    @settings(max_examples=40, deadline=None, derandomize=True)
    @given(block=st.sampled_from([64, 128]),
           steps=st.lists(st.tuples(st.integers(1, 700), st.sampled_from(['next', 'restart', 'gap']),
                                    st.integers(1, 300)), min_size=1, max_size=6),
           seed=st.integers(0, 2 ** 16), page=st.sampled_from([0, 16, 48]))
    def check(block, steps, seed, page):
        ksp.BLOCK = block
        ksp._KMEAN_CACHE.clear()
        oracle = O.KMeanCacheOracle(block)
        keys = torch.randn(6 * 1000 + 8, 2, 8, generator=torch.Generator().manual_seed(seed)).to(torch.bfloat16)
        kf = keys.float().numpy()
        paged = _paged_copy(keys, page, seed) if page else None
        end = 0
        for n, kind, gap in steps:
            q_start = 0 if kind == 'restart' or end == 0 else end + (gap if kind == 'gap' else 0)
            kv_len = q_start + n
            hist = ksp._PagedRows(paged[0], paged[1], kv_len) if page else keys
            got = ksp._cached_block_means('fuzz', 7, keys[q_start:kv_len], q_start, kv_len, key_all=hist)
            ref = oracle.update('fuzz', 7, kf[q_start:kv_len], q_start, kv_len, key_all=kf)
            np.testing.assert_array_equal(got.numpy(), ref)
            assert ksp._KMEAN_CACHE[('fuzz', 7)]['last_kv'] == kv_len
            end = kv_len
    check()


def _paged_copy(x, page, seed):
    """x [rows, heads, D] spread over shuffled pages of a cache with spare pages: (cache, int32 table)."""
    npages = -(-x.shape[0] // page)
    total = npages + 3
    perm = torch.randperm(total, generator=torch.Generator().manual_seed(seed))[:npages]
    cache = torch.full((total, page) + tuple(x.shape[1:]), float('nan'), dtype=x.dtype)
    padded = torch.cat([x, x.new_zeros((npages * page - x.shape[0],) + tuple(x.shape[1:]))])
    cache[perm] = padded.view((npages, page) + tuple(x.shape[1:]))
    return cache, perm.to(torch.int32)


def test_paged_sources_match_gathered(ksp, monkeypatch):
    """The hook's caches built from _PagedRows (the pages read in place) equal the ones built from the
    gathered history: block-mean rebuilds (chunk starting on and inside a block), scales per tensor and
    per head, and the FP8 KV cache."""
    from sm120_attn import ops
    quant_calls = []

    def fake_quantize(x, scale, mode, out, transpose=False, rows_pad=0):
        out.copy_((x.float() * scale.reshape(1, -1, 1)).round().clamp(-100, 100).to(torch.int8).view(torch.uint8))

    def fake_quantize_paged(cache, table, row0, scale, mode, out):
        quant_calls.append((row0, out.shape[0]))
        rows = cache[table.long()].reshape(-1, cache.shape[2], cache.shape[3])
        fake_quantize(rows[row0:row0 + out.shape[0]], scale, mode, out)

    monkeypatch.setattr(ops, 'quantize', fake_quantize)
    monkeypatch.setattr(ops, 'quantize_paged', fake_quantize_paged)
    ksp.BLOCK = 64
    g = torch.Generator().manual_seed(5)
    k = torch.randn(3000, 2, 8, generator=g).to(torch.bfloat16)
    v = torch.randn(3000, 2, 8, generator=g).to(torch.bfloat16)
    q = torch.randn(500, 4, 8, generator=g).to(torch.bfloat16)
    kc, table = _paged_copy(k, 16, 1)
    vc, _ = _paged_copy(v, 16, 1)
    for q_start in (1024, 1000):
        kv_len = q_start + 500
        kp = ksp._PagedRows(kc, table, kv_len)
        ksp._KMEAN_CACHE.clear()
        a = ksp._cached_block_means('P', 1, k[q_start:kv_len], q_start, kv_len, key_all=kp).clone()
        ksp._KMEAN_CACHE.clear()
        b = ksp._cached_block_means('P', 1, k[q_start:kv_len], q_start, kv_len, key_all=k[:kv_len])
        assert torch.equal(a, b)
    for per_head in (False, True):
        ksp._SCALE_CACHE.clear()
        sa = ksp._cached_scales('P', 1, q, ksp._PagedRows(kc, table, 1500), ksp._PagedRows(vc, table, 1500), 1000,
                                per_head=per_head)
        ksp._SCALE_CACHE.clear()
        sb = ksp._cached_scales('P', 1, q, k[:1500], v[:1500], 1000, per_head=per_head)
        assert sa == sb
    sc = (0.1, 0.02, 0.03)
    ksp._KV8_CACHE.clear()
    k8a, v8a = ksp._cached_kv8('P', 1, ksp._PagedRows(kc, table, 1500), ksp._PagedRows(vc, table, 1500), 1000, 1500,
                               sc)
    assert quant_calls == [(0, 1500), (0, 1500)]
    k8a, v8a = k8a.clone(), v8a.clone()
    ksp._KV8_CACHE.clear()
    k8b, v8b = ksp._cached_kv8('P', 1, k, v, 1000, 1500, sc)
    assert torch.equal(k8a, k8b) and torch.equal(v8a, v8b)
    ksp._KV8_CACHE.clear()


def test_km_slot_written_bookkeeping(ksp):
    """km_slot hands the producer of a chunk's keys the entry's km to write the block means into (a new
    request, or one continuing at q_start); _cached_block_means(written=True) then records the chunk.
    A gap gives no slot (the unfused path rebuilds), and `written` without a slot is an error."""
    ksp.BLOCK = 64
    k = torch.randn(3000, 2, 8, generator=torch.Generator().manual_seed(2)).to(torch.bfloat16)
    km = ksp.km_slot('S', 0, 0, 1000, 2, 8, 'cpu')
    assert km is not None and km.shape[1] >= 16
    from sm120_attn import ops
    ops.block_means(k[:1000], 0, 64, km, 0)                  # the producer's write
    got = ksp._cached_block_means('S', 0, k[:1000], 0, 1000, written=True)
    entry = ksp._KMEAN_CACHE[('S', 0)]
    assert entry['nb'] == 16 and entry['last_kv'] == 1000 and 'slot' not in entry
    _, ref = O.block_means(k[:1000].float().numpy(), 0, 64)
    np.testing.assert_array_equal(got.numpy(), ref)
    km2 = ksp.km_slot('S', 0, 1000, 1800, 2, 8, 'cpu')      # continues: the same entry
    assert km2 is entry['km']
    ops.block_means(k[1000:1800], 1000, 64, km2, 0)
    got2 = ksp._cached_block_means('S', 0, k[1000:1800], 1000, 1800, written=True)
    ref2 = O.KMeanCacheOracle(64)
    ref2.update('S', 0, k[:1000].float().numpy(), 0, 1000)
    want = ref2.update('S', 0, k[1000:1800].float().numpy(), 1000, 1800)
    np.testing.assert_array_equal(got2.numpy(), want)
    assert ksp.km_slot('S', 0, 2000, 2500, 2, 8, 'cpu') is None   # gap: rebuilt by the unfused path
    with pytest.raises(RuntimeError):
        ksp._cached_block_means('S', 0, k[2000:2500], 2000, 2500, written=True)


def test_host_metadata_read_once_per_step(ksp):
    """The hook reads query_start_loc / seq_lens / first pages from the device once per metadata object
    (vLLM passes one object to every layer of a step), never reuses them for another object, and does
    not cache objects that cannot be weakly referenced."""
    import gc

    class Counted:
        def __init__(self, values):
            self.values, self.reads = values, 0

        def tolist(self):
            self.reads += 1
            return list(self.values)

        def __getitem__(self, idx):                      # block_table[:n, 0]
            return self

    class Meta:
        def __init__(self, qsl, seq, pages):
            self.query_start_loc, self.seq_lens, self.block_table = Counted(qsl), Counted(seq), Counted(pages)

    m = Meta([0, 5], [9], [3])
    for _ in range(4):                                   # four layers of one step
        assert ksp._host_metadata(m) == ([0, 5], [9], [3])
    assert (m.query_start_loc.reads, m.seq_lens.reads, m.block_table.reads) == (1, 1, 1)
    del m
    gc.collect()
    m2 = Meta([0, 7], [11], [4])                          # next step (possibly at the same address)
    assert ksp._host_metadata(m2) == ([0, 7], [11], [4])
    ns = types.SimpleNamespace(query_start_loc=Counted([0, 1]), seq_lens=Counted([2]), block_table=Counted([5]))
    ksp._host_metadata(ns)
    ksp._host_metadata(ns)
    assert ns.seq_lens.reads == 2                        # no weak reference: read every time


def test_cached_kv8_random_sequences(ksp, monkeypatch):
    """Property test: over any sequence of calls - contiguous chunks (with the full history or only
    the chunk's rows), restarts, gaps, scale changes, growth past the capacity - the e4m3 K/V the
    cache returns equal a fresh quantisation of rows [0, kv_len) with the current scales."""
    from hypothesis import given, settings, strategies as st
    from sm120_attn import ops

    def fake_quantize(x, scale, mode, out, transpose=False, rows_pad=0):
        out.copy_((x.float() * scale.reshape(1, 1, 1)).round().clamp(-100, 100).to(torch.int8).view(torch.uint8))

    monkeypatch.setattr(ops, 'quantize', fake_quantize)
    g = torch.Generator().manual_seed(5)
    k = torch.randn(40000, 2, 8, generator=g).to(torch.bfloat16)
    v = torch.randn(40000, 2, 8, generator=g).to(torch.bfloat16)

    def fresh(x, kv_len, s):
        out = torch.empty(kv_len, 2, 8, dtype=torch.uint8)
        fake_quantize(x[:kv_len], torch.tensor([1.0 / s]), 0, out)
        return out

    @settings(max_examples=40, deadline=None, derandomize=True)
    @given(steps=st.lists(st.tuples(st.integers(1, 5000), st.sampled_from(['next', 'next_rows', 'restart', 'gap', 'rescale'])),
                          min_size=1, max_size=7))
    def check(steps):
        ksp._KV8_CACHE.clear()
        end, sc = 0, (0.1, 0.02, 0.03)
        for n, kind in steps:
            if kind == 'rescale':
                sc = (0.1, sc[1] * 1.5, sc[2])
            q_start = 0 if kind == 'restart' or end == 0 else end + (777 if kind == 'gap' else 0)
            kv_len = q_start + n
            if kv_len > k.shape[0]:
                return
            if kind == 'next_rows' and q_start > 0:
                entry = ksp._KV8_CACHE.get(('P', 0))
                if entry is None or entry['rows'] != q_start or entry['scales'] != (sc[1], sc[2]):
                    continue                                   # chunk-only rows need a warm entry
                r0 = q_start - q_start % 16
                k8, v8 = ksp._cached_kv8('P', 0, k[r0:kv_len], v[r0:kv_len], q_start, kv_len, sc, k_row0=r0)
            else:
                k8, v8 = ksp._cached_kv8('P', 0, k, v, q_start, kv_len, sc)
            assert torch.equal(k8, fresh(k, kv_len, sc[1])) and torch.equal(v8, fresh(v, kv_len, sc[2]))
            end = kv_len
    check()
    ksp._KV8_CACHE.clear()


def test_block_masks_rejects_unpadded_input(ksp):
    sp = ksp.SparsePrefill(8, 2, 128, 'cpu')
    ksp.BLOCK = 64
    with pytest.raises(AssertionError):
        sp.block_masks(torch.zeros(100, 8, 128, dtype=torch.bfloat16), None, 64,
                       km=torch.zeros(2, 4, 128))


def test_reference_helper_matches_oracle():
    """`sparse_prefill.reference` (head-major K, per-KV-head masks) against the oracle."""
    import sm120_attn.sparse_prefill as m
    old = m.BLOCK
    m.BLOCK = 64
    try:
        q, k, v, _ = synth.make_qkv(100, 300, 4, 2, 128, seed=8)
        masks = torch.ones(2, 2, 5, dtype=torch.bool)
        masks[:, :, 1] = False
        out = m.reference(q, k.transpose(0, 1), v.transpose(0, 1), 200, masks)
        hm = masks.numpy().repeat(2, 0)
        # the reference expands masks over rows starting at row 0 of q (no front padding)
        ref = O.attention_ref(q.float().numpy(), k.float().numpy(), v.float().numpy(), 200, hm, q_block=64,
                              kv_block=64)
        np.testing.assert_allclose(out.numpy(), ref, rtol=1e-4, atol=2e-5)
    finally:
        m.BLOCK = old
