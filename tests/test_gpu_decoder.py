"""End-to-end prefill harness (benchmark configuration 5) on the GPU: its elementwise kernels against plain
fp32 PyTorch, and a small decoder's prefill through the sparse attention path against an fp32
reference forward of the same weights."""
import math

import pytest
import torch

from sm120_attn import decoder as dd
from sm120_attn import ops

DEV = torch.device('cuda') if torch.cuda.is_available() else None
pytestmark = pytest.mark.gpu


def _bf16(*shape, seed=0, scale=1.0):
    g = torch.Generator(device=DEV)
    g.manual_seed(seed)
    return (torch.randn(*shape, generator=g, device=DEV) * scale).to(torch.bfloat16)


@pytest.mark.parametrize('hidden', [512, 2048, 4096, 5120, 8192])
@pytest.mark.parametrize('with_delta', [True, False])
def test_add_rmsnorm_matches_torch(hidden, with_delta):
    rows, eps = 300, 1e-6
    h = _bf16(rows, hidden, seed=1)
    delta = _bf16(rows, hidden, seed=2, scale=0.5) if with_delta else None
    w = _bf16(hidden, seed=3)
    s = h.float() + (delta.float() if with_delta else 0.0)
    x_ref = s * torch.rsqrt(s.pow(2).mean(-1, keepdim=True) + eps) * w.float()
    x = torch.empty_like(h)
    ops.add_rmsnorm(h, w, x, eps, delta=delta)
    torch.cuda.synchronize()
    assert torch.equal(h, s.to(torch.bfloat16))                     # residual updated in place, rounded once
    torch.testing.assert_close(x.float(), x_ref, rtol=8e-3, atol=8e-3)


def test_rope_qkv_matches_torch():
    rows, H, Hk, D, pos0, theta = 200, 8, 2, 128, 5000, 1e6
    qkv = _bf16(rows, (H + 2 * Hk) * D, seed=4)
    table = dd.rope_table(pos0 + rows + 64, D, theta, DEV)
    q = torch.empty(rows, H, D, dtype=torch.bfloat16, device=DEV)
    kc = torch.zeros(rows + 10, Hk, D, dtype=torch.bfloat16, device=DEV)
    vc = torch.zeros_like(kc)
    ops.rope_qkv(qkv, H, Hk, D, table, pos0, q, kc[10:], vc[10:])
    torch.cuda.synchronize()
    x = qkv.float().view(rows, H + 2 * Hk, D)
    c = table[pos0:pos0 + rows, :D // 2][:, None, :]
    s = table[pos0:pos0 + rows, D // 2:][:, None, :]
    x1, x2 = x[..., :D // 2], x[..., D // 2:]
    rot = torch.cat([x1 * c - x2 * s, x2 * c + x1 * s], dim=-1)
    torch.testing.assert_close(q.float(), rot[:, :H], rtol=8e-3, atol=8e-3)
    torch.testing.assert_close(kc[10:].float(), rot[:, H:H + Hk], rtol=8e-3, atol=8e-3)
    assert torch.equal(vc[10:], qkv.view(rows, H + 2 * Hk, D)[:, H + Hk:])   # v copied unchanged
    assert torch.all(kc[:10] == 0) and torch.all(vc[:10] == 0)                # nothing outside the rows
    with pytest.raises(Exception):
        ops.rope_qkv(qkv, H, Hk, D, table[:pos0], pos0, q, kc[10:], vc[10:])   # positions past the table


def test_silu_mul_matches_torch():
    rows, inter = 333, 1000
    gu = _bf16(rows, 2 * inter, seed=5, scale=3.0)
    out = torch.empty(rows, inter, dtype=torch.bfloat16, device=DEV)
    ops.silu_mul(gu, out)
    torch.cuda.synchronize()
    ref = torch.nn.functional.silu(gu[:, :inter].float()) * gu[:, inter:].float()
    torch.testing.assert_close(out.float(), ref, rtol=8e-3, atol=8e-3)


SMALL = dict(layers=2, hidden=512, heads=8, kv_heads=2, head_dim=128, inter=1024, vocab=1024, init_std=0.05)


def _reference_logits(model, ids, e4m3_chunk=None):
    """fp32 forward of the model's weights; with e4m3_chunk, q, k and v are rounded to e4m3 with the
    scales the FP8 path derives (amax of the first chunk x SCALE_MARGIN / 448), so only the kernel's
    own rounding of P and its accumulation order separate the two."""
    import sm120_attn.sparse_prefill as ksp
    cfg = model.cfg
    scale = 1 / math.sqrt(cfg.head_dim)

    def attn(L, q, k, v):
        if e4m3_chunk is not None:
            deq = []
            for t in (q, k, v):
                s = t[:e4m3_chunk].abs().amax().clamp_min(1e-6) * ksp.SCALE_MARGIN / 448.0
                deq.append((t / s).clamp(-448, 448).to(torch.float8_e4m3fn).float() * s)
            q, k, v = deq
        return dd.causal_attention(q, k, v, scale)
    return dd.reference_prefill(cfg, model.layers, model.embed, model.lm_head, ids, attn)[0]


def _rel_l2(a, b):
    return ((a.float() - b.float()).norm() / b.float().norm()).item()


@pytest.mark.parametrize('kernel', ['sm120', 'sm120fp8'])
def test_small_decoder_dense_matches_fp32_reference(kernel):
    """tau 1 (every block kept): the chunked prefill (1024-token chunks, ragged last chunk) through
    this library's kernels against an fp32 forward of the same weights with exact causal attention.
    BF16 attention: last-token logits within 2e-2 rel-L2 (this pins the harness: chunking, RoPE,
    caches, norms, MLP).  FP8 attention: within 8e-2 of the fp32 forward given the same e4m3 q, k, v
    and within 0.15 of the exact one.  What remains with equal q, k, v is e4m3 P (3.6% RMS per
    element): on these near-flat random-weight attention rows the output is itself O(1/sqrt(n)), so
    that is 3-4% per attention output, and the residual stream (embedding std 0.05, smaller than the
    attention contribution) carries it through two layers (measured 0.062 and 0.092)."""
    cfg = dd.DecoderConfig(**SMALL)
    model = dd.TPDecoder(cfg, DEV, seed=7, tau=1.0, kernel=kernel, max_tokens=4096, chunk=1024, min_kv=0)
    ids = torch.randint(0, cfg.vocab, (2348,), generator=torch.Generator().manual_seed(1)).to(DEV)
    got = model.prefill(ids, return_logits=True)
    ops.check_status(DEV)
    exact = _rel_l2(got, _reference_logits(model, ids))
    if kernel == 'sm120':
        assert exact < 2e-2, exact
    else:
        same_q = _rel_l2(got, _reference_logits(model, ids, e4m3_chunk=1024))
        assert same_q < 8e-2 and exact < 0.15, (same_q, exact)
    model.release_caches()


def test_small_decoder_fp8_kv_cache_bit_identical():
    """Sparse selection (tau 0.95) over several chunks: keeping e4m3 K/V across chunks gives the same
    logits, bit for bit, as re-quantising the history in every chunk; the first token is the argmax."""
    cfg = dd.DecoderConfig(**SMALL)
    ids = torch.randint(0, cfg.vocab, (3000,), generator=torch.Generator().manual_seed(2)).to(DEV)
    outs = []
    for kv_cache in (False, True):
        model = dd.TPDecoder(cfg, DEV, seed=9, tau=0.95, kernel='sm120fp8', fp8_kv_cache=kv_cache,
                             max_tokens=4096, chunk=1024, min_kv=0)
        outs.append((model.prefill(ids, return_logits=True), model.prefill(ids)))
        model.release_caches()
    ops.check_status(DEV)
    assert torch.equal(outs[0][0], outs[1][0])
    assert int(outs[0][1]) == int(outs[0][0].argmax())
    assert torch.isfinite(outs[0][0]).all()
