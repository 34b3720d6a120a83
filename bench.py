#!/usr/bin/env python
"""Headline benchmark: sparse FP8 prefill attention on B200, TFLOPS on executed blocks.

One step = one prefill chunk through the drop-in API `SparsePrefill.forward_sm120fp8` with the
incremental block-mean cache (`_cached_block_means`): pool the chunk's keys into the cache
(kernel a), pool + quantise the queries (kernel a), score and select blocks (kernel b, two
launches), quantise K and V, block-sparse FP8 attention (kernel c).  Shape of benchmark configuration 2: Q 8192 rows at offset 57344
against 65536 keys, 64 query / 8 KV heads, head_dim 128, block 128, tau 0.95, seeded synthetic
inputs with the benchmark's hot-block injection.  Inputs (q 134 MB, k/v 134 MB each) exceed the
126 MB L2, so no flush is needed between steps.

value = (sum over ranks of causal FLOPs x kept fraction) / (max over ranks of the device time of
the K timed steps) - the reference's "sparse TFLOPS" definition (tests/test_fa_bf16.py:105-120).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b200|reference]
    torchrun --nproc-per-node N bench.py --gpus N ...      (one process per GPU)

Multi-GPU: units are KV-head groups with no data-path collective.  Default `--scaling strong`: the
8 KV heads of one problem are split over the N GPUs (8/N KV heads and their query heads per rank,
the partition of a tensor-parallel deployment), value = the problem's FLOPs / the slowest rank's
time.  `--scaling weak`: every rank owns 8 KV heads (64 query heads) of a problem with 8N KV heads.
`--impl reference` times the reference algorithm's CPU restatement (oracle/, numpy) on the host
cores on a bounded sample of the same workload (rank 0 only).

`--workload` selects the other measured configurations (the default line is the headline):
  dense      dense causal FP8 attention (tau = 1, no block lists), per-head e4m3 scales, same shape;
             TFLOPS of the causal FLOPs against the FP8 tensor peak
  selection  the selection path alone: K-chunk block means into the cache, Q pooling, block
             selection to CSR lists; GB/s of its algorithmic bytes against the HBM peak
  chunked    a 262144-token prefill in 32 chunks of 8192 through the drop-in API with the block-mean
             and scale caches carried across chunks (sink + local window + 16 hot blocks per KV head);
             TFLOPS on executed blocks over the whole prefill, ms per chunk in `config`
"""
from __future__ import annotations

import argparse
import json
import os
import subprocess
import sys
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
for p in (ROOT / 'qwen38-sparse-attn_b200', ROOT, ROOT / 'tests'):
    if str(p) not in sys.path:
        sys.path.insert(0, str(p))

METRIC = 'sparse prefill attention TFLOPS (exec blocks) + prefill TTFT @64K/128K/256K, 1/2/4/8 B200'
H_FULL, HK_FULL, D = 64, 8, 128
N_Q, KV, BLOCK, TAU = 8192, 65536, 128, 0.95
Q_START = KV - N_Q
# Kernels of this package launched per step: K-chunk block means, the one-pass query selection (with
# the fused e4m3 copy of q), K e4m3, V e4m3, attention.
LAUNCHES_PER_STEP = 5
ATTN_KERNEL = 'attn_fwd_kernel<fp8>'
# DRAM bytes (read + write) per attention launch measured by one ncu capture
# (`dram__bytes_read.sum + dram__bytes_write.sum` of the attention kernel in
# `bench.py --steps 2 --warmup 3 --no-cpu-baseline --profile-range`), keyed by what fixes them:
# (kernel, injection strength, query heads per GPU).  A line whose configuration has no capture
# reports traffic null rather than another configuration's figure.
ATTN_DRAM_CAPTURES = {
    ('attn_fwd_kernel<fp8>', 'unit', 64): 326326784,       # 220.0 MB read + 106.3 MB written
}


def peaks():
    f = ROOT / 'MEASURED_PEAKS.json'
    if f.exists():
        d = json.loads(f.read_text())
        return float(d['hbm_gbs']), float(d['bf16_tflops']), 'measured'
    return 6650.0, 1590.0, 'fallback'


def causal_flops(h, d, n, kv):
    return 4.0 * h * d * n * (kv - n + (n + 1) / 2)


class Clocks:
    """nvidia-smi sampling of SM clocks and throttle reasons during the timed region."""

    FIELDS = ('index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,'
              'clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,'
              'clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap')

    def __init__(self, gpu_index):
        self.gpu = gpu_index
        self.proc = None

    def start(self):
        try:
            self.proc = subprocess.Popen(['nvidia-smi', f'--id={self.gpu}', f'--query-gpu={self.FIELDS}',
                                          '--format=csv,noheader,nounits', '-lms', '200'],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None

    def stop(self):
        if self.proc is None:
            return {'sm_mhz': None, 'sm_max_mhz': None, 'reasons': ['nvidia-smi unavailable']}
        self.proc.terminate()
        try:
            out, _ = self.proc.communicate(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
            out, _ = self.proc.communicate()
        sm, mx, reasons = [], None, set()
        names = ['hw_slowdown', 'hw_thermal_slowdown', 'sw_thermal_slowdown', 'sw_power_cap']
        for line in out.strip().splitlines():
            parts = [x.strip() for x in line.split(',')]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                mx = float(parts[2])
            except ValueError:
                continue
            for nm, val in zip(names, parts[5:9]):
                if val.lower() == 'active':
                    reasons.add(nm)
        sm.sort()
        return {'sm_mhz': sm[len(sm) // 2] if sm else None, 'sm_max_mhz': mx, 'reasons': sorted(reasons),
                'samples': len(sm)}


def rank_shape_kv_heads(n):
    """KV heads of rank 0 of an n-GPU strong split of the benchmark's 8 KV heads."""
    from sm120_attn.shard import kv_head_range
    try:
        lo, hi = kv_head_range(0, n, HK_FULL)
    except ValueError as e:
        raise SystemExit(f'--rank-shape: {e}')
    return hi - lo


def make_rank_inputs(hk, seed, strength, device):
    import synth
    q, k, v, _ = synth.make_qkv(N_Q, KV, hk * (H_FULL // HK_FULL), hk, D, block=BLOCK, q_start=Q_START, seed=seed,
                                strength=strength, hot=6, device=device)
    return q.contiguous(), k.contiguous(), v.contiguous()


def check_chunk_slice(q, k, v, out, counts, lists, scales, h, hk, tiles=2):
    """Correctness check of one benchmarked chunk, run once outside the timed region: the last `tiles`
    128-row query tiles of the query heads of KV head 0, against a torch fp32 reference on the GPU.

    * selection: pooled fp32 scores, softmax, descending sort and float64 cumulative mass (the tau rule
      of sparse_prefill.py:64-84) must give the kernel's block lists, except blocks whose cumulative
      mass lies within 1e-4 of tau or that tie the boundary probability;
    * attention: fp32 softmax attention on the same e4m3 operands (the glue's quantisation) and the
      kernel's lists must be within rel-L2 3e-2 of the kernel's bf16 output.
    Returns a dict of the figures; 'ok' is False when either check fails.
    """
    import torch
    from sm120_attn import ops
    from sm120_attn._native import SA_QUANT_MUL_BF16
    g = h // hk
    MB, NB = N_Q // BLOCK, KV // BLOCK
    dev = q.device
    scale = D ** -0.5
    tile_ids = list(range(MB - tiles, MB))
    rows = torch.arange((MB - tiles) * BLOCK, N_Q, device=dev)
    kf = k[:, 0].float()                                                    # [KV, D] of KV head 0
    km = kf.view(NB, BLOCK, D).mean(1)
    cnt, lst = counts.view(h, MB), lists.view(h, MB, -1)
    sel_bad, mism = 0, 0
    for hh in range(g):
        for m in tile_ids:
            qm = q[m * BLOCK:(m + 1) * BLOCK, hh].float().mean(0)
            gi = Q_START // BLOCK + m
            logit = (km[:gi + 1] @ qm) * scale
            p = torch.softmax(logit, 0)
            ps, order = torch.sort(p, descending=True)
            csum = torch.cumsum(ps.double(), 0)
            keep = int((csum.float() < TAU).sum().item()) + 1
            ref = torch.zeros(NB, dtype=torch.bool, device=dev)
            ref[order[:keep]] = True
            ref[gi] = True
            ref[0] = True
            got = torch.zeros(NB, dtype=torch.bool, device=dev)
            c = int(cnt[hh, m].item())
            got[lst[hh, m, :c].long()] = True
            for j in torch.nonzero(got != ref).flatten().tolist():
                mism += 1
                pos = int((order == j).nonzero().item()) if j <= gi else -1
                if pos < 0:
                    sel_bad += 1
                    continue
                inc = float(csum[pos])
                exc = inc - float(ps[pos])
                edge = [float(ps[t]) for t in (keep - 1, keep) if 0 <= t <= gi]
                if not (abs(inc - TAU) < 1e-4 or abs(exc - TAU) < 1e-4 or
                        any(abs(float(ps[pos]) - e) <= 1e-5 * e for e in edge)):
                    sel_bad += 1
    # attention on the kernel's lists and the glue's e4m3 operands
    sq, sk, sv = scales
    inv = torch.tensor([1.0 / sq, 1.0 / sk, 1.0 / sv], dtype=torch.float32, device=dev)
    q8 = torch.empty(len(rows), g, D, dtype=torch.uint8, device=dev)
    ops.quantize(q[rows][:, :g].contiguous(), inv[0:1], SA_QUANT_MUL_BF16, q8)
    k8 = torch.empty(KV, 1, D, dtype=torch.uint8, device=dev)
    v8 = torch.empty(KV, 1, D, dtype=torch.uint8, device=dev)
    ops.quantize(k[:, 0:1], inv[1:2], SA_QUANT_MUL_BF16, k8)
    ops.quantize(v[:, 0:1], inv[2:3], SA_QUANT_MUL_BF16, v8)
    f8 = torch.float8_e4m3fn
    qd = q8.view(f8).float() * sq
    kd = k8.view(f8).float()[:, 0] * sk
    vd = v8.view(f8).float()[:, 0] * sv
    pos_k = torch.arange(KV, device=dev)
    num = den = 0.0
    for hh in range(g):
        s_ = (qd[:, hh] @ kd.T) * scale                                     # [rows, KV]
        allowed = pos_k[None, :] <= (Q_START + rows)[:, None]
        blk = torch.zeros(tiles, NB, dtype=torch.bool, device=dev)
        for i, m in enumerate(tile_ids):
            c = int(cnt[hh, m].item())
            blk[i, lst[hh, m, :c].long()] = True
        allowed &= blk.repeat_interleave(BLOCK, 0).repeat_interleave(BLOCK, 1)
        s_ = s_.masked_fill(~allowed, float('-inf'))
        ref = torch.softmax(s_, -1) @ vd
        got = out[rows, hh].float()
        num += float(((got - ref) ** 2).sum())
        den += float((ref ** 2).sum())
    rel = (num / max(den, 1e-30)) ** 0.5
    return {'ok': sel_bad == 0 and rel < 3e-2, 'rows_checked': int(len(rows)) * g, 'heads': g,
            'mask_mismatches': mism, 'mask_unexplained': sel_bad, 'attn_rel_l2': round(rel, 5),
            'reference': 'torch fp32 on the GPU (selection tau rule; masked softmax attention on the same e4m3 '
                         'operands)', 'tolerance': 'masks exact outside the 1e-4 tau band / ties; rel-L2 3e-2'}


def run_b200(args):
    import torch
    import torch.distributed as dist
    world = int(os.environ.get('WORLD_SIZE', '1'))
    rank = int(os.environ.get('RANK', '0'))
    local = int(os.environ.get('LOCAL_RANK', '0'))
    torch.cuda.set_device(local)
    dev = torch.device('cuda', local)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group('nccl', timeout=timedelta(seconds=120), device_id=dev)
    import sm120_attn.sparse_prefill as ksp
    from sm120_attn import ops
    from sm120_attn.shard import kv_head_range, reduce_over_ranks
    ksp.BLOCK = BLOCK
    if args.scaling == 'strong':
        try:
            lo, hi = kv_head_range(rank, world, HK_FULL)     # this rank's KV heads of the one problem
        except ValueError as e:
            raise SystemExit(f'strong scaling: {e}')
        hk = hi - lo
    else:
        hk = HK_FULL                                         # every rank runs a full problem
    if args.rank_shape > 1 and world == 1:                   # one rank's share of an N-GPU strong split
        hk = rank_shape_kv_heads(args.rank_shape)
    h = hk * (H_FULL // HK_FULL)
    q, k, v = make_rank_inputs(hk, 1000 + rank, args.strength, dev)
    sp = ksp.SparsePrefill(h, hk, D, dev, tau=TAU, min_kv=0, min_q=0, kernel='sm120fp8')
    out = torch.empty(N_Q, h, D, dtype=torch.bfloat16, device=dev)
    layer = 'bench'
    # request state before this chunk: history keys 0..Q_START are in the cache (built once, untimed)
    ksp._KMEAN_CACHE.clear()
    ksp._cached_block_means(layer, 0, k[:Q_START], 0, Q_START)
    scales = ksp._cached_scales(layer, 0, q, k, v, 0)

    def rewind():
        e = ksp._KMEAN_CACHE[(layer, 0)]
        e['last_kv'] = Q_START
        e['nb'] = Q_START // BLOCK

    def step(qq, kk_chunk):
        km = ksp._cached_block_means(layer, 0, kk_chunk, Q_START, KV)
        sp.forward_sm120fp8(qq, k, v, Q_START, out=out, km=km, scales=scales)

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize(dev)

    # ---------------- device-resident timed region (clocks sampled from warm-up through the e2e run,
    # since one timed region is shorter than a few nvidia-smi sampling periods)
    clocks = Clocks(local)
    clocks.start()
    for _ in range(args.warmup):
        rewind()
        step(q, k[Q_START:])
    sp.kernel_events = []
    barrier()
    stream = torch.cuda.current_stream(dev)
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    if args.profile_range:
        torch.cuda.profiler.start()
    t0.record(stream)
    for _ in range(args.steps):
        rewind()
        step(q, k[Q_START:])
    t1.record(stream)
    barrier()
    if args.profile_range:
        torch.cuda.profiler.stop()
    ms_total = t0.elapsed_time(t1)
    attn_ms = [s.elapsed_time(e) for s, e in sp.kernel_events]
    sp.kernel_events = None
    kept_blocks = int(sp.last_counts.sum().item())
    causal_blocks = h * ((Q_START // BLOCK) * (N_Q // BLOCK) + (N_Q // BLOCK) * (N_Q // BLOCK + 1) // 2)
    kept = kept_blocks / causal_blocks
    flops = causal_flops(h, D, N_Q, KV) * kept
    tile_flops = kept_blocks * 4.0 * D * 128 * 128
    # bytes the attention launch must move at least: q8 and the first KV rows of k8 / v8 read once,
    # the block lists read, the bf16 output written
    algo_bytes = N_Q * h * D + 2 * KV * hk * D + 2 * N_Q * h * D + 4 * h * (N_Q // BLOCK) + \
        4 * kept_blocks
    # ---------------- end-to-end through the public API with pinned host buffers.  Every step copies
    # its chunk's q, k and v in from pinned host memory and its output back; two device buffer sets
    # and two copy streams let step i+1's upload and step i-1's download run under step i's compute
    # (a serving loop's double buffering).  The timed region spans the first upload to the last
    # download.
    q_h = q.cpu().pin_memory()
    k_h = k[Q_START:].cpu().pin_memory()
    v_h = v[Q_START:].cpu().pin_memory()
    o_h = [torch.empty(out.shape, dtype=out.dtype).pin_memory() for _ in range(2)]
    bufs = [(torch.empty_like(q), k.clone(), v.clone(), torch.empty_like(out)) for _ in range(2)]
    cs_in, cs_out = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
    in_ready = [torch.cuda.Event() for _ in range(2)]
    comp_done = [torch.cuda.Event() for _ in range(2)]
    out_done = [torch.cuda.Event() for _ in range(2)]

    def upload(i):
        qd, kb, vb, _ = bufs[i % 2]
        cs_in.wait_event(comp_done[i % 2])                       # step i-2 has finished with the set
        with torch.cuda.stream(cs_in):
            qd.copy_(q_h, non_blocking=True)
            kb[Q_START:].copy_(k_h, non_blocking=True)
            vb[Q_START:].copy_(v_h, non_blocking=True)
            in_ready[i % 2].record(cs_in)

    def compute(i):
        qd, kb, vb, ob = bufs[i % 2]
        stream.wait_event(in_ready[i % 2])
        stream.wait_event(out_done[i % 2])                        # step i-2's output has left the set
        rewind()
        km = ksp._cached_block_means(layer, 0, kb[Q_START:], Q_START, KV)
        sp.forward_sm120fp8(qd, kb, vb, Q_START, out=ob, km=km, scales=scales)
        comp_done[i % 2].record(stream)

    def download(i):
        cs_out.wait_event(comp_done[i % 2])
        with torch.cuda.stream(cs_out):
            o_h[i % 2].copy_(bufs[i % 2][3], non_blocking=True)
            out_done[i % 2].record(cs_out)

    def e2e_run(n_steps, start_event=None):
        if start_event is not None:
            cs_in.wait_event(start_event)
        upload(0)
        for i in range(n_steps):
            if i + 1 < n_steps:
                upload(i + 1)
            compute(i)
            download(i)
        for b in range(2):
            stream.wait_event(out_done[b])

    e2e_run(max(2, args.warmup))
    barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    e2e_run(args.steps, e0)
    e1.record(stream)
    barrier()
    o_h = o_h[0]
    e2e_ms = e0.elapsed_time(e1)
    clk = clocks.stop()
    h2d = q_h.numel() * 2 + k_h.numel() * 2 + v_h.numel() * 2
    d2h = o_h.numel() * 2
    ops.check_status(dev)
    # ---------------- correctness of the benchmarked output (outside the timed regions): the last
    # e2e step wrote bufs[(steps - 1) % 2] from the same inputs as every step
    out_last = bufs[(args.steps - 1) % 2][3]
    check = check_chunk_slice(q, k, v, out_last, sp.last_counts, sp.last_lists, scales, h, hk)
    # ---------------- reductions over ranks
    (ms_total, e2e_ms, attn_avg, neg_min), (flops_all, tile_all, n_failed) = reduce_over_ranks(
        [ms_total, e2e_ms, sum(attn_ms) / max(len(attn_ms), 1), -ms_total],
        [flops, tile_flops, 0.0 if check['ok'] else 1.0], device=dev)
    hbm, bf16, how = peaks()
    fp8_peak = 2.0 * bf16
    value = flops_all * args.steps / (ms_total * 1e-3) / 1e12
    e2e_val = flops_all * args.steps / (e2e_ms * 1e-3) / 1e12
    achieved = (tile_all / world) / (attn_avg * 1e-3) / 1e12
    line = {
        'metric': METRIC,
        'value': round(value, 2),
        'unit': 'TFLOPS',
        'n_gpus': world,
        'steps': args.steps,
        'warmup': args.warmup,
        'ms_per_step': round(ms_total / args.steps, 4),
        'higher_is_better': True,
        'scaling': args.scaling,
        'vs_baseline': None,
        'dtype': 'fp8-e4m3 (fp32 accumulate, bf16 in/out)',
        'data': 'synthetic (seeded N(0,1) q/k/v with sink + 6 hot blocks per KV head)',
        'config': {
            **chunk_config(args, world),
            'gpus_active': world, 'kv_heads_per_gpu': hk,
            'ms_per_step_fastest_rank': round(-neg_min / args.steps, 4),
            'kept_fraction': round(kept, 4),
            'l2': 'inputs larger than L2 (q 134 MB, k 134 MB, v 134 MB per GPU); no flush',
        },
        'roofline': {
            'bound': 'tensor', 'kernel': ATTN_KERNEL,
            'achieved': round(achieved, 1), 'peak': round(fp8_peak, 1), 'unit': 'TFLOP/s',
            'frac': round(achieved / fp8_peak, 4),
            'peak_source': f'2 x {how} bf16 dense burst ({bf16} TF/s, MEASURED_PEAKS.json): B200 e4m3 dense rate is '
                           'twice bf16',
            'attn_ms_per_launch': round(attn_avg, 4),
            'traffic': ATTN_DRAM_CAPTURES.get((ATTN_KERNEL, args.strength, h)),
            'algorithmic_bytes': algo_bytes,
        },
        'e2e': {'value': round(e2e_val, 2), 'unit': 'TFLOPS', 'h2d_bytes_per_step': h2d, 'd2h_bytes_per_step': d2h,
                'ms_per_step': round(e2e_ms / args.steps, 4),
                'path': 'pinned host q/k/v of the chunk -> SparsePrefill.forward_sm120fp8 -> pinned host output; '
                        'double-buffered: uploads and downloads on two copy streams overlap neighbouring steps\' compute'},
        'gpu_launches': LAUNCHES_PER_STEP * args.steps,
        'clocks': clk,
    }
    line['check'] = check
    if not args.no_also and not n_failed:
        line['config']['also'] = secondary_figures(args, h, hk, dev, rank, world)
    if args.ttft_tokens > 0 and not n_failed:
        # second half of the metric: prefill TTFT of the config-5 decoder, measured on the same ranks
        # after the chunk workload (its tensors released first)
        del q, k, v, out, bufs, q_h, k_h, v_h
        ksp._KMEAN_CACHE.clear()
        torch.cuda.empty_cache()
        line['config']['ttft'] = measure_ttft(args.ttft_tokens, dev, rank, world, local)
    if n_failed:
        if rank == 0:
            print(f'bench: output check failed on {int(n_failed)} rank(s): {check}; no result line', file=sys.stderr,
                  flush=True)
        if world > 1:
            dist.barrier()
            dist.destroy_process_group()
        raise SystemExit(3)
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        line['cpu_baseline'] = cpu_baseline(args.strength)
    if rank == 0:
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def _chunk_variant(args, h, hk, dev, rank, world, strength):
    """The default chunk step at another injection strength, device-resident: max-over-ranks ms per
    step, kept fraction, executed-tile TFLOPS and the attention launch's ms."""
    import torch
    import sm120_attn.sparse_prefill as ksp
    from sm120_attn.shard import reduce_over_ranks
    q, k, v = make_rank_inputs(hk, 1000 + rank, strength, dev)
    sp = ksp.SparsePrefill(h, hk, D, dev, tau=TAU, min_kv=0, min_q=0, kernel='sm120fp8')
    out = torch.empty(N_Q, h, D, dtype=torch.bfloat16, device=dev)
    layer = 'bench-' + strength
    ksp._cached_block_means(layer, 0, k[:Q_START], 0, Q_START)
    scales = ksp._cached_scales(layer, 0, q, k, v, 0)

    def rewind():
        e = ksp._KMEAN_CACHE[(layer, 0)]
        e['last_kv'], e['nb'] = Q_START, Q_START // BLOCK

    def step():
        km = ksp._cached_block_means(layer, 0, k[Q_START:], Q_START, KV)
        sp.forward_sm120fp8(q, k, v, Q_START, out=out, km=km, scales=scales)
    for _ in range(args.warmup):
        rewind()
        step()
    sp.kernel_events = []
    ms = _timed(step, args.steps, dev, world, before=rewind)
    attn = [a.elapsed_time(b) for a, b in sp.kernel_events]
    sp.kernel_events = None
    kept_blocks = int(sp.last_counts.sum().item())
    causal_blocks = h * ((Q_START // BLOCK) * (N_Q // BLOCK) + (N_Q // BLOCK) * (N_Q // BLOCK + 1) // 2)
    (ms, attn_ms), (tile_flops, kept_sum, causal_sum) = reduce_over_ranks(
        [ms, sum(attn) / max(len(attn), 1)], [kept_blocks * 4.0 * D * 128 * 128, kept_blocks, causal_blocks],
        device=dev)
    del ksp._KMEAN_CACHE[(layer, 0)]
    return {'injection': strength, 'kept_fraction': round(kept_sum / causal_sum, 4),
            'ms_per_step': round(ms / args.steps, 4),
            'tflops_executed': round(tile_flops * args.steps / (ms * 1e-3) / 1e12, 1),
            'attn_ms_per_launch': round(attn_ms, 4)}


def secondary_figures(args, h, hk, dev, rank, world):
    """The benchmark's other configurations, measured in the same run on the same ranks (device-resident,
    CUDA events, max over ranks): the chunk at strong injection, dense causal FP8 (tau 1, config 3) and
    the selection of one chunk (config 2)."""
    import types
    from sm120_attn.shard import reduce_over_ranks
    sub = types.SimpleNamespace(**{**vars(args), 'steps': max(3, min(args.steps, 10))})
    also = {'strong_injection_chunk': _chunk_variant(sub, h, hk, dev, rank, world, 'strong')}
    d = _dense(sub, h, hk, dev, rank)
    (ms,), (work,) = reduce_over_ranks([d['ms']], [d['work']], device=dev)
    also['dense_fp8'] = {'ms_per_step': round(ms / sub.steps, 4),
                         'tflops': round(work * sub.steps / (ms * 1e-3) / 1e12, 1),
                         'workload': d['config']['workload']}
    sel = _selection(sub, h, hk, dev, rank)
    (ms, kms), (work, kwork) = reduce_over_ranks([sel['ms'], sel['kernel_ms']], [sel['work'], sel['kernel_work']],
                                                 device=dev)
    hbm, _, _ = peaks()
    also['selection'] = {'ms_per_step': round(ms / sub.steps, 4),
                         'gbs': round(work * sub.steps / (ms * 1e-3) / 1e9, 1),
                         'kernel': sel['kernel'], 'kernel_us': round(kms * 1e3, 1),
                         'kernel_frac_of_hbm': round(kwork / (kms * 1e-3) / 1e9 / hbm, 4)}
    also['steps'] = sub.steps
    return also


def _rank_env():
    import torch
    import torch.distributed as dist
    world = int(os.environ.get('WORLD_SIZE', '1'))
    rank = int(os.environ.get('RANK', '0'))
    local = int(os.environ.get('LOCAL_RANK', '0'))
    torch.cuda.set_device(local)
    dev = torch.device('cuda', local)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group('nccl', timeout=timedelta(seconds=120), device_id=dev)
    return world, rank, local, dev


PROFILE_RANGE = False        # set from --profile-range: bracket the first timed region for ncu


def _timed(fn, steps, dev, world, before=None):
    """Device time (ms) of `steps` calls of fn on the current stream, barrier + synchronize on both sides."""
    global PROFILE_RANGE
    import torch
    import torch.distributed as dist

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize(dev)
    barrier()
    stream = torch.cuda.current_stream(dev)
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    prof = PROFILE_RANGE
    PROFILE_RANGE = False
    if prof:
        torch.cuda.profiler.start()
    t0.record(stream)
    for _ in range(steps):
        if before is not None:
            before()
        fn()
    t1.record(stream)
    barrier()
    if prof:
        torch.cuda.profiler.stop()
    return t0.elapsed_time(t1)


def _kernel_ms(fn, dev, reps=5):
    """Average device time of one call of fn alone (CUDA events on the launching stream)."""
    import torch
    stream = torch.cuda.current_stream(dev)
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize(dev)
    a.record(stream)
    for _ in range(reps):
        fn()
    b.record(stream)
    torch.cuda.synchronize(dev)
    return a.elapsed_time(b) / reps


def _dense(args, h, hk, dev, rank):
    """Config 3: dense causal FP8 attention, per-head scales, no lists."""
    import torch
    from sm120_attn import ops
    from sm120_attn._native import SA_QUANT_DIV
    from sm120_attn.kernels import attention_sm120_fp8
    q, k, v = make_rank_inputs(hk, 2000 + rank, args.strength, dev)
    scl = [ops.absmax(t, per_head=True).clamp_min_(1e-6) / 448.0 for t in (q, k, v)]
    q8, k8, v8 = (torch.empty(t.shape, dtype=torch.uint8, device=dev) for t in (q, k, v))
    for t, s8, sc in zip((q, k, v), (q8, k8, v8), scl):
        ops.quantize(t, sc, SA_QUANT_DIV, s8)
    out = torch.empty(N_Q, h, D, dtype=torch.bfloat16, device=dev)

    def step():
        ops.attn_fp8(q8, k8, v8, out, KV, 0, Q_START, None, None, 64, scl[0], scl[1], scl[2], D ** -0.5)
    for _ in range(args.warmup):
        step()
    ms = _timed(step, args.steps, dev, int(os.environ.get('WORLD_SIZE', '1')))
    flops = causal_flops(h, D, N_Q, KV)
    # e2e: the drop-in driver on host tensors (per-tensor scales, quantised on the device)
    q_h, k_h, v_h = (t.cpu().pin_memory() for t in (q, k, v))
    o_h = torch.empty(out.shape, dtype=out.dtype).pin_memory()
    qd, kd, vd = (torch.empty_like(t) for t in (q, k, v))

    def e2e():
        for d_, h_ in ((qd, q_h), (kd, k_h), (vd, v_h)):
            d_.copy_(h_, non_blocking=True)
        attention_sm120_fp8(qd, kd, vd, Q_START, out=out)
        o_h.copy_(out, non_blocking=True)
    e2e()
    e2e_ms = _timed(e2e, args.steps, dev, int(os.environ.get('WORLD_SIZE', '1')))
    ops.check_status(dev)
    return {'ms': ms, 'e2e_ms': e2e_ms, 'work': flops, 'unit': 'TFLOPS', 'scale': 1e12,
            'kernel': 'attn_fwd_kernel<fp8>', 'kernel_ms': ms / args.steps, 'kernel_work': flops,
            'bound': 'tensor', 'h2d': sum(t.numel() * 2 for t in (q_h, k_h, v_h)), 'd2h': o_h.numel() * 2,
            'launches': 1,
            'config': {'workload': f'dense causal FP8 attention (tau 1, no lists): q {N_Q} @ {Q_START} vs {KV} keys, '
                                   f'H {h}/Hk {hk}/D {D}, per-head e4m3 scales amax/448',
                       'e2e_path': 'pinned host bf16 q/k/v -> attention_sm120_fp8 (per-tensor scales, 3 host syncs) '
                                   '-> pinned host output'}}


def _selection(args, h, hk, dev, rank):
    """Config 2: K-chunk block means into the cache, Q pooling, selection to CSR lists."""
    import torch
    import sm120_attn.sparse_prefill as ksp
    from sm120_attn import ops
    from sm120_attn._native import SA_SELECT_PER_HEAD
    ksp.BLOCK = BLOCK
    q, k, _ = make_rank_inputs(hk, 3000 + rank, args.strength, dev)
    sp = ksp.SparsePrefill(h, hk, D, dev, tau=TAU, min_kv=0, min_q=0, kernel='sm120')
    layer = 'bench-sel'
    ksp._KMEAN_CACHE.clear()
    ksp._cached_block_means(layer, 0, k[:Q_START], 0, Q_START)
    MB, NB = N_Q // BLOCK, KV // BLOCK
    counts = torch.empty(h * MB, dtype=torch.int32, device=dev)
    lists = torch.empty(h * MB, NB, dtype=torch.int32, device=dev)
    kc = k[Q_START:]

    def rewind():
        e = ksp._KMEAN_CACHE[(layer, 0)]
        e['last_kv'] = Q_START
        e['nb'] = Q_START // BLOCK

    def step(qq=q, kk=kc):
        km = ksp._cached_block_means(layer, 0, kk, Q_START, KV)
        sp._select(qq, Q_START, Q_START // BLOCK, MB, km, NB, SA_SELECT_PER_HEAD, counts=counts, lists=lists)
    for _ in range(args.warmup):
        rewind()
        step()
    ms = _timed(step, args.steps, dev, int(os.environ.get('WORLD_SIZE', '1')), before=rewind)
    nnz = int(counts.sum().item())
    nbytes = 2 * N_Q * h * D + 2 * N_Q * hk * D + 4 * hk * NB * D + 4 * hk * MB * D + 4 * h * MB + 4 * nnz
    km = ksp._KMEAN_CACHE[(layer, 0)]['km'][:, :NB]
    fused = ops.select_q_supported(h, hk, D, NB, SA_SELECT_PER_HEAD)
    sel_ms = _kernel_ms(lambda: sp._select(q, Q_START, Q_START // BLOCK, MB, km, NB, SA_SELECT_PER_HEAD, counts=counts,
                                           lists=lists), dev)
    # the one-pass kernel reads the query chunk and the key means and writes the CSR lists
    sel_bytes = 2 * N_Q * h * D + 4 * hk * NB * D + 4 * h * MB + 4 * nnz
    q_h, k_h = q.cpu().pin_memory(), kc.cpu().pin_memory()
    c_h = torch.empty(counts.shape, dtype=counts.dtype).pin_memory()
    l_h = torch.empty(lists.shape, dtype=lists.dtype).pin_memory()
    qd, kd = torch.empty_like(q), torch.empty_like(kc)

    def e2e():
        qd.copy_(q_h, non_blocking=True)
        kd.copy_(k_h, non_blocking=True)
        step(qd, kd)
        c_h.copy_(counts, non_blocking=True)
        l_h.copy_(lists, non_blocking=True)
    rewind()
    e2e()
    e2e_ms = _timed(e2e, args.steps, dev, int(os.environ.get('WORLD_SIZE', '1')), before=rewind)
    ops.check_status(dev)
    return {'ms': ms, 'e2e_ms': e2e_ms, 'work': nbytes, 'unit': 'GB/s', 'scale': 1e9,
            'kernel': 'select_fused_kernel' if fused else 'block_means_kernel + score_kernel + select_kernel',
            'kernel_ms': sel_ms, 'kernel_work': sel_bytes, 'bound': 'hbm',
            'h2d': q_h.numel() * 2 + k_h.numel() * 2, 'd2h': c_h.numel() * 4 + l_h.numel() * 4,
            'launches': 2 if fused else 3,
            'config': {**selection_config(args, h, hk),
                       'bytes_per_step': nbytes, 'nnz': nnz,
                       'note': 'value = algorithmic bytes (q + k chunk read, km read/append, CSR write) / time; '
                               'roofline on the query-side selection launch alone (q, km read, CSR write)'}}


def _chunked(args, h, hk, dev, rank):
    """Config 4: 262144-token prefill in 32 chunks of 8192, caches carried across chunks."""
    import torch
    import sm120_attn.sparse_prefill as ksp
    import synth
    from sm120_attn import ops
    ksp.BLOCK = BLOCK
    total, chunk = 262144, 8192
    q, k, v, _ = synth.make_qkv(total, total, h, hk, D, block=BLOCK, q_start=0, seed=4000 + rank,
                                strength='strong', hot=16, local=4, device=dev)
    sp = ksp.SparsePrefill(h, hk, D, dev, tau=TAU, min_kv=8192, min_q=0, kernel='sm120fp8')
    out = torch.empty(chunk, h, D, dtype=torch.bfloat16, device=dev)
    layer = 'bench-chunked'
    stream = torch.cuda.current_stream(dev)
    per_chunk = []

    def prefill(record=False):
        ksp._KMEAN_CACHE.clear()
        ksp._SCALE_CACHE.clear()
        ksp._KV8_CACHE.clear()
        flops = 0.0
        for c in range(total // chunk):
            q0 = c * chunk
            qc, kc, vc = q[q0:q0 + chunk], k[:q0 + chunk], v[:q0 + chunk]
            if record:
                a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                a.record(stream)
            km = ksp._cached_block_means(layer, 0, kc[q0:], q0, q0 + chunk)
            scales = ksp._cached_scales(layer, 0, qc, kc, vc, q0)
            kv8 = ksp._cached_kv8(layer, 0, k, v, q0, q0 + chunk, scales) if args.fp8_kv_cache else None
            sp.forward_sm120fp8(qc, kc, vc, q0, out=out, km=km, scales=scales, kv8=kv8)
            if record:
                b.record(stream)
                per_chunk.append((a, b, sp.last_counts.sum()))
    for _ in range(max(1, args.warmup // 3)):
        prefill()
    steps = max(1, min(args.steps, 3))
    ms = _timed(prefill, steps, dev, int(os.environ.get('WORLD_SIZE', '1')))
    prefill(record=True)
    torch.cuda.synchronize(dev)
    chunk_ms = [a.elapsed_time(b) for a, b, _ in per_chunk]
    kept = [int(n.item()) for _, _, n in per_chunk]
    exec_flops = sum(n * 4.0 * D * 128 * 128 for n in kept)
    dense_flops = sum(causal_flops(h, D, chunk, (c + 1) * chunk) for c in range(total // chunk))
    ops.check_status(dev)
    return {'ms': ms, 'steps': steps, 'e2e_ms': None, 'work': exec_flops, 'unit': 'TFLOPS', 'scale': 1e12,
            'kernel': 'attn_fwd_kernel<fp8>', 'kernel_ms': None, 'kernel_work': None, 'bound': 'tensor',
            'h2d': 0, 'd2h': 0, 'launches': 6 * (total // chunk),
            'config': {'workload': f'chunked prefill of {total} tokens in {total // chunk} chunks of {chunk} through '
                                   f'SparsePrefill.forward_sm120fp8, block-mean and scale caches carried; H {h}/Hk {hk}/'
                                   f'D {D}, block {BLOCK}, tau {TAU}; strong injection: sink + local window (4 blocks) '
                                   f'+ 16 hot blocks per KV head; '
                                   + ('FP8 KV cache (each K/V row quantised once)' if args.fp8_kv_cache else
                                      'K/V history re-quantised every chunk (reference behaviour)'),
                       'ms_per_chunk': [round(x, 3) for x in chunk_ms],
                       'kept_fraction_overall': round(exec_flops / dense_flops, 4),
                       'value_definition': 'executed-tile FLOPs (4 D 128 128 per kept 128x128 tile) / prefill time'}}


def _hook(args, h, hk, dev, rank):
    """Config 4 through the vLLM hook: the 262144-token prefill in 32 chunks of 8192, each chunk a
    `try_sparse_forward` call over a paged K/V cache (page 16, pages in shuffled order, fake vLLM
    metadata).  The reference's hook gathers the whole K/V history from the pages every chunk; this
    one reads the pages in place (FP8: the history re-quantised from the pages every chunk, or with
    --fp8-kv-cache only the chunk's own rows; BF16 with --hook-kernel sm120: the attention kernel
    reads the pages itself)."""
    import types
    import torch
    import sm120_attn.sparse_prefill as ksp
    import synth
    from sm120_attn import ops
    ksp.BLOCK = BLOCK
    total, chunk, page = 262144, 8192, 16
    q, k, v, _ = synth.make_qkv(total, total, h, hk, D, block=BLOCK, q_start=0, seed=4000 + rank,
                                strength='strong', hot=16, local=4, device=dev)
    npages = total // page
    perm = torch.randperm(npages + 64, generator=torch.Generator().manual_seed(7))[:npages].to(dev)
    key_cache = torch.empty(npages + 64, page, hk, D, dtype=torch.bfloat16, device=dev)
    value_cache = torch.empty_like(key_cache)
    key_cache[perm.long()] = k.view(npages, page, hk, D)
    value_cache[perm.long()] = v.view(npages, page, hk, D)
    del v
    bt = perm.to(torch.int32).view(1, -1)
    fp8 = args.hook_kernel == 'sm120fp8'
    ksp._CONFIG = {'enabled': True, 'tau': TAU, 'min_kv': 8192, 'min_q': 1024, 'kernel': args.hook_kernel,
                   'fp8_pipeline': 'tma', 'fp8_kv_cache': bool(args.fp8_kv_cache)}
    ksp._STATE.clear()
    impl = types.SimpleNamespace(sliding_window=(-1, -1), scale=D ** -0.5)
    metas = [types.SimpleNamespace(causal=True, max_query_len=chunk, max_seq_len=(c + 1) * chunk,
                                   query_start_loc=torch.tensor([0, chunk], dtype=torch.int32, device=dev),
                                   seq_lens=torch.tensor([(c + 1) * chunk], dtype=torch.int32, device=dev),
                                   block_table=bt) for c in range(total // chunk)]
    out = torch.empty(chunk, h, D, dtype=torch.bfloat16, device=dev)
    stream = torch.cuda.current_stream(dev)
    per_chunk = []

    def prefill(record=False):
        for c, meta in enumerate(metas):
            c0 = c * chunk
            if record:
                a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                a.record(stream)
            ksp.try_sparse_forward(impl, q[c0:c0 + chunk], k[c0:c0 + chunk], key_cache, value_cache, out, meta)
            if record:
                b.record(stream)
                per_chunk.append((a, b, ksp._STATE[next(iter(ksp._STATE))].last_counts.sum()))
    for _ in range(max(1, args.warmup // 3)):
        prefill()
    steps = max(1, min(args.steps, 3))
    ms = _timed(prefill, steps, dev, int(os.environ.get('WORLD_SIZE', '1')))
    prefill(record=True)
    torch.cuda.synchronize(dev)
    chunk_ms = [a.elapsed_time(b) for a, b, _ in per_chunk]
    exec_flops = sum(int(n.item()) * 4.0 * D * 128 * 128 for _, _, n in per_chunk)
    ops.check_status(dev)
    ksp._CONFIG = None
    if fp8:
        how = ('FP8 KV cache: warm chunks read only their own rows' if args.fp8_kv_cache else
               'whole K/V history re-quantised from the pages in place every chunk (the reference gathers it first)')
    else:
        how = 'BF16 attention reading K/V from the pages in place (TMA boxes per page)'
    return {'ms': ms, 'steps': steps, 'e2e_ms': None, 'work': exec_flops, 'unit': 'TFLOPS', 'scale': 1e12,
            'kernel': 'attn_fwd_kernel<fp8>' if fp8 else 'attn_fwd_kernel<bf16>', 'kernel_ms': None,
            'kernel_work': None, 'bound': 'tensor', 'h2d': 0, 'd2h': 0, 'launches': 7 * (total // chunk),
            'dtype': None if fp8 else 'bf16 (fp32 accumulate)',
            'config': {'workload': f'chunked prefill of {total} tokens in {total // chunk} chunks of {chunk} through '
                                   f'the vLLM hook (try_sparse_forward) over a paged K/V cache (page {page}, shuffled '
                                   f'pages); H {h}/Hk {hk}/D {D}, block {BLOCK}, tau {TAU}; C4 injection; ' + how,
                       'ms_per_chunk': [round(x, 3) for x in chunk_ms],
                       'value_definition': 'executed-tile FLOPs / prefill time (host metadata reads included)'}}


def _paged(args, h, hk, dev, rank):
    """BF16 attention over a paged K/V cache read in place (sa_attn_fwd_bf16_paged): the configs[1]
    chunk dense causal (q 8192 @ 57344 vs 65536 keys), pages of --page rows in shuffled order.  Beside
    it (config): the contiguous kernel on the same keys and the gather of the history out of the
    pages that the reference's hook does every chunk."""
    import torch
    from sm120_attn import ops
    q, k, v = make_rank_inputs(hk, 5000 + rank, args.strength, dev)
    page = args.page
    npages = KV // page
    perm = torch.randperm(npages + 64, generator=torch.Generator().manual_seed(7))[:npages].to(dev)
    kc = torch.zeros(npages + 64, page, hk, D, dtype=torch.bfloat16, device=dev)
    vc = torch.zeros_like(kc)
    kc[perm.long()] = k.view(npages, page, hk, D)
    vc[perm.long()] = v.view(npages, page, hk, D)
    table = perm.to(torch.int32)
    out = torch.empty(N_Q, h, D, dtype=torch.bfloat16, device=dev)

    def paged():
        ops.attn_bf16_paged(q, kc, vc, table, out, KV, 0, Q_START, None, None, 64, D ** -0.5)

    def contiguous():
        ops.attn_bf16(q, k, v, out, KV, 0, Q_START, None, None, 64, D ** -0.5)

    def gather():
        return kc[perm.long()].reshape(-1, hk, D), vc[perm.long()].reshape(-1, hk, D)
    for fn in (paged, contiguous, gather):
        for _ in range(args.warmup):
            fn()
    world = int(os.environ.get('WORLD_SIZE', '1'))
    ms = _timed(paged, args.steps, dev, world)
    ms_c = _timed(contiguous, args.steps, dev, world)
    ms_g = _timed(gather, args.steps, dev, world)
    ops.check_status(dev)
    flops = causal_flops(h, D, N_Q, KV)
    return {'ms': ms, 'e2e_ms': None, 'work': flops, 'unit': 'TFLOPS', 'scale': 1e12,
            'kernel': 'attn_fwd_kernel<bf16> (paged)', 'kernel_ms': ms / args.steps, 'kernel_work': flops,
            'bound': 'tensor', 'h2d': 0, 'd2h': 0, 'launches': 1, 'dtype': 'bf16 (fp32 accumulate)',
            'peak_scale': 0.5,
            'config': {'workload': f'dense causal BF16 attention through a paged K/V cache (page {page}, shuffled '
                                   f'pages): q {N_Q} @ {Q_START} vs {KV} keys, H {h}/Hk {hk}/D {D}',
                       'contiguous_ms_per_step': round(ms_c / args.steps, 4),
                       'paged_over_contiguous': round(ms / ms_c, 4),
                       'gather_ms_per_step': round(ms_g / args.steps, 4),
                       'value_definition': 'causal FLOPs / time of the paged kernel'}}


def _decoder_kernels(args, h, hk, dev, rank):
    """The config-5 harness kernels at one 8192-token chunk of the full decoder (1 GPU widths):
    fused residual add + RMSNorm over [8192, 5120], RoPE + K/V cache write of qkv [8192, 80 x 128]
    with the key block means, SwiGLU of gate_up [8192, 2 x 25600].  Inputs are larger than L2 except
    rope's table rows."""
    import torch
    from sm120_attn import ops
    from sm120_attn.decoder import DecoderConfig, rope_table
    cfg = DecoderConfig()
    n, E, D, I = 8192, cfg.hidden, cfg.head_dim, cfg.inter
    Hq, Hkv = cfg.heads, cfg.kv_heads
    g = torch.Generator(device=dev)
    g.manual_seed(rank)
    bf = torch.bfloat16
    hbuf = torch.randn(n, E, generator=g, device=dev).to(bf)
    delta = torch.randn(n, E, generator=g, device=dev).to(bf)
    w = torch.ones(E, dtype=bf, device=dev)
    x = torch.empty(n, E, dtype=bf, device=dev)
    qkv = torch.randn(n, (Hq + 2 * Hkv) * D, generator=g, device=dev).to(bf)
    q = torch.empty(n, Hq, D, dtype=bf, device=dev)
    kc = torch.empty(3 * n, Hkv, D, dtype=bf, device=dev)
    vc = torch.empty_like(kc)
    table = rope_table(3 * n, D, cfg.rope_theta, dev)
    gu = torch.randn(n, 2 * I, generator=g, device=dev).to(bf)
    act = torch.empty(n, I, dtype=bf, device=dev)
    km = torch.empty(Hkv, 3 * n // 128, D, dtype=torch.float32, device=dev)
    # the decoder's RoPE launch also writes the chunk's key block means (sa_rope_qkv_means_bf16)
    kernels = [
        ('add_rmsnorm_kernel', lambda: ops.add_rmsnorm(hbuf, w, x, cfg.eps, delta=delta), 8 * n * E),
        ('rope_qkv_kernel', lambda: ops.rope_qkv(qkv, Hq, Hkv, D, table, 2 * n, q, kc[2 * n:], vc[2 * n:], km=km,
                                                 block=128),
         4 * n * (Hq + 2 * Hkv) * D + 4 * Hkv * (n // 128) * D),
        ('silu_mul_kernel', lambda: ops.silu_mul(gu, act), 6 * n * I),
    ]
    per = {}
    for name, fn, nbytes in kernels:
        for _ in range(3):
            fn()
        per[name] = (_kernel_ms(fn, dev, reps=20), nbytes)
    # the same RoPE write without the means, and the separate block-means pass over the written keys
    unfused = [lambda: ops.rope_qkv(qkv, Hq, Hkv, D, table, 2 * n, q, kc[2 * n:], vc[2 * n:]),
               lambda: ops.block_means(kc[2 * n:], 2 * n, 128, km, 0)]
    for fn in unfused:
        fn()
    unfused_ms = [_kernel_ms(fn, dev, reps=20) for fn in unfused]
    steps = max(1, args.steps)
    ms = _timed(lambda: [fn() for _, fn, _ in kernels], steps, dev, int(os.environ.get('WORLD_SIZE', '1')))
    total = sum(b for _, (_, b) in per.items())
    top = max(per, key=lambda k: per[k][1])
    return {'ms': ms, 'steps': steps, 'e2e_ms': None, 'work': total, 'unit': 'GB/s', 'scale': 1e9,
            'kernel': top, 'kernel_ms': per[top][0], 'kernel_work': per[top][1], 'bound': 'hbm',
            'h2d': 0, 'd2h': 0, 'launches': len(kernels), 'dtype': 'bf16 in/out, fp32 arithmetic',
            'config': {'workload': f'config-5 harness kernels at one {n}-token chunk: add_rmsnorm [{n}, {E}], '
                                   f'rope_qkv [{n}, {Hq}+2x{Hkv} heads x {D}], silu_mul [{n}, 2x{I}]',
                       'per_kernel': {k: {'us': round(t * 1000, 1), 'MB': round(b / 1e6, 1),
                                          'GB/s': round(b / (t * 1e-3) / 1e9, 1)} for k, (t, b) in per.items()},
                       'rope_with_key_means': 'rope_qkv_kernel writes the chunk\'s key block means in the same pass; '
                                              f'unfused: rope {unfused_ms[0] * 1000:.1f} us + block means '
                                              f'{unfused_ms[1] * 1000:.1f} us',
                       'value_definition': 'algorithmic bytes of the three kernels / their time'}}


def measure_ttft(tokens, dev, rank, world, local):
    """Prefill TTFT (s) of the config-5 decoder for one prompt of `tokens` random ids, tensor parallel
    over the ranks of the current process group (the headline line's secondary figure): model built
    from random N(0, 0.02) weights, one untimed 8192-token prefill to warm up, then one timed prefill
    on the device (max over ranks) and one end to end (ids from pinned host memory, first token read
    back)."""
    import torch
    from sm120_attn.decoder import DecoderConfig, TPDecoder
    from sm120_attn.shard import reduce_over_ranks
    cfg = DecoderConfig()
    t_init = time.perf_counter()
    model = TPDecoder(cfg, dev, rank=rank, world=world, group=None, seed=0, tau=TAU, kernel='sm120fp8',
                      fp8_kv_cache=False, max_tokens=tokens, chunk=8192, min_kv=8192, comm_blocks=2)
    torch.cuda.synchronize(dev)
    t_init = time.perf_counter() - t_init
    g = torch.Generator()
    g.manual_seed(0)
    ids_host = torch.randint(0, cfg.vocab, (tokens,), generator=g).pin_memory()
    ids_dev = ids_host.to(dev)
    model.prefill(ids_dev[:min(tokens, 8192)])
    toks = []
    ms = _timed(lambda: toks.append(model.prefill(ids_dev)), 1, dev, world)
    tok_host = torch.empty(1, dtype=torch.int64).pin_memory()

    def e2e():
        tok_host.copy_(model.prefill(ids_host.to(dev, non_blocking=True)).reshape(1), non_blocking=True)
    e2e_ms = _timed(e2e, 1, dev, world)
    kept = float(model.sp.kept_fraction() or 0.0)
    (ms, e2e_ms), _ = reduce_over_ranks([ms, e2e_ms], [0.0], device=dev)
    model.release_caches()
    del model
    torch.cuda.empty_cache()
    return {'tokens': tokens, 'ttft_s': round(ms / 1000.0, 4), 'e2e_ttft_s': round(e2e_ms / 1000.0, 4),
            'first_token': int(toks[-1].item()), 'kept_fraction': round(kept, 4), 'model_init_s': round(t_init, 1),
            'model': f'random-init GQA decoder {cfg.layers} layers, hidden {cfg.hidden}, {cfg.heads}/{cfg.kv_heads} '
                     f'heads, SwiGLU {cfg.inter}, vocab {cfg.vocab}, bf16; 8192-token chunks, sparse FP8 attention '
                     f'tau {TAU}; tensor parallel over {world} GPU(s)',
            'timing': 'device time of one prefill, max over ranks, after one warm-up prefill'}


def run_ttft(args):
    """Config 5: prefill TTFT of the random-init 64-layer GQA decoder (hidden 5120, 64/8 heads, SwiGLU
    25600, vocab 151936) over 65536 / 131072 / 262144 random token ids in 8192-token chunks, sparse
    FP8 attention at tau 0.95, tensor-parallel by KV head over the ranks (NCCL all-reduce after the
    row-parallel projections).  value = TTFT of the 131072-token prompt (benchmark configuration 5)."""
    import torch
    import torch.distributed as dist
    import sm120_attn.sparse_prefill as ksp
    from sm120_attn.decoder import DecoderConfig, TPDecoder
    from sm120_attn.shard import reduce_over_ranks
    world, rank, local, dev = _rank_env()
    contexts = sorted(int(c) for c in args.contexts.split(','))
    headline = 131072 if 131072 in contexts else contexts[-1]
    cfg = DecoderConfig()
    t_init = time.perf_counter()
    model = TPDecoder(cfg, dev, rank=rank, world=world, group=None, seed=0, tau=TAU, kernel='sm120fp8',
                      fp8_kv_cache=args.fp8_kv_cache, max_tokens=contexts[-1], chunk=8192, min_kv=8192,
                      comm_blocks=args.comm_blocks)
    torch.cuda.synchronize(dev)
    t_init = time.perf_counter() - t_init
    g = torch.Generator()
    g.manual_seed(0)
    ids_host = torch.randint(0, cfg.vocab, (contexts[-1],), generator=g).pin_memory()
    ids_dev = ids_host.to(dev)
    for _ in range(args.warmup):                              # warm-up prefills of the shortest prompt
        model.prefill(ids_dev[:contexts[0]])
    steps = 1                                                 # one prefill per prompt length
    ttft, kept, first_tok, attn_ms, attn_flops = {}, {}, {}, 0.0, 0.0
    clocks = Clocks(local)
    clocks.start()
    for T in contexts:
        events = [] if T == headline else None
        model.sp.kernel_events = events
        model.sp._kept_acc = None
        model.sp.stats['blocks_total'] = 0
        toks = []
        ms = _timed(lambda: toks.append(model.prefill(ids_dev[:T])), steps, dev, world)
        model.sp.kernel_events = None
        kept_units = float(model.sp._kept_acc.item()) / steps
        kept[T] = round(float(model.sp.kept_fraction()), 4)
        if events is not None:
            attn_ms = sum(a.elapsed_time(b) for a, b in events) / steps
            attn_flops = kept_units * 4.0 * cfg.head_dim * ksp.BLOCK * ksp.BLOCK
        first_tok[T] = int(toks[-1].item())
        ttft[T] = ms / steps
    # end to end: ids from pinned host memory, first token read back, inside the timed region
    tok_host = torch.empty(1, dtype=torch.int64).pin_memory()

    def e2e():
        ids = ids_host[:headline].to(dev, non_blocking=True)
        tok_host.copy_(model.prefill(ids).reshape(1), non_blocking=True)
    e2e_ms = _timed(e2e, 1, dev, world)
    clk = clocks.stop()
    keys = list(contexts)
    vals, (flops_sum,) = reduce_over_ranks([ttft[T] for T in keys] + [e2e_ms, attn_ms], [attn_flops], device=dev)
    ttft = dict(zip(keys, vals[:len(keys)]))
    e2e_ms, attn_ms = vals[len(keys)], vals[len(keys) + 1]
    hbm, bf16, how = peaks()
    gemm_flops = cfg.prefill_flops(headline)
    chunks = -(-headline // 8192)
    # per layer and chunk: add_rmsnorm + rope + 7 on the attention path, then add_rmsnorm + silu per
    # communication block; 3 absmax per layer on the first chunk; the final add_rmsnorm
    launches = cfg.layers * ((9 + 2 * model.comm_blocks) * chunks + 3) + 1
    line = {
        'metric': METRIC, 'value': round(ttft[headline] / 1000.0, 4), 'unit': 's', 'n_gpus': world, 'steps': steps,
        'warmup': args.warmup, 'ms_per_step': round(ttft[headline], 2), 'higher_is_better': False,
        'scaling': 'strong', 'vs_baseline': None,
        'dtype': 'bf16 GEMMs (cuBLAS), fp8-e4m3 attention (fp32 accumulate), bf16 activations',
        'data': 'synthetic: random N(0, 0.02) bf16 weights, seeded random token ids',
        'config': {'workload': f'C5 prefill TTFT: random-init dense GQA decoder, {cfg.layers} layers, hidden '
                               f'{cfg.hidden}, {cfg.heads}/{cfg.kv_heads} heads, head_dim {cfg.head_dim}, SwiGLU '
                               f'{cfg.inter}, vocab {cfg.vocab}; 8192-token chunks, sparse FP8 attention tau {TAU} '
                               f'(block {ksp.BLOCK}); value = TTFT of the {headline}-token prompt',
                   'ttft_s': {str(T): round(ttft[T] / 1000.0, 4) for T in keys},
                   'kept_fraction': {str(T): kept[T] for T in keys},
                   'first_token': {str(T): first_tok[T] for T in keys}, 'fp8_kv_cache': bool(args.fp8_kv_cache),
                   'parallelism': f'tensor parallel by KV head x{world} (NCCL all-reduce after o_proj and '
                                  f'down_proj in {model.comm_blocks} row block(s), each overlapping the next '
                                  f'block\'s GEMMs; all-gather of the last-token logits)',
                   'gemm_tflops_per_gpu': round(gemm_flops / world / (ttft[headline] * 1e-3) / 1e12, 1),
                   'attention_ms_of_ttft': round(attn_ms, 1), 'model_init_s': round(t_init, 1),
                   'params': cfg.params(), 'l2': 'inputs larger than L2; no flush'},
    }
    if attn_ms > 0:
        ach = flops_sum / world / (attn_ms * 1e-3) / 1e12
        line['roofline'] = {'bound': 'tensor', 'kernel': 'attn_fwd_kernel<fp8> (all launches of the prefill)',
                            'achieved': round(ach, 1), 'peak': round(2 * bf16, 1), 'unit': 'TFLOP/s',
                            'frac': round(ach / (2 * bf16), 4), 'traffic': None,
                            'peak_source': f'{how} (MEASURED_PEAKS.json) x2 for e4m3'}
    line['e2e'] = {'value': round(e2e_ms / 1000.0, 4), 'unit': 's', 'h2d_bytes_per_step': headline * 8,
                   'd2h_bytes_per_step': 8}
    line['gpu_launches'] = launches * steps
    line['clocks'] = clk
    if rank == 0:
        print(json.dumps(line), flush=True)
    model.release_caches()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def run_other(args):
    global PROFILE_RANGE
    from sm120_attn.shard import kv_head_range, reduce_over_ranks
    import torch.distributed as dist
    world, rank, local, dev = _rank_env()
    PROFILE_RANGE = args.profile_range
    if args.scaling == 'strong':
        try:
            lo, hi = kv_head_range(rank, world, HK_FULL)
        except ValueError as e:
            raise SystemExit(f'strong scaling: {e}')
        hk = hi - lo
    else:
        hk = HK_FULL
    if args.rank_shape > 1 and world == 1:
        hk = rank_shape_kv_heads(args.rank_shape)
    h = hk * (H_FULL // HK_FULL)
    clocks = Clocks(local)
    clocks.start()
    res = {'dense': _dense, 'selection': _selection, 'chunked': _chunked, 'hook': _hook, 'paged': _paged,
           'decoder_kernels': _decoder_kernels}[args.workload](
        args, h, hk, dev, rank)
    clk = clocks.stop()
    steps = res.get('steps', args.steps)
    e2e_ms = res['e2e_ms'] if res['e2e_ms'] is not None else res['ms']
    kms = res['kernel_ms'] if res['kernel_ms'] is not None else 0.0
    (ms, e2e_ms, kms), (work,) = reduce_over_ranks([res['ms'], e2e_ms, kms], [res['work']], device=dev)
    hbm, bf16, how = peaks()
    value = work * steps / (ms * 1e-3) / res['scale']
    line = {
        'metric': METRIC, 'value': round(value, 2), 'unit': res['unit'], 'n_gpus': world, 'steps': steps,
        'warmup': args.warmup, 'ms_per_step': round(ms / steps, 4), 'higher_is_better': True,
        'scaling': args.scaling, 'vs_baseline': None,
        'dtype': res.get('dtype') or ('fp8-e4m3 (fp32 accumulate, bf16 in/out)' if res['unit'] == 'TFLOPS'
                                      else 'bf16 in, fp32 scores, int32 CSR'),
        'data': 'synthetic (seeded, benchmark shapes and injection)', 'config': dict(res['config']),
    }
    line['config']['parallelism'] = f'kv-head shards x{world} ({args.scaling}), no collective on the data path'
    line['config']['l2'] = 'inputs larger than L2; no flush'
    if res['kernel_work'] is not None and kms > 0:
        ach = res['kernel_work'] / (kms * 1e-3) / res['scale']
        peak = 2.0 * bf16 * res.get('peak_scale', 1.0) if res['bound'] == 'tensor' else hbm
        line['roofline'] = {'bound': res['bound'], 'kernel': res['kernel'], 'achieved': round(ach, 1),
                            'peak': round(peak, 1), 'unit': 'TFLOP/s' if res['bound'] == 'tensor' else 'GB/s',
                            'frac': round(ach / peak, 4), 'traffic': None,
                            'peak_source': f'{how} (MEASURED_PEAKS.json)' + (
                                ' x2 for e4m3' if res['bound'] == 'tensor' and res.get('peak_scale', 1.0) == 1.0
                                else ' bf16' if res['bound'] == 'tensor' else '')}
    if res['e2e_ms'] is not None:
        line['e2e'] = {'value': round(work * steps / (e2e_ms * 1e-3) / res['scale'], 2), 'unit': res['unit'],
                       'h2d_bytes_per_step': res['h2d'], 'd2h_bytes_per_step': res['d2h'],
                       'ms_per_step': round(e2e_ms / steps, 4)}
    line['gpu_launches'] = res['launches'] * steps
    line['clocks'] = clk
    if rank == 0:
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def cpu_sample(strength, seconds_budget=20.0):
    """Reference algorithm on the host (oracle/, numpy): selection + masked fp32 attention of the
    last `rows` query rows of one KV-head group of the workload; returns (TFLOPS, description, threads)."""
    import numpy as np
    import torch
    import oracle as O
    import synth
    torch.manual_seed(0)
    hk, g = 1, H_FULL // HK_FULL
    q, k, v, _ = synth.make_qkv(N_Q, KV, g * hk, hk, D, block=BLOCK, q_start=Q_START, seed=1000, strength=strength,
                                hot=6)
    qf, kf, vf = (t.float().numpy() for t in (q, k, v))
    t_start = time.perf_counter()
    kc = O.KMeanCacheOracle(BLOCK)
    kc.update('cpu', 0, kf[:Q_START], 0, Q_START)
    km = kc.update('cpu', 0, kf[Q_START:], Q_START, KV)
    qm = O.q_block_means(qf, Q_START, BLOCK)
    masks = O.select_masks(qm, km, Q_START, BLOCK, g * hk, hk, TAU)
    t_sel = time.perf_counter() - t_start
    rows = 256
    done_rows, flops, t_attn = 0, 0.0, 0.0
    n_blocks = N_Q // BLOCK
    m = n_blocks - 1
    while m >= 0 and t_attn < seconds_budget:
        r0 = m * BLOCK
        t0 = time.perf_counter()
        O.attention_ref_threaded(qf[r0:r0 + BLOCK], kf, vf, Q_START + r0, masks[:, m:m + 1], q_block=BLOCK,
                                 kv_block=BLOCK)
        t_attn += time.perf_counter() - t0
        kept = masks[:, m].sum()
        flops += 4.0 * D * BLOCK * BLOCK * kept
        done_rows += BLOCK
        m -= 1
        if done_rows >= rows and t_attn > 2.0:
            break
    tflops = flops / (t_attn + t_sel * done_rows / N_Q) / 1e12
    threads = torch.get_num_threads()
    desc = (f'oracle: selection (numpy fp32) of 1 KV head x 8 query heads over the full chunk ({t_sel:.2f} s) + '
            f'masked fp32 attention of the last {done_rows} query rows x 8 heads on all intra-op threads '
            f'(attention_ref_threaded, the arithmetic of the reference\'s reference(); {t_attn:.2f} s); selection '
            f'time pro-rated to the sampled rows')
    return tflops, desc, threads


def cpu_baseline(strength):
    import torch
    torch.set_num_threads(os.cpu_count() or 1)                 # all host threads (rank 0 at N = 1)
    val, desc, threads = cpu_sample(strength)
    return {'value': round(val, 6), 'unit': 'TFLOPS', 'cores': os.cpu_count(), 'threads': threads, 'kind': 'port',
            'sample': desc}


def cpu_selection_sample(strength):
    """The selection path of the `selection` workload on the host cores with the oracle (numpy): K-chunk
    block means appended to a cache holding the history, Q pooling, per-head tau selection, at the full
    shape; returns (GB/s of the same algorithmic bytes as the GPU arm, description, threads)."""
    import numpy as np
    import torch
    import oracle as O
    import synth
    q, k, _, _ = synth.make_qkv(N_Q, KV, H_FULL, HK_FULL, D, block=BLOCK, q_start=Q_START, seed=3000,
                                strength=strength, hot=6, with_v=False)
    qf, kf = q.float().numpy(), k.float().numpy()
    kc = O.KMeanCacheOracle(BLOCK)
    kc.update('cpu-sel', 0, kf[:Q_START], 0, Q_START)
    t0 = time.perf_counter()
    km = kc.update('cpu-sel', 0, kf[Q_START:], Q_START, KV)
    qm = O.q_block_means(qf, Q_START, BLOCK)
    masks = O.select_masks(qm, km, Q_START, BLOCK, H_FULL, HK_FULL, TAU)
    sec = time.perf_counter() - t0
    MB, NB = N_Q // BLOCK, KV // BLOCK
    nnz = int(masks.sum())
    nbytes = 2 * N_Q * H_FULL * D + 2 * N_Q * HK_FULL * D + 4 * HK_FULL * NB * D + 4 * HK_FULL * MB * D + \
        4 * (H_FULL * MB + 1) + 4 * nnz
    desc = (f'oracle (numpy) selection path of the whole chunk: K-chunk means, Q pooling, tau selection of '
            f'{H_FULL * MB} rows over {NB} blocks ({sec:.2f} s)')
    return nbytes / sec / 1e9, desc, torch.get_num_threads()


def run_reference(args):
    rank = int(os.environ.get('RANK', '0'))
    world = int(os.environ.get('WORLD_SIZE', '1'))
    if rank != 0:
        return
    if args.workload not in ('chunk', 'selection'):
        print(json.dumps({'impl': 'reference', 'unavailable': f'no CPU arm for the {args.workload} workload: the '
                          'reference CPU path is timed for the default (chunk) and selection workloads'}), flush=True)
        return
    import torch
    # torchrun sets OMP_NUM_THREADS=1 for every rank; rank 0 alone runs this arm and uses all host threads
    torch.set_num_threads(os.cpu_count() or 1)
    sample = cpu_sample if args.workload == 'chunk' else (lambda st, seconds_budget=0: cpu_selection_sample(st))
    unit = 'TFLOPS' if args.workload == 'chunk' else 'GB/s'
    # every one of the K timed steps is a bounded sample of the workload, sized so that the whole
    # run (W + K samples) stays within about 150 s of host time
    budget = max(1.0, min(10.0, 150.0 / max(1, args.steps + args.warmup)))
    vals = []
    desc, threads = '', 0
    for _ in range(max(0, args.warmup)):                       # untimed samples (BLAS threads, caches)
        sample(args.strength, seconds_budget=min(budget, 2.0))
    for _ in range(max(1, args.steps)):
        v, desc, threads = sample(args.strength, seconds_budget=budget)
        vals.append(v)
    value = sum(vals) / len(vals)
    base = chunk_config(args, world) if args.workload == 'chunk' else selection_config(args, H_FULL, HK_FULL)
    line = {
        'metric': METRIC, 'value': round(value, 6), 'unit': unit, 'impl': 'reference', 'n_gpus': world,
        'steps': len(vals), 'warmup': max(0, args.warmup), 'higher_is_better': True, 'scaling': args.scaling,
        'vs_baseline': None, 'dtype': 'fp32', 'data': 'synthetic (seeded, same workload as the b200 arm)',
        'config': base,
        'cpu_baseline': {'value': round(value, 6), 'unit': unit, 'cores': os.cpu_count(), 'threads': threads,
                         'kind': 'port', 'sample': desc,
                         'arm': 'host cores of rank 0, all threads (the other ranks exit); the reference algorithm '
                                'restated in oracle/ (selection in numpy, attention with the fp32 arithmetic of the '
                                'reference\'s reference() on all intra-op threads); the reference checkout itself '
                                'does not travel to the GPU host'},
        'e2e': {'value': round(value, 6), 'unit': unit, 'h2d_bytes_per_step': 0, 'd2h_bytes_per_step': 0},
    }
    print(json.dumps(line), flush=True)


def chunk_config(args, world):
    """`config` of the default (chunk) workload, shared by both arms."""
    shape = (f'; one GPU running the per-rank share of a {args.rank_shape}-GPU strong split'
             if args.rank_shape > 1 and world == 1 else '')
    return {'workload': f'sparse FP8 prefill chunk (configs[1] shape): q {N_Q} @ {Q_START} vs {KV} keys, '
                        f'H {H_FULL}/Hk {HK_FULL}/D {D}, block {BLOCK}, tau {TAU}, {args.strength} injection' + shape,
            'global_batch': 1, 'seq_len': KV, 'chunk': N_Q,
            'parallelism': f'kv-head shards x{world} ({args.scaling}), no collective on the data path'}


def selection_config(args, h, hk):
    return {'workload': f'selection path (configs[1] shape): K-chunk means into the cache, Q pooling, '
                        f'per-head selection to CSR; q {N_Q} @ {Q_START} vs {KV} keys, H {h}/Hk {hk}/D {D}, '
                        f'block {BLOCK}, tau {TAU}, {args.strength} injection'}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument('--gpus', type=int, default=1)
    ap.add_argument('--steps', type=int, default=20)
    ap.add_argument('--warmup', type=int, default=3)
    ap.add_argument('--impl', default='b200', choices=['b200', 'reference'])
    ap.add_argument('--scaling', default='strong', choices=['weak', 'strong'],
                    help='strong (default): the 8 KV heads of one problem split over the GPUs; weak: every GPU '
                         'runs a whole 8-KV-head problem')
    ap.add_argument('--strength', default='unit', choices=['unit', 'strong'])
    ap.add_argument('--no-cpu-baseline', action='store_true')
    ap.add_argument('--profile-range', action='store_true',
                    help='bracket the timed steps with cudaProfilerStart/Stop (ncu --profile-from-start off)')
    ap.add_argument('--workload', default='chunk',
                    choices=['chunk', 'dense', 'selection', 'chunked', 'hook', 'paged', 'ttft', 'decoder_kernels'])
    ap.add_argument('--page', type=int, default=16, help='paged workload: rows per page of the K/V cache')
    ap.add_argument('--rank-shape', type=int, default=1,
                    help='one GPU runs the per-rank share of an N-GPU strong split (8/N KV heads and their '
                         'query heads), e.g. to measure the last-wave split walks of 8-GPU ranks')
    ap.add_argument('--comm-blocks', type=int, default=2,
                    help='ttft workload: row blocks whose all-reduces overlap the next block\'s GEMMs (1: none)')
    ap.add_argument('--contexts', default='65536,131072,262144',
                    help='ttft workload: prompt lengths (the 131072 one is the reported value)')
    ap.add_argument('--ttft-tokens', type=int, default=65536,
                    help='default workload: also time the prefill TTFT of the config-5 decoder for a prompt of '
                         'this many tokens (config.ttft; 0 skips it)')
    ap.add_argument('--fp8-kv-cache', action='store_true',
                    help='chunked / hook workloads: keep e4m3 K/V across chunks (SM120_SPARSE_FP8_KV_CACHE)')
    ap.add_argument('--hook-kernel', default='sm120fp8', choices=['sm120fp8', 'sm120'],
                    help='hook workload: the FP8 kernel (default) or the BF16 kernel reading the pages in place')
    ap.add_argument('--no-also', action='store_true',
                    help='default workload: skip the secondary figures (strong injection, dense, selection)')
    args = ap.parse_args()
    if args.warmup < 3 and args.impl == 'b200':
        print('note: warmup raised to 3', file=sys.stderr)
        args.warmup = 3
    if args.impl == 'reference' and args.workload == 'ttft':
        if int(os.environ.get('RANK', '0')) == 0:
            print(json.dumps({'impl': 'reference', 'unavailable': 'config 5 (TTFT) has no CPU path in the reference: '
                              'it is measured through a vLLM server on the GPU'}), flush=True)
    elif args.impl == 'reference':
        run_reference(args)
    elif args.workload == 'ttft':
        run_ttft(args)
    elif args.workload == 'chunk':
        run_b200(args)
    else:
        run_other(args)


if __name__ == '__main__':
    main()
