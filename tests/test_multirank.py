"""N>1 path on the CPU: two gloo ranks, each owning half of the KV heads (and their query heads).

Checks that the sharded run needs no data exchange - each rank's block selection and attention on
its own heads, gathered, equal the unsharded problem bit for bit - and that the measurement
reduction (max of times, sum of work) is what the benchmark reports.
"""
import socket

import pytest

from sm120_attn.shard import head_ranges, kv_head_range


def test_kv_head_ranges_partition():
    for world in (1, 2, 4, 8):
        got = [kv_head_range(r, world, 8) for r in range(world)]
        assert got[0][0] == 0 and got[-1][1] == 8
        assert all(a[1] == b[0] for a, b in zip(got, got[1:]))
        assert head_ranges(world - 1, world, 64, 8)[0] == (64 - 64 // world, 64)
    with pytest.raises(ValueError):
        kv_head_range(0, 3, 8)
    with pytest.raises(ValueError):
        kv_head_range(2, 2, 8)


def _free_port():
    with socket.socket(socket.AF_INET, socket.SOCK_STREAM) as s:
        s.bind(('127.0.0.1', 0))
        return s.getsockname()[1]


def test_two_rank_kv_head_shards_match_unsharded(tmp_path):
    import torch.multiprocessing as mp
    import multirank_worker
    world = 2
    mp.start_processes(multirank_worker.run, args=(world, _free_port(), str(tmp_path)), nprocs=world,
                       start_method='spawn', join=True)
    assert sorted(p.name for p in tmp_path.iterdir()) == [f'ok{r}' for r in range(world)]


def test_two_rank_glue_shards_match_unsharded(tmp_path):
    """The product's host glue (block-mean cache, scale cache, block_masks) run per KV-head shard on two
    gloo ranks reproduces the unsharded run."""
    import torch.multiprocessing as mp
    import multirank_worker
    world = 2
    mp.start_processes(multirank_worker.run_glue, args=(world, _free_port(), str(tmp_path)), nprocs=world,
                       start_method='spawn', join=True)
    assert sorted(p.name for p in tmp_path.iterdir()) == [f'ok{r}' for r in range(world)]


def test_two_rank_tp_decoder_matches_unsharded(tmp_path):
    """The C5 decoder's tensor-parallel split (KV-head / intermediate / vocabulary slices, all-reduce
    after the row-parallel projections) reproduces the unsharded model on two gloo ranks."""
    import torch.multiprocessing as mp
    import multirank_worker
    world = 2
    mp.start_processes(multirank_worker.run_tp_decoder, args=(world, _free_port(), str(tmp_path)), nprocs=world,
                       start_method='spawn', join=True)
    assert sorted(p.name for p in tmp_path.iterdir()) == [f'ok{r}' for r in range(world)]


def test_decoder_shards_partition():
    from sm120_attn.decoder import DecoderConfig, shard
    cfg = DecoderConfig()
    for world in (1, 2, 4, 8):
        got = [shard(cfg, r, world) for r in range(world)]
        for field, total in (('q_heads', 64), ('kv_heads', 8), ('inter', 25600), ('vocab', 151936)):
            spans = [getattr(s, field) for s in got]
            assert spans[0][0] == 0 and spans[-1][1] == total
            assert all(a[1] == b[0] for a, b in zip(spans, spans[1:]))
    with pytest.raises(ValueError):
        shard(cfg, 0, 3)
