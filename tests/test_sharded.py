"""CPU: the multi-GPU control logic with gloo ranks (world size 2): shard ranges and image offsets, identical
per-iteration control on every rank, the loss all-gather, and failure detection (a rank that never joins makes the
others' collective fail within the process-group timeout instead of hanging)."""
import datetime
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from ultranca_b200.sharded import ControlChannel, RolloutLengths, shard_range


def free_port():
    with socket.socket() as s:
        s.bind(('127.0.0.1', 0))
        return s.getsockname()[1]


def test_shard_ranges_cover_all_ncas():
    for K in (1, 7, 32, 256, 512):
        for world in (1, 2, 3, 4, 8):
            ranges = [shard_range(K, world, r) for r in range(world)]
            assert ranges[0][0] == 0 and ranges[-1][1] == K
            assert all(a[1] == b[0] for a, b in zip(ranges, ranges[1:]))
            assert max(b - a for a, b in ranges) - min(b - a for a, b in ranges) <= 1
    with pytest.raises(ValueError):
        shard_range(8, 2, 2)


def _worker(rank, world, port, out, mode):
    os.environ['MASTER_ADDR'] = '127.0.0.1'
    os.environ['MASTER_PORT'] = str(port)
    dist.init_process_group('gloo', rank=rank, world_size=world, timeout=datetime.timedelta(seconds=5))
    try:
        ch = ControlChannel((32, 96), seed=123)
        if mode == 'control':
            seq = [ch.next() for _ in range(5)]
            k0, k1 = shard_range(8, world, rank)
            losses = torch.arange(k0, k1, dtype=torch.float32) * 10
            out[rank] = (seq, ch.gather_losses(losses).tolist())
        elif mode == 'uneven':
            # K = 7 over 2 ranks: shards of 3 and 4 NCAs; the gather pads to 4 and trims
            K = 7
            ch = ControlChannel((32, 96), seed=123, K=K)
            k0, k1 = shard_range(K, world, rank)
            first = ch.gather_losses(torch.arange(k0, k1, dtype=torch.float32) + 0.5).tolist()
            second = ch.gather_losses(torch.arange(k0, k1, dtype=torch.float32) * -2).tolist()
            try:  # a rank whose loss count contradicts its shard is refused before the collective
                ch.gather_losses(torch.zeros(k1 - k0 + 1))
                refused = False
            except ValueError:
                refused = True
            out[rank] = (first, second, refused)
        elif mode == 'lengths':
            rl = RolloutLengths((32, 96), seed=9)
            out[rank] = [rl.next() for _ in range(6)]
        elif mode == 'dead_peer':
            if rank == 1:
                return  # leaves without joining the broadcast
            try:
                ch.next()
                ch.next()
                out[rank] = 'no error'
            except Exception as e:  # the collective must fail, not hang
                out[rank] = f'error: {type(e).__name__}'
    finally:
        if mode in ('control', 'uneven', 'lengths'):
            dist.destroy_process_group()


def _run(mode, world=2):
    port = free_port()
    ctx = mp.get_context('spawn')
    out = ctx.Manager().dict()
    procs = [ctx.Process(target=_worker, args=(r, world, port, out, mode)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(60)
        if p.is_alive():
            p.kill()
            pytest.fail(f'{mode}: rank process did not finish')
    return dict(out)


def test_control_broadcast_and_loss_gather():
    out = _run('control')
    seq0, losses0 = out[0]
    seq1, losses1 = out[1]
    assert seq0 == seq1  # identical (rollout length, seed) on every rank
    assert all(32 <= n < 96 for n, _ in seq0) and len({s for _, s in seq0}) == 5
    assert losses0 == losses1 == [0.0, 10.0, 20.0, 30.0, 40.0, 50.0, 60.0, 70.0]


def test_dead_peer_fails_fast():
    out = _run('dead_peer')
    assert out[0].startswith('error'), out


def test_uneven_shards_gather_in_nca_order():
    """K not divisible by the world size (7 NCAs on 2 ranks): every rank receives all 7 losses in NCA order, twice in
    a row (no stale padding), and a loss count that contradicts the rank's shard is refused."""
    out = _run('uneven')
    for r in (0, 1):
        first, second, refused = out[r]
        assert first == [k + 0.5 for k in range(7)]
        assert second == [-2.0 * k for k in range(7)]
        assert refused


def test_rollout_lengths_identical_on_every_rank():
    out = _run('lengths')
    assert out[0] == out[1]
    assert all(32 <= n < 96 for n in out[0]) and len(set(out[0])) > 1
