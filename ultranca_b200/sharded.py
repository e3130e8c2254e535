"""K-sharded multi-GPU training of a group of NCAs: one process per GPU, no data-path collective.

The K NCAs are independent except for the shared rollout length of an iteration (the reference's group loop draws one
length per iteration for the whole group, train.py:133). Rank r of N owns NCAs shard_range(K, N, r): their weights,
Adam state, pool and targets. Rank 0 draws the rollout length of each iteration and broadcasts it; the step seeds are
identical on every rank and every kernel takes the shard's global image offset, so a rank's update masks are exactly
the single-GPU masks of its NCAs. Per-NCA losses are all-gathered for logging (train.py:213-217 keeps the mean of the
last 32 per NCA). Shards may differ by one NCA (K not divisible by N): the gather pads every rank's losses to the
largest shard and trims the padding. The backend is NCCL on GPUs and gloo for the CPU tests of this control logic.

ShardedTrainer: host-driven iterations (RolloutTrainer), with (rollout length, base seed) broadcast per iteration.
ShardedPoolTrainer: the device-driven group loop (PoolTrainer, one CUDA graph replay per iteration) that bench.py
measures: the control block's key is broadcast once and every rank derives the same rollout seeds from it on the
device; the rollout length of iteration i + 1 is broadcast while iteration i runs.
"""
import numpy as np
import torch
import torch.distributed as dist


def shard_range(K, world, rank):
    """NCAs [k0, k1) of `rank`: contiguous, sizes differ by at most one."""
    if not 0 <= rank < world:
        raise ValueError(f'rank {rank} outside world of {world}')
    return K * rank // world, K * (rank + 1) // world


class ControlChannel:
    """Rank 0's per-iteration control (rollout length, base seed), broadcast to every rank, and the loss all-gather.

    rollout: [low, high) rollout lengths (train.py:133 draws np.random.randint(low, high)); seed: rank 0's generator
    seed. device: where the collective tensors live ('cuda' for NCCL, 'cpu' for gloo)."""

    def __init__(self, rollout=(32, 96), seed=0, device='cpu', group=None, K=None):
        self.K = K  # NCAs of the whole group (None: every rank holds the same number)
        self.low, self.high = rollout
        self.rng = np.random.default_rng(seed)
        self.device = torch.device(device)
        self.group = group
        self.buf = torch.zeros(2, dtype=torch.int64, device=self.device)
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0

    def next(self):
        """-> (rollout length, base seed), identical on every rank."""
        if self.rank == 0:
            length = int(self.rng.integers(self.low, self.high)) if self.high > self.low else int(self.low)
            seed = int(self.rng.integers(0, 2 ** 62))
            self.buf.copy_(torch.tensor([length, seed], dtype=torch.int64))
        if self.world > 1:
            dist.broadcast(self.buf, 0, group=self.group)
        return int(self.buf[0]), int(self.buf[1])

    def gather_losses(self, losses):
        """This rank's per-NCA losses (k1 - k0,) -> all ranks' losses concatenated in NCA order. Shards of different
        sizes (K not divisible by the world size) need the group's K at construction: every rank then sends a buffer of
        the largest shard's size (a collective with equal counts everywhere) and the padding is dropped."""
        if self.world == 1:
            return losses
        K = self.K if self.K is not None else self.world * losses.numel()
        k0, k1 = shard_range(K, self.world, self.rank)
        if losses.numel() != k1 - k0:
            raise ValueError(f'rank {self.rank} holds {losses.numel()} losses, its shard of K={K} has {k1 - k0} '
                             '(give ControlChannel the group\'s K when shards differ in size)')
        per = -(-K // self.world)
        buf = torch.zeros(per, dtype=losses.dtype, device=losses.device)
        buf[:k1 - k0] = losses.reshape(-1)
        out = torch.empty(self.world * per, dtype=losses.dtype, device=losses.device)
        dist.all_gather_into_tensor(out, buf, group=self.group)
        parts = []
        for r in range(self.world):
            a, b = shard_range(K, self.world, r)
            parts.append(out[r * per:r * per + (b - a)])
        return torch.cat(parts)


class RolloutLengths:
    """Rank 0 draws each iteration's rollout length from [low, high) (train.py:133) and broadcasts it. The length of
    the next iteration is requested as soon as the current one is taken, on a side stream when the tensors live on a
    GPU, so that reading it on the host never waits for the step kernels of the iteration in flight."""

    def __init__(self, rollout=(32, 96), seed=0, device='cpu', group=None):
        self.low, self.high = rollout
        self.rng = np.random.default_rng(seed)
        self.device = torch.device(device)
        self.group = group
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        cuda = self.device.type == 'cuda'
        self.buf = torch.zeros(1, dtype=torch.int64, device=self.device)
        self.host = torch.zeros(1, dtype=torch.int64).pin_memory() if cuda else torch.zeros(1, dtype=torch.int64)
        self.side = torch.cuda.Stream(self.device) if cuda else None
        self.ready = torch.cuda.Event() if cuda else None
        self._request()

    def _draw(self):
        return int(self.rng.integers(self.low, self.high)) if self.high > self.low else int(self.low)

    def _request(self):
        if self.side is None:
            if self.rank == 0:
                self.buf.fill_(self._draw())
            if self.world > 1:
                dist.broadcast(self.buf, 0, group=self.group)
            self.host.copy_(self.buf)
            return
        with torch.cuda.stream(self.side):
            if self.rank == 0:
                self.buf.fill_(self._draw())
            if self.world > 1:
                dist.broadcast(self.buf, 0, group=self.group)
            self.host.copy_(self.buf, non_blocking=True)
            self.ready.record(self.side)

    def next(self):
        """-> this iteration's rollout length (the same on every rank); requests the next one."""
        if self.ready is not None:
            self.ready.synchronize()
        n = int(self.host[0])
        self._request()
        return n


class ShardedTrainer:
    """This rank's share of a group: RolloutTrainer over its NCAs + the control channel. `w1, b1, w2` are this shard's
    weights (K/N of them); rollouts up to `max_steps` steps."""

    def __init__(self, w1, b1, w2, B, H, W, max_steps, k0, rollout=(32, 96), control_seed=0, K=None, **trainer_kw):
        from .training import RolloutTrainer
        world = dist.get_world_size() if dist.is_initialized() else 1
        rank = dist.get_rank() if dist.is_initialized() else 0
        K = K if K is not None else w1.shape[0] * world
        if (k0, k0 + w1.shape[0]) != shard_range(K, world, rank):
            raise ValueError(f'rank {rank} holds NCAs [{k0}, {k0 + w1.shape[0]}), its shard of K={K} is '
                             f'{shard_range(K, world, rank)}')
        self.trainer = RolloutTrainer(w1, b1, w2, B, H, W, max_steps, image_offset=k0 * B, **trainer_kw)
        dev = 'cuda' if dist.is_initialized() and dist.get_backend() == 'nccl' else 'cpu'
        self.control = ControlChannel(rollout, control_seed, device=dev, K=K)

    def iteration(self, x0, target):
        steps, seed = self.control.next()
        loss, xT = self.trainer.iteration(x0, target, seed, steps=steps)
        return self.control.gather_losses(loss), xT, steps


class ShardedPoolTrainer:
    """This rank's share of a group, driven from the device (training.PoolTrainer: pool sample with seed injection,
    rollout, loss, backward, fused reduce + Adam, pool write-back, one CUDA graph replay per iteration). w1, b1, w2,
    pool (K_r, P, C, H, W) and target are this shard's (NCAs shard_range(K, world, rank)); K is the group's size."""

    def __init__(self, w1, b1, w2, pool, target, B, H, W, max_steps, K, rollout=(32, 96), control_seed=0, key=0,
                 inject_every=16, seed_kind=0, timed=0, graph=True, **trainer_kw):
        from .training import PoolTrainer, RolloutTrainer
        self.world = dist.get_world_size() if dist.is_initialized() else 1
        self.rank = dist.get_rank() if dist.is_initialized() else 0
        k0, k1 = shard_range(K, self.world, self.rank)
        if w1.shape[0] != k1 - k0:
            raise ValueError(f'rank {self.rank} holds {w1.shape[0]} NCAs, its shard of K={K} is [{k0}, {k1})')
        self.K, self.k0 = K, k0
        dev = w1.device
        self.trainer = RolloutTrainer(w1, b1, w2, B, H, W, max_steps, image_offset=k0 * B, **trainer_kw)
        keybuf = torch.tensor([int(key) - (1 << 64) if int(key) >= (1 << 63) else int(key)], dtype=torch.int64,
                              device=dev)
        if self.world > 1:  # one key for every rank: the same rollout seeds everywhere
            dist.broadcast(keybuf, 0)
        self.loop = PoolTrainer(self.trainer, pool, target, inject_every=inject_every,
                                seed_kind=seed_kind, key=int(keybuf.item()) % (1 << 64),
                                graph=graph, timed=timed, nca_offset=k0)
        self.lengths = RolloutLengths(rollout, control_seed, device=dev)
        self.control = ControlChannel(rollout, control_seed, device=dev, K=K)

    def iteration(self):
        """One iteration of the group; returns every rank's per-NCA losses in NCA order (device tensor)."""
        n = self.lengths.next()
        loss = self.loop.iteration(n)
        return self.control.gather_losses(loss)
