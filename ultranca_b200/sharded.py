"""K-sharded multi-GPU training of a group of NCAs: one process per GPU, no data-path collective.

The K NCAs are independent except for the shared rollout length of an iteration (the reference's group loop draws one
length per iteration for the whole group, train.py:133). Rank r of N owns NCAs [r K / N, (r + 1) K / N): their weights,
Adam state, pool and targets. Per iteration, rank 0 draws (rollout length, base seed) and broadcasts them; every rank
derives the step seeds as splitmix64(base, step) and passes its global image offset to the kernels, so its update masks
are exactly the single-GPU masks of its NCAs. Per-NCA losses are all-gathered for logging (train.py:213-217 keeps the
mean of the last 32 per NCA). The backend is NCCL on GPUs and gloo for the CPU tests of this control logic.
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

    def __init__(self, rollout=(32, 96), seed=0, device='cpu', group=None):
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
        """This rank's per-NCA losses (k1 - k0,) -> all ranks' losses concatenated in NCA order (every rank must hold
        the same number of NCAs: use a K divisible by the world size)."""
        if self.world == 1:
            return losses
        out = torch.empty(self.world * losses.numel(), dtype=losses.dtype, device=losses.device)
        dist.all_gather_into_tensor(out, losses.contiguous(), group=self.group)
        return out


class ShardedTrainer:
    """This rank's share of a group: RolloutTrainer over its NCAs + the control channel. `w1, b1, w2` are this shard's
    weights (K/N of them); rollouts up to `max_steps` steps."""

    def __init__(self, w1, b1, w2, B, H, W, max_steps, k0, rollout=(32, 96), control_seed=0, **trainer_kw):
        from .training import RolloutTrainer
        self.trainer = RolloutTrainer(w1, b1, w2, B, H, W, max_steps, image_offset=k0 * B, **trainer_kw)
        dev = 'cuda' if dist.is_initialized() and dist.get_backend() == 'nccl' else 'cpu'
        self.control = ControlChannel(rollout, control_seed, device=dev)

    def iteration(self, x0, target):
        steps, seed = self.control.next()
        loss, xT = self.trainer.iteration(x0, target, seed, steps=steps)
        return self.control.gather_losses(loss), xT, steps
