"""Training-iteration callers of the step (the reference's train.py:117-146 loop for the benchmark configurations),
driven through the C-ABI without autograd:

  pool sample -> `steps` forward steps (each step's input state kept for the backward, as _Step saves x,
  nca_ops.py:27) -> synthetic loss and its gradient -> `steps` backward steps in reverse, each adding its per-CTA
  weight-gradient partials to the partial workspace (zeroed once), then one reduce of the whole rollout's gradient
  instead of a reduce (or a torch add) per step -> per-NCA per-tensor gradient normalisation + Adam + MultiStepLR in
  one launch (train.py:136-141).

The synthetic loss replaces the OT texture loss (which needs VGG16 weights and datasets): per NCA, the mean squared
error of channels 0-2 to a target plus 10 x the overflow |x - clamp(x, -1, 1)| summed (config.yml overflow_weight).
"""
import ctypes

import torch

from ._lib import check, lib, ptr
from .nca_ops import backward_workspace, step_seed

LOSS_CHUNKS = 64
STAGE_MAIN, STAGE_ADJOINT, STAGE_REDUCE, STAGE_PARTIAL_ADD = 1, 2, 4, 8  # include/ultranca_b200.h NCA_STAGE_*


def _stream(dev):
    return ctypes.c_void_p(torch.cuda.current_stream(dev).cuda_stream)


def synthetic_loss(x, target, overflow_weight=10.0, gy=None, loss=None, work=None):
    """x (K, B, C, H, W), target (K, 3, H, W) -> (loss (K,), gy = d sum(loss) / dx), deterministic."""
    K, B, C, H, W = x.shape
    gy = torch.empty_like(x) if gy is None else gy
    loss = torch.empty(K, device=x.device) if loss is None else loss
    work = torch.empty(K * LOSS_CHUNKS * 2, device=x.device) if work is None else work
    with torch.cuda.device(x.device):
        check(lib.nca_synthetic_loss(ptr(x), ptr(target), ptr(gy), ptr(loss), ptr(work), K, B, C, H, W,
                                     float(overflow_weight), _stream(x.device)))
    return loss, gy


class FusedAdam:
    """torch.optim.Adam + MultiStepLR with the per-NCA per-tensor gradient normalisation of train.py:138-139, for the
    three stacked weight tensors (w1, b1, w2), in one launch per iteration. The iteration counter lives on the device
    (so a captured CUDA graph replays correctly)."""

    def __init__(self, params, lr=1e-3, betas=(0.9, 0.999), eps=1e-8, milestones=(256, 512), gamma=0.5):
        self.params = list(params)
        assert len(self.params) == 3
        self.K = self.params[0].shape[0]
        self.m = [torch.zeros_like(p) for p in self.params]
        self.v = [torch.zeros_like(p) for p in self.params]
        self.iteration = torch.zeros(1, dtype=torch.int64, device=self.params[0].device)
        self.lr, self.betas, self.eps, self.gamma = lr, betas, eps, gamma
        self.milestones = (ctypes.c_int64 * 8)(*list(milestones)[:8])
        self.n_milestones = min(len(milestones), 8)

    def step(self, grads):
        p, g, m, v = self.params, [t.contiguous() for t in grads], self.m, self.v
        dev = p[0].device
        with torch.cuda.device(dev):
            check(lib.nca_adam_step(ptr(p[0]), ptr(p[1]), ptr(p[2]), ptr(g[0]), ptr(g[1]), ptr(g[2]), ptr(m[0]),
                                    ptr(m[1]), ptr(m[2]), ptr(v[0]), ptr(v[1]), ptr(v[2]), self.K, p[0][0].numel(),
                                    p[1][0].numel(), p[2][0].numel(), ptr(self.iteration), float(self.lr),
                                    float(self.betas[0]), float(self.betas[1]), float(self.eps), float(self.gamma),
                                    self.milestones, self.n_milestones, _stream(dev)))


class RolloutTrainer:
    """One training iteration of K NCAs (B images each) over a rollout of `steps` fwd+bwd steps, with every buffer
    preallocated (no allocation inside an iteration). image_offset: global index of this shard's first image."""

    def __init__(self, w1, b1, w2, B, H, W, steps, update_rate=0.5, growing=False, fp32=False, lr=1e-3,
                 milestones=(256, 512), gamma=0.5, overflow_weight=10.0, image_offset=0):
        self.w1, self.b1, self.w2 = w1, b1, w2
        self.K, self.HID, PIN = w1.shape
        self.C = PIN // 4
        self.B, self.H, self.W, self.steps = B, H, W, steps
        self.N = self.K * B
        self.rate, self.growing, self.fp32 = float(update_rate), bool(growing), bool(fp32)
        self.overflow_weight, self.image_offset = float(overflow_weight), int(image_offset)
        dev = w1.device
        shape = (self.K, B, self.C, H, W)
        self.states = torch.empty((steps + 1,) + shape, device=dev)
        self.gy = [torch.empty(shape, device=dev) for _ in range(2)]
        self.grads = [torch.zeros_like(w1), torch.zeros_like(b1), torch.zeros_like(w2)]
        self.loss = torch.empty(self.K, device=dev)
        self.loss_work = torch.empty(self.K * LOSS_CHUNKS * 2, device=dev)
        nmap = (steps, self.N, H, W) if growing else (0,)
        self.alive = torch.empty(nmap, dtype=torch.uint8, device=dev)
        self.alpha = torch.empty((self.N, H, W) if growing else (0,), device=dev)
        self.dp_floats, self.partial_floats, _ = backward_workspace(self.C, self.HID, fp32, self.N, H, W, self.K,
                                                                    update_rate, growing, dev)
        self.dp = torch.empty(self.dp_floats, device=dev)
        self.partial = torch.empty(self.partial_floats, device=dev)
        self.opt = FusedAdam((w1, b1, w2), lr=lr, milestones=milestones, gamma=gamma)

    def forward_steps(self, seed, steps=None):
        s = self.states
        st = _stream(s.device)
        for i in range(self.steps if steps is None else steps):
            alive = ptr(self.alive[i]) if self.growing else None
            check(lib.nca_forward(ptr(s[i]), ptr(self.w1), ptr(self.b1), ptr(self.w2), ptr(s[i + 1]),
                                  ptr(self.alpha) if self.growing else None, alive, self.N, self.C, self.H, self.W,
                                  self.K, self.HID, self.B, step_seed(seed, i), self.rate, int(self.fp32),
                                  int(self.growing), self.image_offset, st))

    def backward_steps(self, seed, gy_last, steps=None):
        s, g = self.states, self.grads
        st = _stream(s.device)
        cur = gy_last
        self.partial.zero_()  # every step adds its partials; one reduce at the end
        args = lambda i, cur, nxt: (ptr(s[i]), ptr(cur), ptr(self.alive[i]) if self.growing else None, ptr(self.w1),
                                    ptr(self.b1), ptr(self.w2), ptr(nxt), ptr(g[0]), ptr(g[1]), ptr(g[2]), ptr(self.dp),
                                    self.dp_floats, ptr(self.partial), self.partial_floats, self.N, self.C, self.H,
                                    self.W, self.K, self.HID, self.B, step_seed(seed, i), self.rate, int(self.fp32),
                                    int(self.growing), self.image_offset, 0)
        for i in reversed(range(self.steps if steps is None else steps)):
            nxt = self.gy[1] if cur is self.gy[0] else self.gy[0]
            check(lib.nca_backward_stages(*args(i, cur, nxt), STAGE_MAIN | STAGE_ADJOINT | STAGE_PARTIAL_ADD, st))
            cur = nxt
        check(lib.nca_backward_stages(*args(0, cur, cur), STAGE_REDUCE, st))  # the rollout's gradient -> grads
        return cur

    def iteration(self, x0, target, seed, steps=None):
        """x0 (K, B, C, H, W) -> (per-NCA loss (K,), final state), both on the device; a rollout of `steps` (default:
        the buffer length) fwd + bwd steps, then the fused optimiser step updates w1, b1, w2 in place."""
        n = self.steps if steps is None else int(steps)
        if not 1 <= n <= self.steps:
            raise ValueError(f'rollout length {n} outside 1..{self.steps}')
        with torch.cuda.device(self.w1.device):
            self.states[0].copy_(x0)
            self.forward_steps(seed, n)
            synthetic_loss(self.states[n], target, self.overflow_weight, self.gy[0], self.loss, self.loss_work)
            self.backward_steps(seed, self.gy[0], n)
            self.opt.step(self.grads)
        return self.loss, self.states[n]
