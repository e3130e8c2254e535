"""Training-iteration callers of the step (the reference's train.py:117-146 loop for the benchmark configurations),
driven through the C-ABI without autograd:

  pool sample -> `steps` forward steps (each step's input state kept for the backward, as _Step saves x,
  nca_ops.py:27) -> synthetic loss and its gradient -> `steps` backward steps in reverse, each adding its per-CTA
  weight-gradient partials to the partial workspace (zeroed once) -> one launch that reduces the whole rollout's
  gradient and applies the per-NCA per-tensor gradient normalisation + Adam + MultiStepLR (train.py:136-141).

RolloutTrainer runs one iteration from a batch and a seed given by the host. PoolTrainer runs the reference's whole
group-loop iteration (train.py:126-142: pool sampling, seed injection, rollout, loss, update, pool write-back) from
the device, with the iteration's seeds in a device control block, so that each rollout length is captured once as a
CUDA graph and every later iteration is one graph replay.

The synthetic loss replaces the OT texture loss (which needs VGG16 weights and datasets): per NCA, the mean squared
error of channels 0-2 to a target plus 10 x the overflow |x - clamp(x, -1, 1)| summed (config.yml overflow_weight).
"""
import ctypes

import torch

from ._lib import check, lib, ptr
from .nca_ops import backward_workspace, step_seed

LOSS_CHUNKS = 64
STAGE_MAIN, STAGE_ADJOINT, STAGE_REDUCE, STAGE_PARTIAL_ADD, STAGE_X_STABLE = 1, 2, 4, 8, 16  # NCA_STAGE_*


def _stream(dev):
    return ctypes.c_void_p(torch.cuda.current_stream(dev).cuda_stream)


def _timed(timers, kind, launch, on=True):
    """launch(), bracketed by a pair of timing events appended to `timers` as (kind, start, end) when timers is a list
    (and `on`). The events are external, so that inside a CUDA-graph capture they become event-record nodes of the
    graph and time the kernel on every replay."""
    if timers is None or not on:
        launch()
        return
    e0, e1 = torch.cuda.Event(enable_timing=True, external=True), torch.cuda.Event(enable_timing=True, external=True)
    e0.record()
    launch()
    e1.record()
    timers.append((kind, e0, e1))


def synthetic_loss(x, target, overflow_weight=10.0, gy=None, loss=None, work=None):
    """x (K, B, C, H, W), target (K, TC, H, W) -> (loss (K,), gy = d sum(loss) / dx), deterministic: per NCA the mean
    squared error of channels 0 .. TC-1 to the target + overflow_weight x the summed overflow |x - clamp(x, -1, 1)|.
    TC = 3 with overflow_weight = 10: the texture configurations; TC = 4 with overflow_weight = 0: the growing NCA's
    L2 to a premultiplied RGBA target (train.py:97-99)."""
    K, B, C, H, W = x.shape
    gy = torch.empty_like(x) if gy is None else gy
    loss = torch.empty(K, device=x.device) if loss is None else loss
    work = torch.empty(K * LOSS_CHUNKS * 2, device=x.device) if work is None else work
    with torch.cuda.device(x.device):
        check(lib.nca_task_loss(ptr(x), ptr(target), ptr(gy), ptr(loss), ptr(work), K, B, C, H, W, target.shape[1],
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
        self.dp_floats, self.partial_floats, _ = backward_workspace(self.C, self.HID, fp32, self.N, H, W, self.K,
                                                                    update_rate, growing, dev)
        self.dp = torch.empty(self.dp_floats, device=dev)
        self.partial = torch.empty(self.partial_floats, device=dev)
        self.opt = FusedAdam((w1, b1, w2), lr=lr, milestones=milestones, gamma=gamma)

    def forward_steps(self, seed, steps=None, seed_dev=None, timers=None, timer_stride=1):
        """Forward steps 0 .. steps-1 from states[0]; step i's update mask uses step_seed(seed, i), or, with seed_dev
        (a device pointer to the rollout seed), the same seed read on the device when the kernel runs. timers: a list
        that receives ('fwd', start, end) events around the launches of steps i % timer_stride == timer_stride // 2."""
        s = self.states
        st = _stream(s.device)
        for i in range(self.steps if steps is None else steps):
            alive = ptr(self.alive[i]) if self.growing else None
            common = (ptr(s[i]), ptr(self.w1), ptr(self.b1), ptr(self.w2), ptr(s[i + 1]),
                      None, alive, self.N, self.C, self.H, self.W, self.K,
                      self.HID, self.B)
            tail = (self.rate, int(self.fp32), int(self.growing), self.image_offset, st)
            on = i % timer_stride == timer_stride // 2
            if seed_dev is None:
                _timed(timers, 'fwd', lambda: check(lib.nca_forward(*common, step_seed(seed, i), *tail)), on)
            else:
                _timed(timers, 'fwd', lambda: check(lib.nca_forward_dseed(*common, seed_dev, i, *tail)), on)

    def backward_steps(self, seed, gy_last, steps=None, reduce=True, seed_dev=None, timers=None, timer_stride=1):
        """Backward steps in reverse, each adding its weight-gradient partials; reduce: one fixed-order reduce of the
        rollout's partials into grads (otherwise reduce_adam does it). Returns the gradient of states[0]. timers: a
        list that receives ('bwd', start, end) events around the launches of steps i % timer_stride ==
        timer_stride // 2."""
        s, g = self.states, self.grads
        st = _stream(s.device)
        cur = gy_last
        self.partial.zero_()  # every step adds its partials; one reduce at the end

        def call(i, cur, nxt, stages):
            head = (ptr(s[i]), ptr(cur), ptr(self.alive[i]) if self.growing else None, ptr(self.w1), ptr(self.b1),
                    ptr(self.w2), ptr(nxt), ptr(g[0]), ptr(g[1]), ptr(g[2]), ptr(self.dp), self.dp_floats,
                    ptr(self.partial), self.partial_floats, self.N, self.C, self.H, self.W, self.K, self.HID, self.B)
            tail = (self.rate, int(self.fp32), int(self.growing), self.image_offset, 0, stages, st)
            if seed_dev is None:
                check(lib.nca_backward_stages(*head, step_seed(seed, i), *tail))
            else:
                check(lib.nca_backward_stages_dseed(*head, seed_dev, i, *tail))

        for i in reversed(range(self.steps if steps is None else steps)):
            nxt = self.gy[1] if cur is self.gy[0] else self.gy[0]
            # the saved states were written before the zeroing above (a kernel of its own): stable for the backward
            _timed(timers, 'bwd', lambda: call(i, cur, nxt, STAGE_MAIN | STAGE_ADJOINT | STAGE_PARTIAL_ADD |
                                               STAGE_X_STABLE), i % timer_stride == timer_stride // 2)
            cur = nxt
        if reduce:
            call(0, cur, cur, STAGE_REDUCE)  # the rollout's gradient -> grads
        return cur

    def reduce_adam(self):
        """The rollout's gradient from the partial workspace -> grads, then the optimiser step, in one launch
        (bitwise equal to the REDUCE stage followed by FusedAdam.step)."""
        o, g = self.opt, self.grads
        check(lib.nca_reduce_adam_step(ptr(self.partial), self.partial_floats, self.N, self.C, self.H, self.W, self.K,
                                       self.HID, self.B, int(self.fp32), int(self.growing), ptr(g[0]), ptr(g[1]),
                                       ptr(g[2]), ptr(self.w1), ptr(self.b1), ptr(self.w2), ptr(o.m[0]), ptr(o.m[1]),
                                       ptr(o.m[2]), ptr(o.v[0]), ptr(o.v[1]), ptr(o.v[2]), ptr(o.iteration),
                                       float(o.lr), float(o.betas[0]), float(o.betas[1]), float(o.eps),
                                       float(o.gamma), o.milestones, o.n_milestones, _stream(self.w1.device)))

    def _check_rows_alignment(self):
        # reduce_adam assumes the backward ran on 16-byte-aligned buffers (torch allocations and whole-image slices)
        for t in (self.states, self.gy[0], self.gy[1]):
            assert t.data_ptr() % 16 == 0

    def iteration(self, x0, target, seed, steps=None, fused=True):
        """x0 (K, B, C, H, W) -> (per-NCA loss (K,), final state), both on the device; a rollout of `steps` (default:
        the buffer length) fwd + bwd steps, then the optimiser step updates w1, b1, w2 in place (fused: in the same
        launch as the gradient reduction; otherwise a reduce launch and a FusedAdam launch, bitwise the same)."""
        n = self.steps if steps is None else int(steps)
        if not 1 <= n <= self.steps:
            raise ValueError(f'rollout length {n} outside 1..{self.steps}')
        with torch.cuda.device(self.w1.device):
            self.states[0].copy_(x0)
            self.forward_steps(seed, n)
            synthetic_loss(self.states[n], target, self.overflow_weight, self.gy[0], self.loss, self.loss_work)
            self.backward_steps(seed, self.gy[0], n, reduce=not fused)
            if fused:
                self._check_rows_alignment()
                self.reduce_adam()
            else:
                self.opt.step(self.grads)
        return self.loss, self.states[n]


SEED_TEXTURE, SEED_GROWING = 0, 1  # seed states of nca_pool_sample (train.py Texture.seed / Growing.seed)


class PoolTrainer:
    """The reference's group-loop iteration (train.py:126-142) for a RolloutTrainer, driven from the device:

        control advance (iteration index, rollout seed) -> pool sample of B distinct entries per NCA, with the seed
        state injected every `inject_every` iterations -> rollout -> loss -> backward -> fused reduce + Adam -> pool
        write-back.

    Nothing in an iteration is read from the host but the rollout length, so each length is recorded once as a CUDA
    graph (graph=True) and replayed; graph=False launches the same sequence directly (the two are bitwise equal).
    pool: (K, P, C, H, W) on the trainer's device, updated in place. key: seed of the control block's draws.
    timed = s > 0: timing events around the step launches of every s-th step (in the graph as event-record nodes);
    kernel_times() returns them. A timed length is recorded as two graphs replayed in turn, so that the times of one
    replay are read while the next runs."""

    def __init__(self, trainer, pool, target, inject_every=16, seed_kind=SEED_TEXTURE, key=0, graph=True,
                 timed=0, nca_offset=0):
        t = trainer
        if tuple(pool.shape[:1] + pool.shape[2:]) != (t.K, t.C, t.H, t.W) or not pool.is_contiguous():
            raise ValueError(f'pool must be a contiguous (K, P, C, H, W) = ({t.K}, P, {t.C}, {t.H}, {t.W}) tensor')
        self.t, self.pool, self.target = t, pool, target
        self.P = pool.shape[1]
        self.inject_every, self.seed_kind, self.graph = int(inject_every), int(seed_kind), bool(graph)
        self.nca_offset = int(nca_offset)  # global index of this shard's NCA 0 (the pool draws follow it)
        dev = t.w1.device
        self.ctl = torch.zeros(4, dtype=torch.int64, device=dev)
        self.ctl[0] = int(key) - (1 << 64) if int(key) >= (1 << 63) else int(key)
        self.idx = torch.empty(t.K * t.B, dtype=torch.int64, device=dev)
        self.graphs = {}  # rollout length -> [(graph, its timer list or None)]
        self.launched = False  # the first iteration runs directly (the library's one-time set-up happens there)
        self.timed = int(timed)
        self.times = {}  # kind -> [ms] of the launches timed so far
        self._pending = []  # timer lists of launched iterations not read yet
        self._next = {}  # rollout length -> graph copy to replay next

    def _body(self, n, timers=None):
        t = self.t
        st = _stream(t.w1.device)
        seed_dev = self.ctl.data_ptr() + 3 * 8
        check(lib.nca_control_advance(ptr(self.ctl), st))
        check(lib.nca_pool_sample(ptr(self.pool), ptr(t.states[0]), ptr(self.idx), ptr(self.ctl), t.K, self.P, t.B,
                                  t.C, t.H, t.W, self.inject_every, self.seed_kind, self.nca_offset, st))
        t.forward_steps(None, n, seed_dev=seed_dev, timers=timers, timer_stride=max(self.timed, 1))
        synthetic_loss(t.states[n], self.target, t.overflow_weight, t.gy[0], t.loss, t.loss_work)
        t.backward_steps(None, t.gy[0], n, reduce=False, seed_dev=seed_dev, timers=timers,
                         timer_stride=max(self.timed, 1))
        t.reduce_adam()
        check(lib.nca_pool_store(ptr(self.pool), ptr(t.states[n]), ptr(self.idx), t.K, self.P, t.B, t.C, t.H, t.W,
                                 st))

    def iteration(self, steps=None):
        """One training iteration with a rollout of `steps` (default: the trainer's length); returns the per-NCA
        losses (device tensor, overwritten by the next iteration)."""
        t = self.t
        n = t.steps if steps is None else int(steps)
        if not 1 <= n <= t.steps:
            raise ValueError(f'rollout length {n} outside 1..{t.steps}')
        t._check_rows_alignment()
        with torch.cuda.device(t.w1.device):
            if not self.graph or not self.launched:
                timers = [] if self.timed else None
                self._body(n, timers)
                if timers:
                    self._pending.append(timers)
                self.launched = True
                return t.loss
            copies = self.graphs.get(n)
            if copies is None:
                copies = []
                for _ in range(2 if self.timed else 1):
                    timers = [] if self.timed else None
                    g = torch.cuda.CUDAGraph()
                    with torch.cuda.graph(g):
                        self._body(n, timers)
                    copies.append((g, timers))
                self.graphs[n] = copies
            c = self._next.get(n, 0)
            self._next[n] = (c + 1) % len(copies)
            g, timers = copies[c]
            if timers:
                if any(p is timers for p in self._pending):  # its previous replay: read before it is re-recorded
                    self._read(timers)
                self._pending.append(timers)
            g.replay()
        return t.loss

    def _read(self, timers):
        timers[-1][2].synchronize()
        for kind, e0, e1 in timers:
            self.times.setdefault(kind, []).append(e0.elapsed_time(e1))
        self._pending = [p for p in self._pending if p is not timers]

    def kernel_times(self, reset=False):
        """{kind: [ms per timed launch]} over the iterations run so far (timed > 0; synchronises); reset: start a new
        collection afterwards."""
        for timers in list(self._pending):
            self._read(timers)
        out = self.times
        if reset:
            self.times = {}
        return out

    def iteration_index(self):
        """Index of the last iteration started (host read; synchronises)."""
        return int(self.ctl[2].item())
