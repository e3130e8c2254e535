"""Benchmark of the fused NCA step: cell-updates/s of a 64-step fwd+bwd rollout training iteration of K texture NCAs.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
    torchrun --nproc-per-node N bench.py --gpus N ...     (one rank per GPU)

Workload (per GPU): K = 32 texture NCAs (12 channels, 96 hidden), batch 2 per NCA drawn
from a pool of 64 seeded U[-0.1, 0.1] states per NCA, 128 x 128 circular grid, update rate 0.5, TF32 MMA; one step
of this benchmark is one training iteration: 64 forward steps, the synthetic L2 + 10 x overflow loss, 64 backward
steps, per-NCA per-tensor gradient normalisation + Adam (lr 1e-3, halved at 256 / 512), pool write-back. With N GPUs
each rank owns 32 NCAs (weak scaling, K = 32 N in total); rank 0 broadcasts the rollout length and seed over NCCL and
the per-NCA losses are all-gathered, as the reference's group loop would log them. Inputs: 64 saved states of 50 MB
per iteration (3.2 GB) exceed the 126 MB L2, so no flush is needed between iterations.

value: K B H W steps x iterations / (max over ranks of the CUDA-event time of the timed iterations). Each iteration
       is the reference's group-loop iteration run from the device (ultranca_b200.training.PoolTrainer: pool sample
       with seed injection, rollout, loss, backward, fused reduce + Adam, pool write-back), replayed as one CUDA
       graph; timing events recorded inside the graph around every 16th step's launches give the per-kernel times
       of the roofline.
e2e:   the same metric through the public operator API (ultranca_b200.nca_ops.step under autograd, the call
       train.py makes), with the batch copied host -> device from pinned memory and the losses copied back every
       iteration inside the timed region.
--impl reference: the reference's eager PyTorch step (the CPU restatement in oracle/, fp32, all host threads) on a
       bounded sample of the same workload; it prints its own JSON line and no GPU is used.
--config 4: a supplemental line (not the default): BASELINE configuration 4 per GPU, i.e. its 8-GPU shard of 64
       texture NCAs, B = 4, 256 x 256 (the row kernels over column strips), 96-step rollout, pool of 16 states per
       NCA; 64 NCAs per GPU at any N (weak scaling: K = 512 at N = 8).
"""
import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

import torch

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

K_PER_GPU, B, C, HID, H, W, STEPS, POOL, RATE = 32, 2, 12, 96, 128, 128, 64, 64, 0.5
TIMER_STRIDE = 16  # timing events around every 16th step's forward and backward launch (4 + 4 per iteration)
METRIC = 'cell-updates/s fwd+bwd, 64-step rollout'
UNIT = 'cell-updates/s'


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument('--gpus', type=int, default=1)
    ap.add_argument('--steps', type=int, default=10)
    ap.add_argument('--warmup', type=int, default=3)
    ap.add_argument('--impl', default='ours', choices=['ours', 'reference'])
    ap.add_argument('--config', type=int, default=1, choices=[1, 4])
    ap.add_argument('--no-e2e', action='store_true')
    ap.add_argument('--no-cpu', action='store_true')
    ap.add_argument('--no-ref-kernels', action='store_true')
    return ap.parse_args()


# ------------------------------------------------------------------------------------------------ clocks
class ClockSampler:
    """nvidia-smi samples (every 200 ms) of this rank's GPU during the timed region."""
    FIELDS = ('index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,'
              'clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,'
              'clocks_event_reasons.sw_power_cap')

    def __init__(self, gpu_index):
        self.gpu, self.lines, self.proc = gpu_index, [], None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(['nvidia-smi', f'--query-gpu={self.FIELDS}', '--format=csv,noheader,nounits',
                                          '-i', str(self.gpu), '-lms', '200'], stdout=subprocess.PIPE,
                                         stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
        except OSError:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
            self.thread.join(timeout=5)

    def summary(self):
        rows = [[f.strip() for f in l.split(',')] for l in self.lines if l.count(',') >= 8]
        if not rows:
            return {'sm_mhz': None, 'sm_max_mhz': None, 'reasons': ['nvidia-smi unavailable']}
        sm = [float(r[1]) for r in rows if r[1].replace('.', '').isdigit()]
        mx = [float(r[2]) for r in rows if r[2].replace('.', '').isdigit()]
        names = ('hw_slowdown', 'hw_thermal_slowdown', 'sw_thermal_slowdown', 'sw_power_cap')
        reasons = sorted({n for r in rows for n, v in zip(names, r[5:9]) if v.lower() == 'active'})
        return {'sm_mhz': statistics.median(sm) if sm else None, 'sm_max_mhz': max(mx) if mx else None,
                'reasons': reasons, 'samples': len(rows)}


# ------------------------------------------------------------------------------------------------ CPU arms
def cpu_sample(steps, threads):
    """The reference's eager fp32 step (CPU restatement, oracle/) with autograd over a `steps`-step rollout of one
    texture NCA (B = 2, 128 x 128) + synthetic loss backward. Returns (cell-updates, seconds)."""
    from oracle import nca_oracle as O
    torch.set_num_threads(threads)
    x, w1, b1, w2, target = O.make_config_inputs(1, B, C, HID, H, W, seed=0)
    w1, b1, w2 = (t.requires_grad_() for t in (w1, b1, w2))
    masks = [O.mask_for(1, B, H, W, O.step_seed(7, i), RATE) for i in range(steps)]
    t0 = time.perf_counter()
    cur = x
    for i in range(steps):
        cur = O.reference_step(cur, w1, b1, w2, masks[i])
    obj, _ = O.synthetic_loss(cur, target)
    obj.backward()
    dt = time.perf_counter() - t0
    return B * H * W * steps, dt


def cpu_baseline(max_seconds=20.0):
    threads = os.cpu_count() or 1
    cells, dt = cpu_sample(4, threads)  # warm-up and size the sample
    steps = max(4, min(STEPS, int(max_seconds / max(dt / 4, 1e-3))))
    cells, dt = cpu_sample(steps, threads)
    return {'value': cells / dt, 'unit': UNIT, 'cores': threads, 'kind': 'port',
            'sample': f'1 texture NCA x B={B} x {H}x{W}, {steps}-step fwd+bwd rollout + synthetic loss, eager fp32 '
                      f'reference_step (oracle/nca_oracle.py) on {threads} host threads, {dt:.1f} s'}


def run_reference(args):
    rank = int(os.environ.get('RANK', '0'))
    if rank != 0:
        return
    threads = os.cpu_count() or 1
    steps_per_sample = 8
    for _ in range(max(args.warmup, 0)):
        cpu_sample(steps_per_sample, threads)
    total_cells, total_t = 0, 0.0
    for _ in range(args.steps):
        cells, dt = cpu_sample(steps_per_sample, threads)
        total_cells += cells
        total_t += dt
    v = total_cells / total_t
    line = {'metric': METRIC, 'value': v, 'unit': UNIT, 'n_gpus': args.gpus, 'steps': args.steps,
            'warmup': args.warmup, 'ms_per_step': 1000 * total_t / args.steps, 'higher_is_better': True,
            'scaling': 'weak', 'vs_baseline': None, 'dtype': 'fp32', 'data': 'synthetic', 'impl': 'reference',
            'config': config(args.gpus, 'the reference eager PyTorch step on the host CPU'),
            'cpu_baseline': {'value': v, 'unit': UNIT, 'cores': threads, 'kind': 'port',
                             'sample': f'per step: 1 texture NCA x B={B} x {H}x{W}, {steps_per_sample}-step fwd+bwd '
                                       f'rollout + synthetic loss, eager fp32 (oracle/nca_oracle.py reference_step)'},
            'e2e': {'value': v, 'unit': UNIT, 'h2d_bytes_per_step': 0, 'd2h_bytes_per_step': 0}}
    print(json.dumps(line), flush=True)


def measure_tf32_tflops(dev, n=8192, reps=10):
    """Dense TF32 throughput of this GPU: torch.matmul of two n x n fp32 matrices with TF32 tensor cores allowed
    (2 n^3 flop per product), best of `reps` after warm-up, CUDA events. Untimed by the benchmark."""
    prev = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = True
    try:
        g = torch.Generator(device=dev).manual_seed(0)
        a = torch.randn(n, n, device=dev, generator=g)
        b = torch.randn(n, n, device=dev, generator=g)
        c = torch.empty(n, n, device=dev)
        for _ in range(3):
            torch.matmul(a, b, out=c)
        best = float('inf')
        for _ in range(reps):
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            torch.matmul(a, b, out=c)
            e1.record()
            e1.synchronize()
            best = min(best, e0.elapsed_time(e1))
        del a, b, c
        torch.cuda.empty_cache()
        return 2.0 * n ** 3 / (best / 1000.0) / 1e12
    finally:
        torch.backends.cuda.matmul.allow_tf32 = prev


def use_config(cfg):
    """Switch the workload constants to BASELINE configuration `cfg` (1: the default; 4: its 8-GPU shard per GPU)."""
    global K_PER_GPU, B, H, W, STEPS, POOL, METRIC, CONFIG
    CONFIG = cfg
    if cfg == 4:
        K_PER_GPU, B, H, W, STEPS, POOL = 64, 4, 256, 256, 96, 16
        METRIC = 'cell-updates/s fwd+bwd, 96-step rollout'


CONFIG = 1


def config(n, note=None):
    state_mb = K_PER_GPU * B * C * H * W * 4 / 1e6
    c = {'workload': f'texture NCA training iteration: K={K_PER_GPU * n} NCAs ({K_PER_GPU} per GPU), B={B}, '
                     f'{H}x{W}, {C} ch / {HID} hidden, {STEPS}-step rollout fwd+bwd, p={RATE}, synthetic L2+overflow '
                     f'loss, grad-norm + Adam (BASELINE config {CONFIG}'
                     f'{"" if CONFIG == 1 else ", the per-GPU shard of K=512 over 8 GPUs"})',
         'K': K_PER_GPU * n, 'B': B, 'H': H, 'W': W, 'steps_per_rollout': STEPS, 'update_rate': RATE,
         'parallelism': f'K-sharded x{n}',
         'l2': f'inputs larger than L2 ({STEPS} saved states of {state_mb:.0f} MB per iteration)'}
    if note:
        c['note'] = note
    return c


# ------------------------------------------------------------------------------------------------ GPU arm
def main():
    args = parse()
    use_config(args.config)
    if args.impl == 'reference':
        run_reference(args)
        return
    from oracle import nca_oracle as O  # seeded synthetic inputs only (same generator as the tests)
    from ultranca_b200 import nca_ops, training

    world = int(os.environ.get('WORLD_SIZE', '1'))
    rank = int(os.environ.get('RANK', '0'))
    local = int(os.environ.get('LOCAL_RANK', '0'))
    torch.cuda.set_device(local)
    dev = torch.device('cuda', local)
    dist = None
    if world > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group('nccl', timeout=datetime.timedelta(seconds=120), device_id=dev)

    tf32_tflops = measure_tf32_tflops(dev)  # before anything else runs: the compute side of the step roofline
    K = K_PER_GPU
    k0 = rank * K  # this rank's first NCA
    # seeded inputs of this shard (NCA k's weights / targets / pool depend on k only)
    g = torch.Generator().manual_seed(1000 + rank)
    _, w1, b1, w2, target = O.make_config_inputs(K, 1, C, HID, H, W, seed=1000 + rank)
    pool = ((torch.rand(K, POOL, C, H, W, generator=g) * 2 - 1) * 0.1).to(dev)
    w1, b1, w2, target = (t.to(dev).contiguous() for t in (w1, b1, w2, target))
    trainer = training.RolloutTrainer(w1, b1, w2, B, H, W, STEPS, RATE, growing=False, fp32=False,
                                      image_offset=k0 * B)
    # the reference's group-loop iteration on the device (pool sample + seed injection every 16 iterations, rollout,
    # loss, backward, fused reduce + Adam, pool write-back), one CUDA graph replay per iteration; the control block's
    # key is shared by every rank (broadcast once), so all ranks draw the same rollout seeds, and the pool draws of
    # NCA k follow its global index
    key = torch.tensor([20240611], dtype=torch.int64, device=dev)
    if dist is not None:
        dist.broadcast(key, 0)
    loop = training.PoolTrainer(trainer, pool, target, inject_every=16, seed_kind=training.SEED_TEXTURE,
                                key=int(key.item()), graph=True, timed=TIMER_STRIDE, nca_offset=k0)
    stream = torch.cuda.current_stream(dev)
    # rank 0 draws the rollout length per iteration and broadcasts it (config 1: always STEPS)
    ctl = torch.zeros(1, dtype=torch.int64, device=dev)
    losses_all = torch.zeros(world * K, device=dev)

    # The length for iteration i + 1 is broadcast on a side stream while iteration i runs, so reading it on the host
    # never waits for the step kernels (single GPU: drawn on the host, nothing to broadcast).
    side = torch.cuda.Stream(dev)
    ctl_host = torch.zeros(1, dtype=torch.int64).pin_memory()
    ctl_ready = torch.cuda.Event()

    def prefetch_control():
        with torch.cuda.stream(side):
            if rank == 0:
                ctl.fill_(STEPS)
            if dist is not None:
                dist.broadcast(ctl, 0)
            ctl_host.copy_(ctl, non_blocking=True)
            ctl_ready.record(side)

    def take_control():
        ctl_ready.synchronize()
        steps = int(ctl_host[0])
        assert steps == STEPS
        prefetch_control()
        return steps

    def iteration():
        loop.iteration(take_control())
        if dist is not None:
            dist.all_gather_into_tensor(losses_all, trainer.loss)
        return trainer.loss

    prefetch_control()

    # warm-up (the first iteration launches directly; the graph is recorded at the second)
    for i in range(args.warmup):
        iteration()
    torch.cuda.synchronize()
    loop.kernel_times(reset=True)
    if dist is not None:
        dist.barrier()
    torch.cuda.synchronize()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clocks:
        start.record(stream)
        for i in range(args.steps):
            iteration()
        end.record(stream)
        torch.cuda.synchronize()
    if dist is not None:
        dist.barrier()
    torch.cuda.synchronize()
    ms = start.elapsed_time(end)
    stage_times = loop.kernel_times()
    if dist is not None:
        t = torch.tensor([ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    cells_per_iter = world * K * B * H * W * STEPS
    value = cells_per_iter * args.steps / (ms / 1000.0)
    rows = nca_ops.launch_info(C, HID, False, K * B, H, W, K)['rows_path']
    # per iteration: control 1, pool sample 2, forward 1 / step, loss 2, backward 1 / step (row path; main + adjoint
    # on the tile path, main + edge fix-up over column strips), fused reduce + Adam 1, iteration counter 1, pool
    # write-back 1
    launches_per_iter = 1 + 2 + STEPS + 2 + STEPS * (1 if rows == 1 else 2) + 1 + 1 + 1
    # roofline of the dominant kernel (the larger mean of the sampled forward and backward launches)
    mean = {k: statistics.mean(v) for k, v in stage_times.items()}
    dom = max(mean, key=mean.get)
    avg_ms = mean[dom]
    # algorithmic bytes per cell (fp32, 12 channels): forward reads x and writes y (96 B); the fused backward reads x
    # and gy and writes gx (144 B); the tile-path backward main kernel reads x and gy (96 B)
    alg_per_cell = 96 if dom == 'fwd' else (144 if rows else 96)
    alg_bytes = K * B * H * W * alg_per_cell
    peaks = {}
    try:
        peaks = json.load(open(os.path.join(ROOT, 'MEASURED_PEAKS.json')))
    except (OSError, ValueError):
        pass
    peak = peaks.get('hbm_gbs', 6650.0)
    achieved = alg_bytes / (avg_ms / 1000.0) / 1e9
    traffic = None
    try:  # per-launch DRAM bytes of one ncu capture of the config-1 step
        tr = json.load(open(os.path.join(ROOT, 'profiles', 'traffic.json')))
        if CONFIG == 1:
            traffic = tr.get({'fwd': 'fwd_rows_kernel' if rows else 'fwd_kernel',
                              'bwd': 'bwd_rows_kernel' if rows else 'bwd_kernel_tc'}[dom])
    except (OSError, ValueError):
        pass
    # the step roofline (per cell-step, p = 0.5: 17,280 flop of the MLP forward and backward, 240 B of state traffic):
    # the slower of the flops at the TF32 peak measured here and the bytes at the measured HBM bandwidth
    cell_steps = K * B * H * W * STEPS
    step_compute_ms = cell_steps * 17280.0 / (tf32_tflops * 1e12) * 1e3
    step_hbm_ms = cell_steps * 240.0 / (peak * 1e9) * 1e3
    step_roof_ms = max(step_compute_ms, step_hbm_ms)
    roofline = {'bound': 'hbm', 'achieved': achieved, 'peak': peak, 'unit': 'GB/s', 'frac': achieved / peak,
                'traffic': traffic,
                'kernel': {'fwd': 'fwd_rows_kernel<12,96,2>' if rows else 'fwd_kernel<12,96,TC>',
                           'bwd': 'bwd_rows_kernel<12,96,4>' if rows else 'bwd_kernel_tc<12,96>'}[dom] +
                          (' (column strips)' if rows == 2 else ''),
                'algorithmic_bytes_per_launch': alg_bytes, 'avg_launch_ms': avg_ms,
                'timed_launches': {k: len(v) for k, v in stage_times.items()},
                'launch_ms': {k: v for k, v in mean.items()},
                'peak_source': 'MEASURED_PEAKS.json hbm_gbs (of measured)' if 'hbm_gbs' in peaks else 'fallback',
                'stage_ms_per_iteration': {k: v * STEPS for k, v in mean.items()},
                'tf32_tflops_measured': tf32_tflops,
                'step_roofline': {'compute_ms': step_compute_ms, 'hbm_ms': step_hbm_ms, 'bound_ms': step_roof_ms,
                                  'bound': 'hbm' if step_hbm_ms >= step_compute_ms else 'tensor',
                                  'frac_of_iteration': step_roof_ms / (ms / args.steps)}}

    # e2e through the public operator API with host buffers
    e2e = None
    if not args.no_e2e:
        e2e = run_e2e(args, dev, rank, world, dist, K, w1, b1, w2, target, nca_ops, training)

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu:
        cpu = cpu_baseline()
    ref_b200 = None
    if rank == 0 and world == 1 and not args.no_ref_kernels:
        ref_b200 = reference_kernels_b200(args, dev)

    if rank == 0:
        line = {'metric': METRIC, 'value': value, 'unit': UNIT, 'n_gpus': world, 'steps': args.steps,
                'warmup': args.warmup, 'ms_per_step': ms / args.steps, 'higher_is_better': True, 'scaling': 'weak',
                'vs_baseline': None, 'dtype': 'tf32', 'data': 'synthetic', 'config': config(world),
                'roofline': roofline, 'cpu_baseline': cpu, 'e2e': e2e, 'clocks': clocks.summary(),
                'gpu_launches': launches_per_iter * args.steps, 'reference_kernels_b200': ref_b200,
                'launch': nca_ops.launch_info(C, HID, False, K * B, H, W, K)}
        print(json.dumps(line), flush=True)
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()


def reference_kernels_b200(args, dev):
    """The reference's own CUDA kernels (ncaops/nca_step.cuh compiled for sm_100a, oracle/_ref) on the same workload
    and GPU: 64 forward launches (states kept, as the reference's autograd saves x), 64 backward launches (pack,
    backward, adjoint, reduce) and the per-step weight-gradient accumulation autograd performs. A comparison point,
    not this repository's product; None when oracle/_ref was not built."""
    from oracle import nca_oracle as O
    from oracle import ref_kernels as R
    if not R.available():
        return None
    from ultranca_b200 import nca_ops
    x0, w1, b1, w2, _ = O.make_config_inputs(K_PER_GPU, B, C, HID, H, W, seed=5)
    x0, w1, b1, w2 = (t.to(dev).contiguous() for t in (x0, w1, b1, w2))
    states = torch.empty((STEPS + 1,) + tuple(x0.shape), device=dev)
    gy = torch.randn_like(x0)
    bwd = R.Backward(K_PER_GPU, B, C, HID, H, W, RATE)
    outs = [torch.empty_like(x0), torch.empty_like(w1), torch.empty_like(b1), torch.empty_like(w2)]
    acc = [torch.zeros_like(w1), torch.zeros_like(b1), torch.zeros_like(w2)]

    def it(i):
        states[0].copy_(x0)
        for s in range(STEPS):
            y, _ = R.forward(states[s], w1, b1, w2, RATE, nca_ops.step_seed(i, s))
            states[s + 1].copy_(y)
        g = gy
        for s in reversed(range(STEPS)):
            gx, dw1, db1, dw2 = bwd(states[s], g, None, w1, b1, w2, nca_ops.step_seed(i, s), out=outs)
            for a_, d_ in zip(acc, (dw1, db1, dw2)):
                a_.add_(d_)
            g = gx.clone()

    for i in range(args.warmup):
        it(i)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    n_it = max(1, min(args.steps, 5))
    e0.record()
    for i in range(n_it):
        it(100 + i)
    e1.record()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / n_it
    return {'value': K_PER_GPU * B * H * W * STEPS / (ms / 1000.0), 'unit': UNIT, 'ms_per_step': ms,
            'note': 'the reference CUDA kernels (ncaops/nca_step.cuh, mma.sync TF32) compiled for sm_100a and run on '
                    'this B200 on the same 64-step fwd+bwd rollout (1 GPU, without the optimiser step and without '
                    'Python/autograd overhead), timed with CUDA events'}


def run_e2e(args, dev, rank, world, dist, K, w1, b1, w2, target, nca_ops, training):
    """The training iteration as train.py runs it on the drop-in operator: nca_ops.step per step under autograd,
    backward through _Step, the fused optimiser; batch H2D from pinned host memory, losses D2H, every iteration. The
    batch of iteration i + 1 is copied on a side stream while iteration i computes (two device buffers; a buffer is
    refilled once the iteration that read it, whose autograd graph keeps it, has finished)."""
    g = torch.Generator().manual_seed(77 + rank)
    host = ((torch.rand(K, B, C, H, W, generator=g) * 2 - 1) * 0.1).pin_memory()
    ws = [t.clone().requires_grad_() for t in (w1, b1, w2)]
    opt = training.FusedAdam(ws)
    loss_host = torch.empty(K).pin_memory()
    stream = torch.cuda.current_stream(dev)
    copy_stream = torch.cuda.Stream(dev)
    dbuf = [torch.empty(host.shape, device=dev) for _ in range(2)]
    ready = [torch.cuda.Event() for _ in range(2)]
    done = [torch.cuda.Event() for _ in range(2)]
    pending = set()

    def prefetch(i):
        b = i % 2
        with torch.cuda.stream(copy_stream):
            if b in pending:
                copy_stream.wait_event(done[b])  # the iteration that last read this buffer has finished
            dbuf[b].copy_(host, non_blocking=True)
            ready[b].record(copy_stream)

    def it(i):
        b = i % 2
        if i == first[0]:
            prefetch(i)
        prefetch(i + 1)
        stream.wait_event(ready[b])
        x = dbuf[b]
        for s in range(STEPS):
            x = nca_ops.step(x, *ws, RATE, seed=1000 * i + s, image_offset=rank * K * B)
        loss, gy = training.synthetic_loss(x.detach(), target)
        x.backward(gy)
        opt.step([w.grad for w in ws])
        for w in ws:
            w.grad = None
        loss_host.copy_(loss, non_blocking=True)
        done[b].record(stream)
        pending.add(b)

    first = [0]
    for i in range(args.warmup):
        it(i)
    torch.cuda.synchronize()
    if dist is not None:
        dist.barrier()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    first[0] = args.warmup  # the timed region copies its own first batch too
    pending.clear()
    start.record(stream)
    for i in range(args.steps):
        it(args.warmup + i)
    end.record(stream)
    torch.cuda.synchronize()
    ms = start.elapsed_time(end)
    if dist is not None:
        t = torch.tensor([ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    return {'value': world * K * B * H * W * STEPS * args.steps / (ms / 1000.0), 'unit': UNIT,
            'h2d_bytes_per_step': host.numel() * 4, 'd2h_bytes_per_step': K * 4,
            'path': 'ultranca_b200.nca_ops.step under autograd (train.py call pattern) + fused Adam',
            'ms_per_step': ms / args.steps}


if __name__ == '__main__':
    main()
