"""Benchmark of the fused NCA step: cell-updates/s of BASELINE's configurations on B200s.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--config 1|2|3|4]
    torchrun --nproc-per-node N bench.py --gpus N ...     (one rank per GPU)

Configurations (one "step" of this benchmark = one training iteration, or one no-grad rollout for configuration 3):
  1 (default): K = 32 texture NCAs per GPU (12 channels, 96 hidden), batch 2 drawn from a pool of 64 seeded
     U[-0.1, 0.1] states per NCA, 128 x 128 circular grid, update rate 0.5, TF32; one iteration = 64 forward steps,
     the synthetic L2 + 10 x overflow loss, 64 backward steps, per-NCA per-tensor gradient normalisation + Adam
     (lr 1e-3, halved at 256 / 512), pool write-back, seed injection every 16 iterations. Weak scaling: K = 32 N.
  2: K = 64 growing NCAs in all (16 channels, 128 hidden), batch 8 from a pool of 64 seed states per NCA (one living
     cell at the centre), 72 x 72, an 80-step rollout fwd+bwd, L2 to a synthetic premultiplied RGBA disc, grad-norm +
     Adam; update rates 0.5 (the line's value) and 1.0 (reported beside it). Strong scaling: K / N NCAs per GPU.
  3: no-grad rollout of K = 256 texture NCAs in all, batch 4, 256 x 256, 128 steps, rate 0.5. Strong scaling.
  4: the per-GPU shard of configuration 4: 64 texture NCAs per GPU, B = 4, 256 x 256, 96-step rollout fwd+bwd, pool of
     16 states per NCA. Weak scaling (K = 512 at N = 8).
The default run (configuration 1) also measures configurations 2 and 3 with fewer iterations and reports them under
"configs" in the same JSON line (outside the line's own timed region), so every driver run records them.

Multi-GPU: one process per GPU, K-sharded (ultranca_b200.sharded.ShardedPoolTrainer); rank 0 broadcasts the control
block's key once and the rollout length every iteration over NCCL, the per-NCA losses are all-gathered. No data-path
collective. Times are CUDA-event times on the launching stream, max over ranks.

value: cell-updates (K B H W steps, all ranks) per second of the timed iterations. Each training iteration is the
       reference's group-loop iteration run from the device (training.PoolTrainer, one CUDA graph replay); timing
       events recorded inside the graph around every 16th step's launches give the per-kernel times of the roofline.
       Inputs exceed the 126 MB L2 (the saved states of a rollout, the 3.2 GB state of configuration 3), so there is
       no flush between iterations.
e2e:   the same metric through the public operator API (nca_ops.step under autograd + fused Adam, or nca_ops.rollout)
       with the batch copied host -> device from pinned memory and the result (losses, or the final states) copied
       back every step inside the timed region.
--fp32: the accuracy mode (nca_ops.step(..., fp32=True), which train.py selects with tf32: false) instead of TF32.
--impl reference: the reference's eager PyTorch step (its CPU restatement in oracle/, fp32, all host threads) on a
       bounded sample of the same workload; rank 0 prints its own JSON line, no GPU is used.
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

CONFIGS = {
    1: dict(kind='train', K=32, scaling='weak', B=2, C=12, HID=96, H=128, W=128, steps=64, pool=64, rates=(0.5,),
            growing=False, overflow=10.0, seed_kind=0),
    2: dict(kind='train', K=64, scaling='strong', B=8, C=16, HID=128, H=72, W=72, steps=80, pool=64, rates=(0.5, 1.0),
            growing=True, overflow=0.0, seed_kind=1),
    3: dict(kind='infer', K=256, scaling='strong', B=4, C=12, HID=96, H=256, W=256, steps=128, rates=(0.5,),
            growing=False),
    4: dict(kind='train', K=64, scaling='weak', B=4, C=12, HID=96, H=256, W=256, steps=96, pool=16, rates=(0.5,),
            growing=False, overflow=10.0, seed_kind=0),
}
TIMER_STRIDE = 16  # timing events around every 16th step's forward and backward launch
UNIT = 'cell-updates/s'
KEY = 20240611  # seed of the device control block (rollout seeds, pool draws)


def metric_of(cfg):
    what = 'fwd+bwd' if cfg['kind'] == 'train' else 'no-grad'
    return f'cell-updates/s {what}, {cfg["steps"]}-step rollout'


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument('--gpus', type=int, default=1)
    ap.add_argument('--steps', type=int, default=10)
    ap.add_argument('--warmup', type=int, default=3)
    ap.add_argument('--impl', default='ours', choices=['ours', 'reference'])
    ap.add_argument('--config', type=int, default=1, choices=sorted(CONFIGS))
    ap.add_argument('--no-e2e', action='store_true')
    ap.add_argument('--no-cpu', action='store_true')
    ap.add_argument('--no-ref-kernels', action='store_true')
    ap.add_argument('--no-extra', action='store_true', help='skip the configurations 2 and 3 of the default run')
    ap.add_argument('--fp32', action='store_true', help="the reference's fp32=True accuracy mode (here: the MLP in "
                    'fp32 on CUDA cores) instead of TF32 tensor cores')
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
def cpu_sample(cfg, steps, threads, rate=None):
    """The reference's eager fp32 step (its CPU restatement, oracle/) on one NCA of the configuration's shape: a
    `steps`-step rollout with autograd + the task loss's backward (training configurations), or without gradients
    (configuration 3). Returns (cell-updates, seconds)."""
    from oracle import nca_oracle as O
    torch.set_num_threads(threads)
    B, C, HID, H, W = cfg['B'], cfg['C'], cfg['HID'], cfg['H'], cfg['W']
    rate = cfg['rates'][0] if rate is None else rate
    if cfg['growing']:
        x, w1, b1, w2, target = O.make_growing_inputs(1, B, C, HID, H, W, seed=0)
    else:
        x, w1, b1, w2, target = O.make_config_inputs(1, B, C, HID, H, W, seed=0)
    masks = [O.mask_for(1, B, H, W, O.step_seed(7, i), rate) for i in range(steps)]
    t0 = time.perf_counter()
    if cfg['kind'] == 'infer':
        with torch.no_grad():
            cur = x
            for i in range(steps):
                cur = O.reference_step(cur, w1, b1, w2, masks[i])
    else:
        w1, b1, w2 = (t.requires_grad_() for t in (w1, b1, w2))
        cur = x
        for i in range(steps):
            cur = O.reference_step(cur, w1, b1, w2, masks[i], cfg['growing'])
        obj = O.growing_loss(cur, target)[0] if cfg['growing'] else O.synthetic_loss(cur, target)[0]
        obj.backward()
    dt = time.perf_counter() - t0
    return B * H * W * steps, dt


def cpu_baseline(cfg, max_seconds=15.0):
    threads = os.cpu_count() or 1
    cells, dt = cpu_sample(cfg, 2, threads)  # warm-up and size the sample
    steps = max(2, min(cfg['steps'], int(max_seconds / max(dt / 2, 1e-3))))
    cells, dt = cpu_sample(cfg, steps, threads)
    grad = 'fwd+bwd rollout + task loss' if cfg['kind'] == 'train' else 'no-grad rollout'
    return {'value': cells / dt, 'unit': UNIT, 'cores': threads, 'kind': 'port',
            'sample': f'extrapolated from 1 NCA x B={cfg["B"]} x {cfg["H"]}x{cfg["W"]}, a {steps}-step {grad}, eager '
                      f'fp32 reference_step (oracle/nca_oracle.py) on {threads} host threads, {dt:.1f} s'}


def run_reference(args, cfg):
    rank = int(os.environ.get('RANK', '0'))
    if rank != 0:
        return
    threads = os.cpu_count() or 1
    steps_per_sample = 8 if cfg['H'] <= 128 else 2
    for _ in range(max(args.warmup, 0)):
        cpu_sample(cfg, steps_per_sample, threads)
    total_cells, total_t = 0, 0.0
    for _ in range(args.steps):
        cells, dt = cpu_sample(cfg, steps_per_sample, threads)
        total_cells += cells
        total_t += dt
    v = total_cells / total_t
    grad = 'fwd+bwd rollout + task loss' if cfg['kind'] == 'train' else 'no-grad rollout'
    line = {'metric': metric_of(cfg), 'value': v, 'unit': UNIT, 'n_gpus': args.gpus, 'steps': args.steps,
            'warmup': args.warmup, 'ms_per_step': 1000 * total_t / args.steps, 'higher_is_better': True,
            'scaling': cfg['scaling'], 'vs_baseline': None, 'dtype': 'fp32', 'data': 'synthetic', 'impl': 'reference',
            'config': config_dict(cfg, args.config, args.gpus, 'the reference eager PyTorch step on the host CPU'),
            'cpu_baseline': {'value': v, 'unit': UNIT, 'cores': threads, 'kind': 'port',
                             'sample': f'per step: 1 NCA x B={cfg["B"]} x {cfg["H"]}x{cfg["W"]}, a {steps_per_sample}'
                                       f'-step {grad}, eager fp32 (oracle/nca_oracle.py reference_step)'},
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


def config_dict(cfg, cid, n, note=None):
    K_total = cfg['K'] * n if cfg['scaling'] == 'weak' else cfg['K']
    per = f'{cfg["K"]} per GPU' if cfg['scaling'] == 'weak' else f'{cfg["K"]} in all, K/N per GPU'
    kind = 'growing' if cfg['growing'] else 'texture'
    if cfg['kind'] == 'train':
        loss = 'L2 to a premultiplied RGBA disc' if cfg['growing'] else 'synthetic L2+overflow loss'
        what = f'{kind} NCA training iteration: K={K_total} NCAs ({per}), B={cfg["B"]}, {cfg["H"]}x{cfg["W"]}, ' \
               f'{cfg["C"]} ch / {cfg["HID"]} hidden, {cfg["steps"]}-step rollout fwd+bwd, p={cfg["rates"][0]}, ' \
               f'{loss}, grad-norm + Adam'
        state_mb = cfg['K'] * cfg['B'] * cfg['C'] * cfg['H'] * cfg['W'] * 4 / 1e6
        l2 = f'inputs larger than L2 ({cfg["steps"]} saved states of {state_mb:.0f} MB per iteration per GPU)'
    else:
        what = f'{kind} NCA no-grad rollout: K={K_total} NCAs ({per}), B={cfg["B"]}, {cfg["H"]}x{cfg["W"]}, ' \
               f'{cfg["C"]} ch / {cfg["HID"]} hidden, {cfg["steps"]} steps, p={cfg["rates"][0]}'
        state_gb = cfg['K'] * cfg['B'] * cfg['C'] * cfg['H'] * cfg['W'] * 4 / 1e9
        l2 = f'inputs larger than L2 ({state_gb:.1f} GB of state in all)'
    c = {'workload': f'{what} (BASELINE config {cid})', 'K': K_total, 'B': cfg['B'], 'H': cfg['H'], 'W': cfg['W'],
         'channels': cfg['C'], 'hidden': cfg['HID'], 'steps_per_rollout': cfg['steps'], 'update_rate': cfg['rates'][0],
         'parallelism': f'K-sharded x{n}', 'l2': l2}
    if note:
        c['note'] = note
    return c


def load_peaks():
    try:
        return json.load(open(os.path.join(ROOT, 'MEASURED_PEAKS.json')))
    except (OSError, ValueError):
        return {}


# ------------------------------------------------------------------------------------------------ GPU arms
class Ctx:
    """Per-process GPU context: rank, world, device, process group, the measured TF32 peak."""

    def __init__(self):
        self.world = int(os.environ.get('WORLD_SIZE', '1'))
        self.rank = int(os.environ.get('RANK', '0'))
        self.local = int(os.environ.get('LOCAL_RANK', '0'))
        torch.cuda.set_device(self.local)
        self.dev = torch.device('cuda', self.local)
        self.dist = None
        if self.world > 1:
            import datetime
            import torch.distributed as dist
            dist.init_process_group('nccl', timeout=datetime.timedelta(seconds=120), device_id=self.dev)
            self.dist = dist
        self.tf32_tflops = measure_tf32_tflops(self.dev)  # the compute side of the step roofline (untimed)
        self.peaks = load_peaks()
        self.hbm = self.peaks.get('hbm_gbs', 6650.0)

    def barrier(self):
        if self.dist is not None:
            self.dist.barrier()
        torch.cuda.synchronize()

    def max_ms(self, ms):
        if self.dist is None:
            return ms
        t = torch.tensor([ms], device=self.dev)
        self.dist.all_reduce(t, op=self.dist.ReduceOp.MAX)
        return float(t.item())


def shard_of(cfg, ctx):
    """(global K, this rank's first NCA, its NCA count)."""
    from ultranca_b200.sharded import shard_range
    if cfg['scaling'] == 'weak':
        return cfg['K'] * ctx.world, ctx.rank * cfg['K'], cfg['K']
    k0, k1 = shard_range(cfg['K'], ctx.world, ctx.rank)
    return cfg['K'], k0, k1 - k0


def weights_of(cfg, k0, Kr, seed):
    """Seeded weights of NCAs [k0, k0 + Kr) (NCA k's depend on k only): w1 ~ N(0, 0.02), b1 ~ N(0, 0.01),
    w2 ~ N(0, 0.02)."""
    C, HID = cfg['C'], cfg['HID']
    ws = []
    for k in range(k0, k0 + Kr):
        g = torch.Generator().manual_seed(seed * 100003 + k)
        ws.append((0.02 * torch.randn(HID, 4 * C, generator=g), 0.01 * torch.randn(HID, generator=g),
                   0.02 * torch.randn(C, HID, generator=g)))
    return [torch.stack(t) for t in zip(*ws)]


def train_inputs(cfg, ctx, k0, Kr):
    """This shard's weights, targets and pool (on the device)."""
    from oracle import nca_oracle as O  # seeded synthetic inputs only
    B, C, HID, H, W, P = cfg['B'], cfg['C'], cfg['HID'], cfg['H'], cfg['W'], cfg['pool']
    if cfg['growing']:  # the group's seeded weights and disc targets, this shard's slice; a pool of seed states
        seed_state, w1, b1, w2, target = O.make_growing_inputs(k0 + Kr, 1, C, HID, H, W, seed=2)
        w1, b1, w2, target = (t[k0:k0 + Kr] for t in (w1, b1, w2, target))
        pool = seed_state[0, 0].expand(Kr, P, C, H, W).contiguous()
    else:
        seed = 1000 + (ctx.rank if cfg['scaling'] == 'weak' else k0)
        g = torch.Generator().manual_seed(seed)
        _, w1, b1, w2, target = O.make_config_inputs(Kr, 1, C, HID, H, W, seed=seed)
        pool = (torch.rand(Kr, P, C, H, W, generator=g) * 2 - 1) * 0.1
    to = lambda t: t.to(ctx.dev).contiguous()
    return to(w1), to(b1), to(w2), to(target), to(pool)


def launches_per_iteration(cfg, steps, rows_path, growing):
    """Kernels of one training iteration: control advance 1, pool sample 2 (draw, gather), per forward step 1 (the
    growing alive mask is computed in the forward's epilogue), loss 2, per backward step 1 (row kernel) or 2 (tile
    path: main + adjoint; column strips: main + edge fix-up), fused reduce + Adam 1, iteration counter 1, pool
    write-back 1."""
    del growing
    fwd = 1
    bwd = 1 if rows_path == 1 else 2
    return 1 + 2 + steps * fwd + 2 + steps * bwd + 1 + 1 + 1


def measure_train(cfg, cid, ctx, steps_timed, warmup, rate, e2e=True, cpu=True, ref_kernels=False, fp32=False):
    """One configuration's training iteration at one update rate: the JSON fields of its line."""
    from ultranca_b200 import nca_ops, sharded
    K_total, k0, Kr = shard_of(cfg, ctx)
    B, C, HID, H, W, S = cfg['B'], cfg['C'], cfg['HID'], cfg['H'], cfg['W'], cfg['steps']
    w1, b1, w2, target, pool = train_inputs(cfg, ctx, k0, Kr)
    job = sharded.ShardedPoolTrainer(w1, b1, w2, pool, target, B, H, W, S, K_total, rollout=(S, S + 1),
                                     key=KEY, inject_every=16, seed_kind=cfg['seed_kind'], timed=TIMER_STRIDE,
                                     update_rate=rate, growing=cfg['growing'], overflow_weight=cfg['overflow'],
                                     fp32=fp32)
    stream = torch.cuda.current_stream(ctx.dev)
    for _ in range(warmup):  # the first iteration launches directly, the graph is recorded at the second
        job.iteration()
    torch.cuda.synchronize()
    job.loop.kernel_times(reset=True)
    ctx.barrier()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(ctx.local) as clocks:
        start.record(stream)
        for _ in range(steps_timed):
            job.iteration()
        end.record(stream)
        torch.cuda.synchronize()
    ctx.barrier()
    ms = ctx.max_ms(start.elapsed_time(end))
    stage_times = job.loop.kernel_times()
    cells_per_iter = K_total * B * H * W * S
    value = cells_per_iter * steps_timed / (ms / 1000.0)
    info = nca_ops.launch_info(C, HID, fp32, Kr * B, H, W, Kr, growing=cfg['growing'])
    rows = info['rows_path'] if not cfg['growing'] else 0
    # the dominant kernel (the larger mean of the sampled forward and backward launches)
    mean = {k: statistics.mean(v) for k, v in stage_times.items()}
    dom = max(mean, key=mean.get)
    avg_ms = mean[dom]
    # algorithmic bytes per cell and launch (fp32): texture forward x in, y out (96 B); fused backward x, gy in, gx
    # out (144 B); tile-path backward main x, gy in (96 B; the adjoint launch is inside the same bracket). Growing
    # (16 channels): forward 128 B + 1 B alive map; backward x, gy in, gx out 192 B + 1 B alive map
    if cfg['growing']:
        alg_per_cell = {'fwd': 129, 'bwd': 193}[dom]
    elif fp32:  # the tile path: forward x in, y out; backward main x, gy in + dp out, adjoint dp, gy in, gx out
        alg_per_cell = {'fwd': 96, 'bwd': 96}[dom]
    else:
        alg_per_cell = {'fwd': 96, 'bwd': 144 if rows else 96}[dom]
    cells = Kr * B * H * W
    achieved = cells * alg_per_cell / (avg_ms / 1000.0) / 1e9
    traffic = None
    if cid == 1 and not cfg['growing'] and not fp32:
        try:  # per-launch DRAM bytes of one ncu capture of the benchmark's kernels (profiles/traffic.json)
            tr = json.load(open(os.path.join(ROOT, 'profiles', 'traffic.json')))
            traffic = tr.get({'fwd': 'fwd_rows_kernel', 'bwd': 'bwd_rows_kernel_x_stable'}[dom])
        except (OSError, ValueError):
            pass
    # the step roofline, per cell-step at update rate p: texture 34,560 p flop (MLP forward + backward) and 240 B;
    # growing 61,440 p flop and 322 B (x, y, gy, gx of 16 channels + the alive map read and written)
    flop_cell, byte_cell = (61440.0, 322.0) if cfg['growing'] else (34560.0, 240.0)
    cell_steps = cells * S
    step_compute_ms = cell_steps * flop_cell * rate / (ctx.tf32_tflops * 1e12) * 1e3
    step_hbm_ms = cell_steps * byte_cell / (ctx.hbm * 1e9) * 1e3
    step_roof_ms = max(step_compute_ms, step_hbm_ms)
    kname = {'fwd': {1: 'fwd_rows_kernel<12,96,2>', 2: 'fwd_rows_kernel<12,96,2,strip>', 0: 'fwd_kernel'},
             'bwd': {1: 'bwd_rows_kernel<12,96,4,x_stable>', 2: 'bwd_rows_kernel<12,96,4,x_stable,strip>',
                     0: 'bwd_kernel_tc + adjoint_kernel'}}[dom][rows]
    if fp32:
        kname = {'fwd': 'fwd_kernel<12,96,fp32>', 'bwd': 'bwd_kernel_cc<12,96> + adjoint_kernel'}[dom]
    roofline = {'bound': 'hbm', 'achieved': achieved, 'peak': ctx.hbm, 'unit': 'GB/s', 'frac': achieved / ctx.hbm,
                'traffic': traffic, 'kernel': kname, 'algorithmic_bytes_per_launch': cells * alg_per_cell,
                'avg_launch_ms': avg_ms, 'timed_launches': {k: len(v) for k, v in stage_times.items()},
                'launch_ms': mean,
                'peak_source': 'MEASURED_PEAKS.json hbm_gbs (of measured)' if 'hbm_gbs' in ctx.peaks else 'fallback',
                'stage_ms_per_iteration': {k: v * S for k, v in mean.items()},
                'tf32_tflops_measured': ctx.tf32_tflops,
                'step_roofline': {'compute_ms': step_compute_ms, 'hbm_ms': step_hbm_ms, 'bound_ms': step_roof_ms,
                                  'bound': 'hbm' if step_hbm_ms >= step_compute_ms else 'tensor',
                                  'frac_of_iteration': step_roof_ms / (ms / steps_timed)}}
    if traffic is not None:
        roofline['traffic_note'] = 'ncu dram bytes of the X_STABLE backward instance the graph replays' \
            if dom == 'bwd' else 'ncu dram bytes of the forward row kernel'
    if cfg['growing']:
        # alive-sparse figures: the cells alive after each step of the last iteration (the saved alive maps)
        t = job.trainer
        frac = float(t.alive[:S].float().mean().item())
        roofline['alive_fraction'] = frac
        roofline['step_roofline']['sparse_bound_ms'] = step_roof_ms * frac
    out = {'value': value, 'ms_per_step': ms / steps_timed, 'roofline': roofline, 'clocks': clocks.summary(),
           'gpu_launches': launches_per_iteration(cfg, S, rows, cfg['growing']) * steps_timed,
           'launch': info, 'losses_finite': bool(torch.isfinite(job.trainer.loss).all().item())}
    del job
    if e2e:
        out['e2e'] = run_e2e_train(cfg, ctx, K_total, k0, Kr, w1, b1, w2, target, rate, steps_timed, warmup, fp32)
    if cpu and ctx.rank == 0 and ctx.world == 1:
        out['cpu_baseline'] = cpu_baseline(cfg)
    if ref_kernels and ctx.rank == 0 and ctx.world == 1:
        out['reference_kernels_b200'] = reference_kernels_b200(cfg, steps_timed, warmup, ctx.dev)
    torch.cuda.empty_cache()
    return out


def run_e2e_train(cfg, ctx, K_total, k0, Kr, w1, b1, w2, target, rate, steps_timed, warmup, fp32=False):
    """The training iteration as train.py runs it on the drop-in operator: nca_ops.step per step under autograd,
    backward through _Step, the fused optimiser; batch H2D from pinned host memory, losses D2H, every iteration. The
    batch of iteration i + 1 is copied on a side stream while iteration i computes (two device buffers; a buffer is
    refilled once the iteration that read it, whose autograd graph keeps it, has finished)."""
    from ultranca_b200 import nca_ops, training
    B, C, H, W, S = cfg['B'], cfg['C'], cfg['H'], cfg['W'], cfg['steps']
    g = torch.Generator().manual_seed(77 + k0)
    if cfg['growing']:
        host = torch.zeros(Kr, B, C, H, W)
        host[:, :, 3:, H // 2, W // 2] = 1.0
        host = host.pin_memory()
    else:
        host = ((torch.rand(Kr, B, C, H, W, generator=g) * 2 - 1) * 0.1).pin_memory()
    ws = [t.clone().requires_grad_() for t in (w1, b1, w2)]
    opt = training.FusedAdam(ws)
    loss_host = torch.empty(Kr).pin_memory()
    stream = torch.cuda.current_stream(ctx.dev)
    copy_stream = torch.cuda.Stream(ctx.dev)
    dbuf = [torch.empty(host.shape, device=ctx.dev) for _ in range(2)]
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
        for s in range(S):
            x = nca_ops.step(x, *ws, rate, cfg['growing'], fp32, seed=1000 * i + s, image_offset=k0 * B)
        loss, gy = training.synthetic_loss(x.detach(), target, cfg['overflow'])
        x.backward(gy)
        opt.step([w.grad for w in ws])
        for w in ws:
            w.grad = None
        loss_host.copy_(loss, non_blocking=True)
        done[b].record(stream)
        pending.add(b)

    first = [0]
    for i in range(warmup):
        it(i)
    torch.cuda.synchronize()
    ctx.barrier()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    first[0] = warmup  # the timed region copies its own first batch too
    pending.clear()
    start.record(stream)
    for i in range(steps_timed):
        it(warmup + i)
    end.record(stream)
    torch.cuda.synchronize()
    ms = ctx.max_ms(start.elapsed_time(end))
    return {'value': K_total * B * H * W * S * steps_timed / (ms / 1000.0), 'unit': UNIT,
            'h2d_bytes_per_step': host.numel() * 4, 'd2h_bytes_per_step': Kr * 4,
            'path': 'ultranca_b200.nca_ops.step under autograd (train.py call pattern) + fused Adam',
            'ms_per_step': ms / steps_timed}


def measure_infer(cfg, cid, ctx, steps_timed, warmup, e2e=True, cpu=True):
    """No-grad rollouts (nca_ops.rollout, the reference's make_rollout path): the JSON fields of the line."""
    from ultranca_b200 import nca_ops
    K_total, k0, Kr = shard_of(cfg, ctx)
    B, C, HID, H, W, S = cfg['B'], cfg['C'], cfg['HID'], cfg['H'], cfg['W'], cfg['steps']
    rate = cfg['rates'][0]
    w1, b1, w2 = (t.to(ctx.dev).contiguous() for t in weights_of(cfg, k0, Kr, 3))
    gen = torch.Generator(device=ctx.dev).manual_seed(3000 + k0)
    x = (torch.rand(Kr, B, C, H, W, device=ctx.dev, generator=gen) * 2 - 1) * 0.1
    stream = torch.cuda.current_stream(ctx.dev)
    for i in range(warmup):
        nca_ops.rollout(x, w1, b1, w2, rate, S, seed=i, image_offset=k0 * B)
    torch.cuda.synchronize()
    ctx.barrier()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(ctx.local) as clocks:
        start.record(stream)
        for i in range(steps_timed):
            y = nca_ops.rollout(x, w1, b1, w2, rate, S, seed=100 + i, image_offset=k0 * B)
        end.record(stream)
        torch.cuda.synchronize()
    ctx.barrier()
    ms = ctx.max_ms(start.elapsed_time(end))
    finite = bool(torch.isfinite(y).all().item())
    del y
    value = K_total * B * H * W * S * steps_timed / (ms / 1000.0)
    info = nca_ops.launch_info(C, HID, False, Kr * B, H, W, Kr)
    # one launch per step and nothing else on the stream: the launch time is the rollout time per step (back-to-back
    # launches overlap their set-up with the previous step's tail, as in the rollout the metric times)
    avg_ms = ms / steps_timed / S
    cells = Kr * B * H * W
    achieved = cells * 96 / (avg_ms / 1000.0) / 1e9
    cell_steps = cells * S
    step_compute_ms = cell_steps * 11520.0 * rate / (ctx.tf32_tflops * 1e12) * 1e3
    step_hbm_ms = cell_steps * 96.0 / (ctx.hbm * 1e9) * 1e3
    step_roof_ms = max(step_compute_ms, step_hbm_ms)
    rows = info['rows_path']
    roofline = {'bound': 'hbm', 'achieved': achieved, 'peak': ctx.hbm, 'unit': 'GB/s', 'frac': achieved / ctx.hbm,
                'traffic': None,
                'kernel': {1: 'fwd_rows_kernel<12,96,2>', 2: 'fwd_rows_kernel<12,96,2,strip>', 0: 'fwd_kernel'}[rows],
                'algorithmic_bytes_per_launch': cells * 96, 'avg_launch_ms': avg_ms,
                'peak_source': 'MEASURED_PEAKS.json hbm_gbs (of measured)' if 'hbm_gbs' in ctx.peaks else 'fallback',
                'tf32_tflops_measured': ctx.tf32_tflops,
                'step_roofline': {'compute_ms': step_compute_ms, 'hbm_ms': step_hbm_ms, 'bound_ms': step_roof_ms,
                                  'bound': 'hbm' if step_hbm_ms >= step_compute_ms else 'tensor',
                                  'frac_of_iteration': step_roof_ms / (ms / steps_timed)}}
    out = {'value': value, 'ms_per_step': ms / steps_timed, 'roofline': roofline, 'clocks': clocks.summary(),
           'gpu_launches': S * steps_timed, 'launch': info, 'states_finite': finite}
    if e2e:
        out['e2e'] = run_e2e_infer(cfg, ctx, K_total, k0, Kr, w1, b1, w2, x, steps_timed)
    del x
    if cpu and ctx.rank == 0 and ctx.world == 1:
        out['cpu_baseline'] = cpu_baseline(cfg)
    torch.cuda.empty_cache()
    return out


def run_e2e_infer(cfg, ctx, K_total, k0, Kr, w1, b1, w2, x_dev, steps_timed):
    """nca_ops.rollout with the initial states copied host -> device from pinned memory and the final states copied
    back, every rollout, inside the timed region."""
    from ultranca_b200 import nca_ops
    B, H, W, S = cfg['B'], cfg['H'], cfg['W'], cfg['steps']
    host_in = x_dev.cpu().pin_memory()
    host_out = torch.empty_like(host_in).pin_memory()
    dbuf = torch.empty_like(x_dev)
    stream = torch.cuda.current_stream(ctx.dev)
    ctx.barrier()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record(stream)
    for i in range(steps_timed):
        dbuf.copy_(host_in, non_blocking=True)
        y = nca_ops.rollout(dbuf, w1, b1, w2, cfg['rates'][0], S, seed=200 + i, image_offset=k0 * B)
        host_out.copy_(y, non_blocking=True)
    end.record(stream)
    torch.cuda.synchronize()
    ms = ctx.max_ms(start.elapsed_time(end))
    return {'value': K_total * B * H * W * S * steps_timed / (ms / 1000.0), 'unit': UNIT,
            'h2d_bytes_per_step': host_in.numel() * 4, 'd2h_bytes_per_step': host_out.numel() * 4,
            'path': 'ultranca_b200.nca_ops.rollout (the reference make_rollout call), states host -> device -> host',
            'ms_per_step': ms / steps_timed}


def reference_kernels_b200(cfg, steps_timed, warmup, dev):
    """The reference's own CUDA kernels (ncaops/nca_step.cuh compiled for sm_100a, oracle/_ref) on the same workload
    and GPU: 64 forward launches (states kept, as the reference's autograd saves x), 64 backward launches (pack,
    backward, adjoint, reduce) and the per-step weight-gradient accumulation autograd performs. A comparison point,
    not this repository's product; None when oracle/_ref was not built."""
    from oracle import nca_oracle as O
    from oracle import ref_kernels as R
    if not R.available():
        return None
    from ultranca_b200 import nca_ops
    K, B, C, HID, H, W, S, RATE = cfg['K'], cfg['B'], cfg['C'], cfg['HID'], cfg['H'], cfg['W'], cfg['steps'], 0.5
    x0, w1, b1, w2, _ = O.make_config_inputs(K, B, C, HID, H, W, seed=5)
    x0, w1, b1, w2 = (t.to(dev).contiguous() for t in (x0, w1, b1, w2))
    states = torch.empty((S + 1,) + tuple(x0.shape), device=dev)
    gy = torch.randn_like(x0)
    bwd = R.Backward(K, B, C, HID, H, W, RATE)
    outs = [torch.empty_like(x0), torch.empty_like(w1), torch.empty_like(b1), torch.empty_like(w2)]
    acc = [torch.zeros_like(w1), torch.zeros_like(b1), torch.zeros_like(w2)]

    def it(i):
        states[0].copy_(x0)
        for s in range(S):
            y, _ = R.forward(states[s], w1, b1, w2, RATE, nca_ops.step_seed(i, s))
            states[s + 1].copy_(y)
        g = gy
        for s in reversed(range(S)):
            gx, dw1, db1, dw2 = bwd(states[s], g, None, w1, b1, w2, nca_ops.step_seed(i, s), out=outs)
            for a_, d_ in zip(acc, (dw1, db1, dw2)):
                a_.add_(d_)
            g = gx.clone()

    for i in range(warmup):
        it(i)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    n_it = max(1, min(steps_timed, 5))
    e0.record()
    for i in range(n_it):
        it(100 + i)
    e1.record()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / n_it
    del states
    torch.cuda.empty_cache()
    return {'value': K * B * H * W * S / (ms / 1000.0), 'unit': UNIT, 'ms_per_step': ms,
            'note': 'the reference CUDA kernels (ncaops/nca_step.cuh, mma.sync TF32) compiled for sm_100a and run on '
                    'this B200 on the same 64-step fwd+bwd rollout (1 GPU, without the optimiser step and without '
                    'Python/autograd overhead), timed with CUDA events'}


def measure(cid, ctx, steps_timed, warmup, args, main=True):
    cfg = CONFIGS[cid]
    if cfg['kind'] == 'infer':
        return measure_infer(cfg, cid, ctx, steps_timed, warmup, e2e=not args.no_e2e, cpu=not args.no_cpu)
    fp32 = bool(getattr(args, 'fp32', False)) and main
    out = measure_train(cfg, cid, ctx, steps_timed, warmup, cfg['rates'][0], e2e=not args.no_e2e,
                        cpu=not args.no_cpu and not fp32, ref_kernels=main and cid == 1 and not args.no_ref_kernels
                        and not fp32, fp32=fp32)
    for rate in cfg['rates'][1:]:  # further update rates (configuration 2): value, time, roofline and clocks
        r = measure_train(cfg, cid, ctx, steps_timed, warmup, rate, e2e=False, cpu=False)
        out[f'rate_{rate}'] = {k: r[k] for k in ('value', 'ms_per_step', 'roofline', 'clocks', 'gpu_launches')}
    return out


def main():
    args = parse()
    cfg = CONFIGS[args.config]
    if args.impl == 'reference':
        run_reference(args, cfg)
        return
    ctx = Ctx()
    res = measure(args.config, ctx, args.steps, args.warmup, args)
    extra = {}
    if args.config == 1 and not args.no_extra and not args.fp32:
        # configurations 2 and 3 with fewer iterations, outside the line's own timed region
        for cid, (n, w) in ((2, (3, 3)), (3, (3, 3))):
            r = measure(cid, ctx, n, w, args, main=False)
            extra[str(cid)] = dict(metric=metric_of(CONFIGS[cid]), unit=UNIT, steps=n, warmup=w,
                                   scaling=CONFIGS[cid]['scaling'], config=config_dict(CONFIGS[cid], cid, ctx.world),
                                   **r)
    if ctx.rank == 0:
        line = {'metric': metric_of(cfg), 'value': res['value'], 'unit': UNIT, 'n_gpus': ctx.world,
                'steps': args.steps, 'warmup': args.warmup, 'ms_per_step': res['ms_per_step'],
                'higher_is_better': True, 'scaling': cfg['scaling'], 'vs_baseline': None,
                'dtype': 'fp32' if args.fp32 else 'tf32',
                'data': 'synthetic', 'config': config_dict(cfg, args.config, ctx.world)}
        line.update({k: v for k, v in res.items() if k not in ('value', 'ms_per_step')})
        line.setdefault('cpu_baseline', None)
        line.setdefault('e2e', None)
        if extra:
            line['configs'] = extra
        print(json.dumps(line), flush=True)
    if ctx.dist is not None:
        ctx.dist.barrier()
        ctx.dist.destroy_process_group()


if __name__ == '__main__':
    main()
