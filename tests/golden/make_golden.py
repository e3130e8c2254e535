"""Generate the golden fixtures in tests/golden/ from the UltraNCA reference's own Python code (run in a container
that has the reference checkout; the fixtures are committed, the GPU box never reads the reference).

    python tests/golden/make_golden.py /path/to/UltraNCA

What comes from the reference itself:
- ncaops/testing/test_nca.py: reference_step (:26-32), alive (:21-23), FILTERS (:11-12) and the splitmix64
  step_seed restatement nested in test() (:128-133), imported with the CUDA module `nca_ops` stubbed out;
- torch.optim.Adam + MultiStepLR driven exactly as train.py:120-122,136-141 do (gradient normalisation restated
  from train.py:138-139, which cannot be imported on a CPU host because train.py:24,28 moves tensors to 'cuda').
The update masks fed to reference_step come from the oracle's Philox restatement (the reference mask exists only
as a CUDA kernel), which is pinned separately by the Random123 known-answer vectors written to philox_kat.json.
"""
import ast
import json
import os
import sys
import types

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))
from oracle import nca_oracle as O  # noqa: E402

# Published known-answer vectors of philox4x32-10 (Random123 distribution, kat_vectors): counter, key -> output.
PHILOX_KAT = [
    {'counter': [0x00000000, 0x00000000, 0x00000000, 0x00000000], 'key': [0x00000000, 0x00000000],
     'out': [0x6627e8d5, 0xe169c58d, 0xbc57ac4c, 0x9b00dbd8]},
    {'counter': [0xffffffff, 0xffffffff, 0xffffffff, 0xffffffff], 'key': [0xffffffff, 0xffffffff],
     'out': [0x408f276d, 0x41c83b0e, 0xa20bc7c6, 0x6d5451fd]},
    {'counter': [0x243f6a88, 0x85a308d3, 0x13198a2e, 0x03707344], 'key': [0xa4093822, 0x299f31d0],
     'out': [0xd16cfe09, 0x94fdcceb, 0x5001e420, 0x24126ea1]},
]


def import_reference(ref_root):
    """test_nca.py with `nca_ops` stubbed (its CUDA extension cannot load here), plus its nested step_seed."""
    sys.modules['nca_ops'] = types.ModuleType('nca_ops')
    path = os.path.join(ref_root, 'ncaops', 'testing', 'test_nca.py')
    import importlib.util
    spec = importlib.util.spec_from_file_location('ref_test_nca', path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    tree = ast.parse(open(path).read())
    test_fn = next(n for n in tree.body if isinstance(n, ast.FunctionDef) and n.name == 'test')
    inner = next(n for n in test_fn.body if isinstance(n, ast.FunctionDef) and n.name == 'step_seed')
    ns = {}
    exec(compile(ast.Module(body=[inner], type_ignores=[]), path, 'exec'), ns)
    return mod, ns['step_seed']


def inputs(K, B, C, HID, H, W, seed, growing):
    return O.make(K, B, C, HID, H, W, seed=seed, growing=growing)


def main(ref_root):
    ref, ref_step_seed = import_reference(ref_root)
    torch.set_num_threads(max(1, os.cpu_count() or 1))
    out = {}

    # forward + gradients of (y * R).sum() through the reference's reference_step (test_nca.py:111-119 pattern)
    cases = [  # name, K, B, C, HID, H, W, rate, growing, seed
        ('tex_8x16_r05', 2, 2, 12, 96, 8, 16, 0.5, False, 1234),
        ('tex_9x13_r10', 1, 1, 12, 96, 9, 13, 1.0, False, 99),
        ('tex_5x37_r05', 1, 2, 12, 96, 5, 37, 0.5, False, 7),
        ('grow_12x10_r05', 1, 2, 16, 128, 12, 10, 0.5, True, 1234),
        ('grow_11x14_r10', 2, 1, 16, 128, 11, 14, 1.0, True, 5),
    ]
    for name, K, B, C, HID, H, W, rate, growing, seed in cases:
        x, w1, b1, w2 = inputs(K, B, C, HID, H, W, seed, growing)
        mask = O.mask_for(K, B, H, W, seed, rate)
        R = torch.randn(x.shape, generator=torch.Generator().manual_seed(seed + 1))
        params = [t.clone().requires_grad_() for t in (x, w1, b1, w2)]
        y = ref.reference_step(*params, mask, growing)
        grads = torch.autograd.grad((y * R).sum(), params)
        rec = dict(x=x, w1=w1, b1=b1, w2=w2, mask=mask, R=R, y=y.detach(), gx=grads[0], dw1=grads[1], db1=grads[2],
                   dw2=grads[3], rate=torch.tensor(rate), growing=torch.tensor(growing), seed=torch.tensor(seed))
        if growing:
            rec['alive_x'] = ref.alive(x)
        out[name] = rec

    # rollout: steps of reference_step with the reference's splitmix64 step seeds (test_nca.py:135-149 pattern)
    for name, C, HID, growing, rate in (('roll_tex', 12, 96, False, 0.5), ('roll_grow', 16, 128, True, 0.5)):
        x, w1, b1, w2 = inputs(2, 2, C, HID, 9, 12, 3, growing)
        ys, cur = [], x
        for i in range(4):
            s = ref_step_seed(99, i)
            cur = ref.reference_step(cur, w1, b1, w2, O.mask_for(2, 2, 9, 12, s, rate), growing).detach()
            ys.append(cur)
        out[name] = dict(x=x, w1=w1, b1=b1, w2=w2, ys=torch.stack(ys), rate=torch.tensor(rate),
                         growing=torch.tensor(growing), seed=torch.tensor(99))

    # dying grid (test_nca.py:151-158): an 8 x 16 all-ones grid with alpha 0.2 dies within 7 steps
    for C, HID in ((12, 96), (16, 128)):
        x = torch.ones(1, 1, C, 8, 16); x[:, :, 3] = 0.2
        w1 = torch.zeros(1, HID, 4 * C); b1 = torch.ones(1, HID)
        w2 = torch.full((1, C, HID), 0.01); w2[:, 3] = -0.025 / HID
        cur = x
        for i in range(7):
            cur = ref.reference_step(cur, w1, b1, w2, torch.ones(1, 1, 1, 8, 16), True)
        out[f'dying_{C}'] = dict(x=x, w1=w1, b1=b1, w2=w2, y7=cur)

    # Adam + MultiStepLR with per-NCA per-tensor normalisation (train.py:120-122,136-141), short milestones
    g = torch.Generator().manual_seed(11)
    K = 3
    params = [0.1 * torch.randn(K, 96, 48, generator=g), 0.1 * torch.randn(K, 96, generator=g),
              0.1 * torch.randn(K, 12, 96, generator=g)]
    grads = [[torch.randn(p.shape, generator=g) * (i + 1) for p in params] for i in range(5)]
    ps = [p.clone().requires_grad_() for p in params]
    opt = torch.optim.Adam(ps, 1e-3)
    sched = torch.optim.lr_scheduler.MultiStepLR(opt, [2, 4], 0.5)
    after = []
    for it in range(5):
        for p, gg in zip(ps, grads[it]):
            p.grad = gg.clone()
        with torch.no_grad():
            for p in ps:
                p.grad /= p.grad.flatten(1).norm(dim=1).reshape(-1, *[1] * (p.dim() - 1)) + 1e-8
            opt.step(); opt.zero_grad(); sched.step()
        after.append([p.detach().clone() for p in ps])
    out['adam'] = dict(w1=params[0], b1=params[1], w2=params[2],
                       g_w1=torch.stack([gg[0] for gg in grads]), g_b1=torch.stack([gg[1] for gg in grads]),
                       g_w2=torch.stack([gg[2] for gg in grads]),
                       w1_after=torch.stack([a[0] for a in after]), b1_after=torch.stack([a[1] for a in after]),
                       w2_after=torch.stack([a[2] for a in after]), milestones=torch.tensor([2, 4]),
                       gamma=torch.tensor(0.5, dtype=torch.float64), lr=torch.tensor(1e-3, dtype=torch.float64))

    flat = {f'{case}/{k}': (v.numpy() if isinstance(v, torch.Tensor) else np.asarray(v)) for case, rec in out.items()
            for k, v in rec.items()}
    np.savez_compressed(os.path.join(HERE, 'reference_step.npz'), **flat)

    seeds = {'seed': 99, 'step_seeds': [str(ref_step_seed(99, i)) for i in range(8)],
             'seed_big': 2 ** 62 - 3, 'step_seeds_big': [str(ref_step_seed(2 ** 62 - 3, i)) for i in range(4)]}
    with open(os.path.join(HERE, 'step_seeds.json'), 'w') as f:
        json.dump(seeds, f, indent=1)
    with open(os.path.join(HERE, 'philox_kat.json'), 'w') as f:
        json.dump([{k: [f'{v:08x}' for v in d[k]] for k in d} for d in PHILOX_KAT], f, indent=1)
    print('wrote', sorted(os.listdir(HERE)))


if __name__ == '__main__':
    main(sys.argv[1] if len(sys.argv) > 1 else '/root/reference')
