"""CPU: the oracle is pinned against the reference's own outputs (tests/golden/, made by make_golden.py from the
reference's test_nca.reference_step / alive / autograd and torch.optim.Adam as train.py drives it) and against the
published Philox4x32-10 known-answer vectors."""
import json
import os

import numpy as np
import pytest
import torch

from oracle import nca_oracle as O

GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), 'golden')


@pytest.fixture(scope='module')
def golden():
    z = np.load(os.path.join(GOLD, 'reference_step.npz'))
    out = {}
    for key in z.files:
        case, name = key.split('/')
        out.setdefault(case, {})[name] = torch.from_numpy(z[key])
    return out


def test_philox_known_answers():
    for kat in json.load(open(os.path.join(GOLD, 'philox_kat.json'))):
        ctr = [int(v, 16) for v in kat['counter']]
        key = [int(v, 16) for v in kat['key']]
        assert O.philox4x32_10(ctr, key) == [int(v, 16) for v in kat['out']]


def test_philox_c_matches_numpy_restatement():
    for (n, h, w, seed, rate, off) in [(3, 37, 50, 1234, 0.5, 0), (2, 8, 16, 2 ** 62 - 5, 0.5, 7), (1, 5, 3, 99, 0.25, 0),
                                       (2, 9, 13, 1, 0.0, 3), (1, 4, 4, 5, 1.0, 0)]:
        assert torch.equal(O.update_mask(n, h, w, seed, rate, off), O.update_mask_np(n, h, w, seed, rate, off))


def test_mask_offset_is_global_image_index():
    full = O.update_mask(6, 9, 13, 77, 0.5)
    assert torch.equal(O.update_mask(2, 9, 13, 77, 0.5, n_offset=3), full[3:5])


def test_mask_statistics():
    # test_nca.py:160-161: update_mask(4, 128, 128, seed=7, 0.5) has mean ~0.5 and values {0, 1}
    m = O.update_mask(4, 128, 128, 7, 0.5)
    assert sorted(m.unique().tolist()) == [0.0, 1.0]
    assert abs(m.mean().item() - 0.5) < 0.01
    assert O.update_mask(1, 16, 16, 7, 1.0).min().item() == 1.0
    assert O.update_mask(1, 16, 16, 7, 0.0).max().item() == 0.0


def test_step_seeds_match_reference_splitmix64():
    s = json.load(open(os.path.join(GOLD, 'step_seeds.json')))
    assert [O.step_seed(s['seed'], i) for i in range(8)] == [int(v) for v in s['step_seeds']]
    assert [O.step_seed(s['seed_big'], i) for i in range(4)] == [int(v) for v in s['step_seeds_big']]
    assert all(O.step_seed_py(s['seed'], i) == int(v) for i, v in enumerate(s['step_seeds']))


@pytest.mark.parametrize('case', ['tex_8x16_r05', 'tex_9x13_r10', 'tex_5x37_r05', 'grow_12x10_r05', 'grow_11x14_r10'])
def test_oracle_step_matches_reference(golden, case):
    g = golden[case]
    growing = bool(g['growing'])
    mask = O.mask_for(*g['x'].shape[:2], *g['x'].shape[3:], int(g['seed']), float(g['rate']))
    assert torch.equal(mask, g['mask']), 'the golden masks come from this restatement'
    y = O.reference_step(g['x'], g['w1'], g['b1'], g['w2'], mask, growing)
    assert torch.allclose(y, g['y'], rtol=0, atol=0)
    grads = O.step_grads(g['x'], g['w1'], g['b1'], g['w2'], mask, g['R'], growing)
    for a, name in zip(grads, ('gx', 'dw1', 'db1', 'dw2')):
        assert O.rel(a, g[name]) < 1e-6, name
    # the hand-written backward (the TF32 oracle's structure) agrees with autograd in fp32
    manual = O.step_backward(g['x'], g['w1'], g['b1'], g['w2'], mask, g['R'], growing, tf32=False)
    for a, name in zip(manual, ('gx', 'dw1', 'db1', 'dw2')):
        assert O.rel(a, g[name]) < 1e-5, name


def test_tf32_oracle_close_to_fp32(golden):
    g = golden['tex_8x16_r05']
    y32 = O.reference_step(g['x'], g['w1'], g['b1'], g['w2'], g['mask'])
    ytf = O.reference_step(g['x'], g['w1'], g['b1'], g['w2'], g['mask'], tf32=True)
    assert 0 < O.rel(ytf, y32) < 1e-2
    gtf = O.step_backward(g['x'], g['w1'], g['b1'], g['w2'], g['mask'], g['R'], tf32=True)
    for a, name in zip(gtf, ('gx', 'dw1', 'db1', 'dw2')):
        assert O.rel(a, g[name]) < 3e-2, name


def test_tf32_round_is_rna():
    v = torch.tensor([1.0, 1.0 + 2 ** -11, 1.0 + 2 ** -12, -(1.0 + 2 ** -11), 3.0, float('inf'), 1.0 + 3 * 2 ** -12])
    r = O.tf32_round(v)
    assert r[0] == 1.0 and r[1] == 1.0 + 2 ** -10 and r[2] == 1.0 and r[3] == -(1.0 + 2 ** -10)  # ties away
    assert r[4] == 3.0 and torch.isinf(r[5]) and r[6] == 1.0 + 2 ** -10


@pytest.mark.parametrize('case', ['roll_tex', 'roll_grow'])
def test_oracle_rollout_matches_reference(golden, case):
    g = golden[case]
    x = g['x']
    for steps in range(1, 5):
        y = O.rollout(x, g['w1'], g['b1'], g['w2'], float(g['rate']), steps, bool(g['growing']), seed=int(g['seed']))
        assert torch.equal(y, g['ys'][steps - 1])


@pytest.mark.parametrize('C', [12, 16])
def test_dying_grid(golden, C):
    g = golden[f'dying_{C}']
    assert torch.equal(g['y7'], torch.zeros_like(g['y7']))
    y = O.rollout(g['x'], g['w1'], g['b1'], g['w2'], 1.0, 7, True, seed=99)
    assert torch.equal(y, torch.zeros_like(y))


def test_adam_reference_matches_golden(golden):
    g = golden['adam']
    grads = [[g['g_w1'][i], g['g_b1'][i], g['g_w2'][i]] for i in range(g['g_w1'].shape[0])]
    after = O.adam_reference([g['w1'], g['b1'], g['w2']], grads, lr=float(g['lr']),
                             milestones=g['milestones'].tolist(), gamma=float(g['gamma']))
    for i, ps in enumerate(after):
        for p, name in zip(ps, ('w1_after', 'b1_after', 'w2_after')):
            assert torch.equal(p, g[name][i])


def test_synthetic_loss_gradient():
    x, w1, b1, w2, target = O.make_config_inputs(2, 2, 12, 96, 8, 8)
    x = (x * 30).requires_grad_()  # push some values past the overflow bounds
    obj, per = O.synthetic_loss(x, target)
    (gx,) = torch.autograd.grad(obj, x)
    K, B, C, H, W = x.shape
    inv = 1.0 / (B * 3 * H * W)
    xd = x.detach()
    expect = torch.zeros_like(xd)
    expect[:, :, :3] = 2 * (xd[:, :, :3] - target[:, None]) * inv
    expect += 10.0 * torch.sign(xd) * (xd.abs() > 1)
    assert torch.allclose(gx, expect, atol=1e-6)
    assert per.shape == (K,)


def test_grouped_perception_matches_conv2d():
    """The kernels' summation grouping of the perception (nca_step.cuh:317-320) equals the conv2d perception of
    test_nca.py up to fp32 rounding, for every filter and circular edge."""
    x = torch.randn(2, 3, 12, 9, 13, generator=torch.Generator().manual_seed(5))
    a, b = O.perceive(x), O.perceive_grouped(x)
    assert a.shape == b.shape
    assert float((a - b).abs().max()) <= 4e-6 * float(a.abs().max())
