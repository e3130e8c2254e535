"""GPU parity of the sm_100a kernels against the CPU oracle (oracle/nca_oracle.py) and the reference's golden outputs,
following the reference's own test plan (ncaops/testing/test_nca.py:57-163): forward over several shapes including
partial tiles, gradients, bitwise determinism and chunk invariance, rollout == repeated steps, the dying grid, the
exact alive predicate, the mask statistic; plus the tensor-core layout self-test, the bit-exact Philox mask, the
sharding offset, the synthetic loss and the fused optimiser.

Tolerances (relative error ||a - b|| / ||b||, test_nca.py:35-36):
  fp32 mode vs fp32 oracle            forward 1e-5, gradients 1e-5   (the reference's FP32 bounds, test_nca.py:17)
  TF32 mode vs TF32-emulating oracle  forward 1e-3, gradients 1e-3   (the parity bar: 1e-3 relative for TF32)
  TF32 mode vs fp32 oracle            forward 1e-2, gradients 3e-2   (the reference's TF32 bounds, test_nca.py:17)
"""
import ctypes
import os

import numpy as np
import pytest
import torch

from oracle import nca_oracle as O

pytestmark = pytest.mark.gpu
DEV = 'cuda'
GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), 'golden')
SIZES = ((12, 96), (16, 128))
FWD_SHAPES = ((3, 2, 128, 128), (2, 3, 37, 50), (1, 1, 8, 16), (3, 2, 80, 80), (17, 2, 129, 65), (1, 1, 6, 200))
BWD_SHAPES = ((3, 2, 64, 64), (2, 3, 37, 50), (1, 1, 5, 140), (2, 2, 23, 100), (1, 3, 4, 8))


@pytest.fixture(scope='module')
def ops():
    from ultranca_b200 import nca_ops
    torch.backends.cuda.matmul.allow_tf32 = False
    torch.backends.cudnn.allow_tf32 = False
    return nca_ops


def gpu(*ts):
    return [t.to(DEV) for t in ts]


def device_error_clear():
    from ultranca_b200._lib import lib
    code = ctypes.c_int()
    assert lib.nca_device_error(ctypes.byref(code), 1) == 0
    return code.value == 0


# ------------------------------------------------------------------------------------------------ tensor cores
UMMA_CASES = [(0, 96, 56), (1, 16, 96), (1, 96, 56), (1, 96, 16), (1, 48, 96), (1, 128, 72), (2, 64, 128),
              (2, 16, 128), (2, 96, 128), (2, 128, 128)]


def umma_selftest(form, N, K, seed=0):
    from ultranca_b200._lib import check, lib
    g = torch.Generator().manual_seed(seed + 100 * form + N + K)
    A = torch.randn(128, K, generator=g)
    B = torch.randn(N, K, generator=g)
    D = torch.empty(128, N, device=DEV)
    Ad, Bd = gpu(A, B)
    check(lib.nca_umma_selftest(form, N, K, ctypes.c_void_p(Ad.data_ptr()), ctypes.c_void_p(Bd.data_ptr()),
                                ctypes.c_void_p(D.data_ptr()), None))
    torch.cuda.synchronize()
    ref = (O.tf32_round(A).double() @ O.tf32_round(B).double().T).float()
    return O.rel(D.cpu(), ref)


@pytest.mark.parametrize('form,N,K', UMMA_CASES)
def test_umma_layout_selftest(form, N, K):
    """Every tcgen05 operand form the step kernels use computes A B^T exactly (up to fp32 accumulation order)."""
    assert umma_selftest(form, N, K) < 1e-5
    assert device_error_clear()


def test_umma_swapped_strides_are_detected():
    """The self-test can tell the two stride conventions of the swizzled MN-major descriptor apart."""
    assert umma_selftest(3, 64, 128) > 1e-2
    assert device_error_clear()


# ------------------------------------------------------------------------------------------------ mask
@pytest.mark.parametrize('n,h,w,seed,rate,off', [(4, 128, 128, 7, 0.5, 0), (3, 37, 50, 1234, 0.5, 0),
                                                 (2, 9, 13, 2 ** 62 - 1, 0.3, 5), (1, 8, 16, 99, 1.0, 0),
                                                 (2, 5, 7, 1, 0.0, 1)])
def test_update_mask_bit_exact(ops, n, h, w, seed, rate, off):
    m = ops.update_mask(n, h, w, seed, rate, image_offset=off)
    assert torch.equal(m.cpu(), O.update_mask(n, h, w, seed, rate, off))


def test_mask_statistic(ops):
    m = ops.update_mask(4, 128, 128, 7, 0.5)  # test_nca.py:160-161
    assert sorted(m.unique().tolist()) == [0.0, 1.0] and abs(m.mean().item() - 0.5) < 0.01


# ------------------------------------------------------------------------------------------------ forward
@pytest.mark.parametrize('C,HID', SIZES)
@pytest.mark.parametrize('rate', [0.5, 1.0])
@pytest.mark.parametrize('growing', [False, True])
def test_forward_parity(ops, C, HID, rate, growing):
    worst = {True: 0.0, False: 0.0}
    worst_vs32 = 0.0
    flips = 0
    for K, B, H, W in FWD_SHAPES:
        x, w1, b1, w2 = O.make(K, B, C, HID, H, W, seed=H * W, growing=growing)
        mask = O.mask_for(K, B, H, W, 1234, rate)
        xd, w1d, b1d, w2d = gpu(x, w1, b1, w2)
        for fp32 in (True, False):
            out = ops.step(xd, w1d, b1d, w2d, rate, growing, fp32=fp32, seed=1234).cpu()
            ref = O.reference_step(x, w1, b1, w2, mask, growing, tf32=not fp32)
            if growing:
                raw = ops.step(xd, w1d, b1d, w2d, rate, False, fp32=fp32, seed=1234).cpu()
                out_alive = O.alive(x) & O.alive(raw)
                assert torch.equal(out, raw * out_alive), 'growing step must apply the exact alive mask'
                ref_raw = O.reference_step(x, w1, b1, w2, mask, False, tf32=not fp32)
                ref_alive = O.alive(x) & O.alive(ref_raw)
                flip = (out_alive != ref_alive)
                flips += int(flip.sum())
                err = max(O.rel(raw, ref_raw), O.rel(out.masked_fill(flip, 0), ref.masked_fill(flip, 0)))
            else:
                err = O.rel(out, ref)
            worst[fp32] = max(worst[fp32], err)
            if not fp32:
                ref32 = O.reference_step(x, w1, b1, w2, mask, growing, tf32=False)
                worst_vs32 = max(worst_vs32, O.rel(out, ref32) if not growing else O.rel(raw, O.reference_step(
                    x, w1, b1, w2, mask, False)))
    assert device_error_clear()
    assert worst[True] < 1e-5, worst
    assert worst[False] < 1e-3, worst
    assert worst_vs32 < 1e-2, worst_vs32
    assert flips <= 32


def test_forward_matches_reference_golden(ops):
    z = np.load(os.path.join(GOLD, 'reference_step.npz'))
    for case in ('tex_8x16_r05', 'tex_9x13_r10', 'tex_5x37_r05', 'grow_12x10_r05', 'grow_11x14_r10'):
        g = {k.split('/')[1]: torch.from_numpy(z[k]) for k in z.files if k.startswith(case + '/')}
        xd, w1d, b1d, w2d = gpu(g['x'], g['w1'], g['b1'], g['w2'])
        y = ops.step(xd, w1d, b1d, w2d, float(g['rate']), bool(g['growing']), fp32=True, seed=int(g['seed'])).cpu()
        assert O.rel(y, g['y']) < 1e-5, case


# ------------------------------------------------------------------------------------------------ backward
def grads_gpu(ops, x, w1, b1, w2, R, rate, growing, fp32, seed):
    params = [t.clone().requires_grad_() for t in gpu(x, w1, b1, w2)]
    out = ops.step(*params, rate, growing, fp32=fp32, seed=seed)
    return [g.cpu() for g in torch.autograd.grad((out * R.to(DEV)).sum(), params)], out.detach()


def unambiguous(x, w1, b1, R, tf32=True, rel_eps=1e-5):
    """R with zeros at the pixels where some hidden pre-activation lies within fp32 accumulation noise of 0 (relative
    rel_eps of the largest |h| of its NCA): there two correct fp32 summation orders may take different sides of the
    ReLU, so those pixels get no upstream gradient and the comparison does not depend on that choice."""
    K, B, C, H, W = x.shape
    r = O.tf32_round if tf32 else (lambda t: t)
    h = r(w1)[:, None] @ r(O.perceive(x)) + b1[:, None, :, None]          # (K, B, HID, HW)
    scale = h.abs().amax(dim=(1, 2, 3), keepdim=True)
    amb = (h.abs() < rel_eps * scale).any(dim=2).reshape(K, B, 1, H, W)
    return R.masked_fill(amb, 0.0), int(amb.sum())


@pytest.mark.parametrize('C,HID', SIZES)
@pytest.mark.parametrize('rate', [0.5, 1.0])
@pytest.mark.parametrize('growing', [False, True])
def test_backward_parity(ops, C, HID, rate, growing):
    worst = {True: 0.0, False: 0.0}
    for K, B, H, W in BWD_SHAPES:
        x, w1, b1, w2 = O.make(K, B, C, HID, H, W, seed=7 + H, growing=growing)
        R0 = torch.randn(x.shape, generator=torch.Generator().manual_seed(3))
        R, n_amb = unambiguous(x, w1, b1, R0)
        assert n_amb <= 0.05 * K * B * H * W
        mask = O.mask_for(K, B, H, W, 99, rate)
        ref32 = O.step_grads(x, w1, b1, w2, mask, R, growing)
        for fp32 in (True, False):
            got, _ = grads_gpu(ops, x, w1, b1, w2, R, rate, growing, fp32, 99)
            # the backward uses the alive mask of its own forward (kernel alive, exact predicate checked above)
            alive_mask = None
            if growing:
                y, alive = ops._forward(*gpu(x, w1, b1, w2), rate, 99, fp32, True)
                alive_mask = alive.cpu().view(K, B, 1, H, W)
            ref = O.step_backward(x, w1, b1, w2, mask, R, growing, tf32=not fp32, alive_mask=alive_mask)
            for a, b, name in zip(got, ref, ('gx', 'dw1', 'db1', 'dw2')):
                e = O.rel(a, b)
                worst[fp32] = max(worst[fp32], e)
                assert e < (1e-5 if fp32 else 1e-3), (name, fp32, (K, B, H, W), e)
            if not fp32:  # TF32 vs fp32 math (the reference's TF32 bound); growing: same alive mask on both sides
                ref32b = ref32 if not growing else O.step_backward(x, w1, b1, w2, mask, R, True, tf32=False,
                                                                    alive_mask=alive_mask)
                for a, b, name in zip(got, ref32b, ('gx', 'dw1', 'db1', 'dw2')):
                    assert O.rel(a, b) < 3e-2, (name, 'vs fp32', (K, B, H, W))
    print(f'backward {C}/{HID} rate={rate} growing={growing}: worst rel err fp32 {worst[True]:.2e}, '
          f'tf32 {worst[False]:.2e}')
    assert device_error_clear()


def test_backward_matches_reference_golden(ops):
    z = np.load(os.path.join(GOLD, 'reference_step.npz'))
    for case in ('tex_8x16_r05', 'tex_5x37_r05', 'grow_12x10_r05', 'grow_11x14_r10'):
        g = {k.split('/')[1]: torch.from_numpy(z[k]) for k in z.files if k.startswith(case + '/')}
        got, _ = grads_gpu(ops, g['x'], g['w1'], g['b1'], g['w2'], g['R'], float(g['rate']), bool(g['growing']), True,
                           int(g['seed']))
        for a, name in zip(got, ('gx', 'dw1', 'db1', 'dw2')):
            assert O.rel(a, g[name]) < 1e-5, (case, name)


@pytest.mark.parametrize('growing', [False, True])
def test_backward_deterministic_and_chunk_invariant(ops, growing):
    """test_nca.py:57-81,120-122: TF32 gradients are bitwise equal across repeats and CHUNK settings."""
    for K, B in ((32, 1), (16, 2), (5, 1)):
        for C, HID in SIZES:
            x, w1, b1, w2 = O.make(K, B, C, HID, 64, 64, growing=growing)
            R = torch.randn(x.shape, generator=torch.Generator().manual_seed(1))
            for fp32 in (False, True):
                ops.CHUNK = K * B
                ref, _ = grads_gpu(ops, x, w1, b1, w2, R, 0.5, growing, fp32, 99)
                for chunk in (2, K * B // 2, K * B - 1, None):
                    ops.CHUNK = chunk
                    got, _ = grads_gpu(ops, x, w1, b1, w2, R, 0.5, growing, fp32, 99)
                    assert all(torch.equal(a, b) for a, b in zip(ref, got)), (K, B, C, fp32, chunk)
    ops.CHUNK = None


# ------------------------------------------------------------------------------------------------ rollout
@pytest.mark.parametrize('C,HID', SIZES)
@pytest.mark.parametrize('growing', [False, True])
def test_rollout_equals_repeated_steps(ops, C, HID, growing):
    """test_nca.py:128-149: rollout(steps) == repeated step() with step_seed, bitwise; x is not modified."""
    x, w1, b1, w2 = gpu(*O.make(2, 2, C, HID, 37, 50, growing=growing))
    original = x.clone()
    for fp32 in (False, True):
        for rate in (0.0, 0.5, 1.0):
            ref = x
            for steps in range(8):
                if steps:
                    ref = ops.step(ref, w1, b1, w2, rate, growing, fp32, seed=O.step_seed(99, steps - 1))
                assert torch.equal(ops.rollout(x, w1, b1, w2, rate, steps, growing, fp32, seed=99), ref)
    assert torch.equal(x, original)


@pytest.mark.parametrize('C,HID', SIZES)
def test_dying_grid(ops, C, HID):
    """test_nca.py:151-158: the dense living grid dies; both ping-pong buffers must end cleared."""
    x = torch.ones(1, 1, C, 8, 16, device=DEV)
    x[:, :, 3] = 0.2
    w1 = torch.zeros(1, HID, 4 * C, device=DEV)
    b1 = torch.ones(1, HID, device=DEV)
    w2 = torch.full((1, C, HID), 0.01, device=DEV)
    w2[:, 3] = -0.025 / HID
    for fp32 in (False, True):
        y = ops.rollout(x, w1, b1, w2, 1., 7, True, fp32, seed=99)
        assert torch.equal(y, torch.zeros_like(y))


def test_rollout_matches_reference_golden(ops):
    z = np.load(os.path.join(GOLD, 'reference_step.npz'))
    for case in ('roll_tex', 'roll_grow'):
        g = {k.split('/')[1]: torch.from_numpy(z[k]) for k in z.files if k.startswith(case + '/')}
        xd, w1d, b1d, w2d = gpu(g['x'], g['w1'], g['b1'], g['w2'])
        for steps in range(1, 5):
            y = ops.rollout(xd, w1d, b1d, w2d, float(g['rate']), steps, bool(g['growing']), True, seed=int(g['seed']))
            assert O.rel(y.cpu(), g['ys'][steps - 1]) < 1e-5, (case, steps)


# ------------------------------------------------------------------------------------------------ sharding offset
def test_image_offset_reproduces_single_gpu_shard(ops):
    """A shard holding NCAs [1, 3) with image_offset = 1 * B computes exactly those NCAs of the full step."""
    x, w1, b1, w2 = gpu(*O.make(4, 2, 12, 96, 32, 32))
    full = ops.step(x, w1, b1, w2, 0.5, seed=5)
    part = ops.step(x[1:3], w1[1:3], b1[1:3], w2[1:3], 0.5, seed=5, image_offset=2)
    assert torch.equal(full[1:3], part)
    R = torch.randn(x.shape, device=DEV)
    ps = [t.clone().requires_grad_() for t in (x, w1, b1, w2)]
    gf = torch.autograd.grad((ops.step(*ps, 0.5, seed=5) * R).sum(), ps)
    qs = [t[1:3].clone().requires_grad_() for t in (x, w1, b1, w2)]
    gp = torch.autograd.grad((ops.step(*qs, 0.5, seed=5, image_offset=2) * R[1:3]).sum(), qs)
    assert torch.equal(gf[0][1:3], gp[0])
    for a, b in zip(gf[1:], gp[1:]):
        assert O.rel(b.cpu(), a[1:3].cpu()) < 1e-5


# ------------------------------------------------------------------------------------------------ loss + optimiser
def test_synthetic_loss(ops):
    from ultranca_b200 import training
    x, w1, b1, w2, target = O.make_config_inputs(3, 2, 12, 96, 40, 24)
    x = x * 30
    obj_ref, per_ref = O.synthetic_loss(x, target)
    xr = x.clone().requires_grad_()
    (g_ref,) = torch.autograd.grad(O.synthetic_loss(xr, target)[0], xr)
    loss, gy = training.synthetic_loss(x.to(DEV), target.to(DEV))
    assert O.rel(loss.cpu(), per_ref) < 1e-5
    assert O.rel(gy.cpu(), g_ref) < 1e-6


def test_fused_adam_matches_torch(ops):
    from ultranca_b200 import training
    z = np.load(os.path.join(GOLD, 'reference_step.npz'))
    g = {k.split('/')[1]: torch.from_numpy(z[k]) for k in z.files if k.startswith('adam/')}
    params = gpu(g['w1'], g['b1'], g['w2'])
    opt = training.FusedAdam(params, lr=float(g['lr']), milestones=g['milestones'].tolist(), gamma=float(g['gamma']))
    for i in range(g['g_w1'].shape[0]):
        opt.step(gpu(g['g_w1'][i], g['g_b1'][i], g['g_w2'][i]))
        for p, name in zip(params, ('w1_after', 'b1_after', 'w2_after')):
            assert O.rel(p.cpu(), g[name][i]) < 1e-6, (i, name)


@pytest.mark.parametrize('rate', [0.02, 0.1, 0.3, 0.9])
@pytest.mark.parametrize('K,B,H,W', [(2, 2, 1, 128), (3, 1, 2, 8), (2, 3, 3, 4), (4, 2, 16, 128), (1, 2, 64, 124)])
def test_row_forward_sparse_tiles(ops, rate, K, B, H, W):
    """The row forward queues the updating pixels into tiles of up to 128 over at most 4 rows: low rates (tiles over
    many sparse rows), one- to three-row images (every row a segment with wrapped halos), narrow rows. Updating
    pixels match the TF32 oracle; the others are copied exactly."""
    C, HID = 12, 96
    assert ops.launch_info(C, HID, False, K * B, H, W, K)['rows_path'] == 1
    x, w1, b1, w2 = O.make(K, B, C, HID, H, W, seed=7 * H + W)
    mask = O.mask_for(K, B, H, W, 99, rate)
    out = ops.step(*gpu(x, w1, b1, w2), rate, seed=99).cpu()
    ref = O.reference_step(x, w1, b1, w2, mask, False, tf32=True)
    keep = (mask == 0).expand_as(x)
    assert torch.equal(out[keep], x[keep])
    assert O.rel(out, ref) < 1e-3
    assert device_error_clear()


@pytest.mark.parametrize('K,B,H,W', [(400, 2, 4, 32), (160, 8, 128, 8)])
def test_row_forward_many_segments_and_grown_grid(ops, K, B, H, W):
    """Bands of several segments (4-row images, two or three NCAs per band: weights restaged, ring and queue kept per
    segment), and more rows than 148 CTAs of MAXROWS rows hold (the grid grows)."""
    C, HID = 12, 96
    info = ops.launch_info(C, HID, False, K * B, H, W, K)
    assert info['rows_path'] == 1
    if K * B * H > 148 * 1024:
        assert info['fwd_grid'] > 148
    x, w1, b1, w2 = O.make(K, B, C, HID, H, W, seed=3)
    mask = O.mask_for(K, B, H, W, 5, 0.5)
    out = ops.step(*gpu(x, w1, b1, w2), 0.5, seed=5).cpu()
    ref = O.reference_step(x, w1, b1, w2, mask, False, tf32=True)
    assert O.rel(out, ref) < 1e-3
    assert device_error_clear()


def test_row_backward_many_segments(ops):
    """Backward bands over many 4-row images and two or three NCAs each (the weight-gradient accumulator flushed to a
    new partial slot and the weights restaged at every NCA switch, halo rows at every image switch; the cost-balanced
    bands differ from the uniform split): TF32 gradients vs the TF32 oracle."""
    C, HID, K, B, H, W = 12, 96, 300, 2, 4, 32
    assert ops.launch_info(C, HID, False, K * B, H, W, K)['rows_path'] == 1
    x, w1, b1, w2 = O.make(K, B, C, HID, H, W, seed=11)
    R0 = torch.randn(x.shape, generator=torch.Generator().manual_seed(4))
    R, n_amb = unambiguous(x, w1, b1, R0)
    mask = O.mask_for(K, B, H, W, 77, 0.5)
    got, _ = grads_gpu(ops, x, w1, b1, w2, R, 0.5, False, False, 77)
    ref = O.step_backward(x, w1, b1, w2, mask, R, False, tf32=True)
    for a, b, name in zip(got, ref, ('gx', 'dw1', 'db1', 'dw2')):
        assert O.rel(a, b) < 1e-3, name
    assert device_error_clear()


@pytest.mark.parametrize('K,B,H,W,rate', [(2, 1, 6, 256, 0.5), (1, 2, 5, 384, 0.5), (2, 1, 1, 256, 1.0),
                                          (1, 1, 3, 512, 0.3), (3, 2, 7, 256, 0.5), (40, 2, 4, 256, 0.5)])
def test_strip_backward_parity(ops, K, B, H, W, rate):
    """Rows wider than 128 (W = 128 S) run the backward row kernel over column strips of 128 with the cross-strip
    adjoint terms added by the edge fix-up: TF32 gradients vs the TF32 oracle, on the whole of gx and on the strip edge
    columns alone (where the fix-up adds), at two to four strips, one-row images, a rate of 1 and bands of many 4-row
    images over several NCAs; repeated calls are bitwise equal."""
    C, HID = 12, 96
    assert ops.launch_info(C, HID, False, K * B, H, W, K)['rows_path'] == 2
    x, w1, b1, w2 = O.make(K, B, C, HID, H, W, seed=5 * H + W + K)
    R0 = torch.randn(x.shape, generator=torch.Generator().manual_seed(6))
    R, n_amb = unambiguous(x, w1, b1, R0)
    assert n_amb <= 0.05 * K * B * H * W
    mask = O.mask_for(K, B, H, W, 31, rate)
    got, _ = grads_gpu(ops, x, w1, b1, w2, R, rate, False, False, 31)
    ref = O.step_backward(x, w1, b1, w2, mask, R, False, tf32=True)
    for a, b, name in zip(got, ref, ('gx', 'dw1', 'db1', 'dw2')):
        assert O.rel(a, b) < 1e-3, (name, O.rel(a, b))
    edges = [c for s in range(W // 128) for c in (128 * s, 128 * s + 127)]
    assert O.rel(got[0][..., edges], ref[0][..., edges]) < 1e-3
    again, _ = grads_gpu(ops, x, w1, b1, w2, R, rate, False, False, 31)
    assert all(torch.equal(a, b) for a, b in zip(got, again))
    assert device_error_clear()


@pytest.mark.parametrize('K,B,H,W,rate', [(2, 1, 6, 256, 0.5), (1, 2, 5, 384, 0.3), (2, 1, 1, 256, 1.0),
                                          (1, 1, 3, 512, 0.02), (40, 2, 4, 256, 0.5), (1, 2, 130, 256, 0.9)])
def test_strip_forward_parity(ops, K, B, H, W, rate):
    """Rows wider than 128 run the row forward over column strips of 128 (masks, prefix counts and tiles per strip;
    4 halo columns on each side of a strip, wrapped at the row's ends): updating pixels match the TF32 oracle, the
    others are copied exactly; two to four strips, one-row images, rates 0.02 to 1, many images and NCAs per band."""
    C, HID = 12, 96
    assert ops.launch_info(C, HID, False, K * B, H, W, K)['rows_path'] == 2
    x, w1, b1, w2 = O.make(K, B, C, HID, H, W, seed=3 * H + W + K)
    mask = O.mask_for(K, B, H, W, 41, rate)
    out = ops.step(*gpu(x, w1, b1, w2), rate, seed=41).cpu()
    ref = O.reference_step(x, w1, b1, w2, mask, False, tf32=True)
    keep = (mask == 0).expand_as(x)
    assert torch.equal(out[keep], x[keep])
    assert O.rel(out, ref) < 1e-3
    edges = [c for s in range(W // 128) for c in (128 * s, 128 * s + 127)]
    assert O.rel(out[..., edges], ref[..., edges]) < 1e-3
    assert device_error_clear()


def test_strip_rollout_equals_repeated_steps(ops):
    """rollout() over column strips equals repeated step() calls bitwise, x unmodified (test_nca.py:128-149)."""
    x, w1, b1, w2 = gpu(*O.make(2, 2, 12, 96, 9, 256, seed=8))
    original = x.clone()
    for rate in (0.5, 1.0):
        ref = x
        for steps in range(5):
            if steps:
                ref = ops.step(ref, w1, b1, w2, rate, seed=O.step_seed(123, steps - 1))
            assert torch.equal(ops.rollout(x, w1, b1, w2, rate, steps, seed=123), ref)
    assert torch.equal(x, original)
    assert device_error_clear()


@pytest.mark.parametrize('fp32', [False, True])
def test_growing_sparse_seed(ops, fp32):
    """Growing NCAs from single live seed cells (the start state of BASELINE config 2: channels 3.. = 1 at one cell,
    16 channels / 128 hidden, 72 x 72), where most tiles are dead and skipped (forward: no cell within two pixels alive
    before the step; backward and adjoint: no alive cell). Over 6 steps: the step output is exactly the dense update
    times the exact alive mask, the dense update matches the oracle; then the gradients of the last step match the
    oracle, and rollout() equals the repeated steps bitwise."""
    C, HID, K, B, H, W = 16, 128, 2, 2, 72, 72
    x = torch.zeros(K, B, C, H, W)
    x[:, :, 3:, H // 2, W // 2] = 1.0
    x[:, 1, 3:, 5, 66] = 1.0  # a second seed near the top-right border
    _, w1, b1, w2 = O.make(K, B, C, HID, 4, 4, seed=21)
    w1d, b1d, w2d = gpu(w1, b1, w2)
    cur = x
    tol = 1e-5 if fp32 else 1e-3
    for i in range(6):
        seed = O.step_seed(17, i)
        xd = cur.to(DEV)
        out = ops.step(xd, w1d, b1d, w2d, 0.5, True, fp32=fp32, seed=seed).cpu()
        raw = ops.step(xd, w1d, b1d, w2d, 0.5, False, fp32=fp32, seed=seed).cpu()
        assert torch.equal(out, raw * (O.alive(cur) & O.alive(raw))), i
        ref_raw = O.reference_step(cur, w1, b1, w2, O.mask_for(K, B, H, W, seed, 0.5), False, tf32=not fp32)
        assert O.rel(raw, ref_raw) < tol, i
        cur = out
    assert (cur[:, :, 3] > 0.1).any()  # still alive somewhere
    roll = ops.rollout(x.to(DEV), w1d, b1d, w2d, 0.5, 6, True, fp32, seed=17).cpu()
    assert torch.equal(roll, cur)
    # gradients of one step from the grown state
    R0 = torch.randn(cur.shape, generator=torch.Generator().manual_seed(9))
    R, _ = unambiguous(cur, w1, b1, R0, tf32=not fp32)
    got, _ = grads_gpu(ops, cur, w1, b1, w2, R, 0.5, True, fp32, 23)
    _, alive = ops._forward(*gpu(cur, w1, b1, w2), 0.5, 23, fp32, True)
    ref = O.step_backward(cur, w1, b1, w2, O.mask_for(K, B, H, W, 23, 0.5), R, True, tf32=not fp32,
                          alive_mask=alive.cpu().view(K, B, 1, H, W))
    for a_, b_, name in zip(got, ref, ('gx', 'dw1', 'db1', 'dw2')):
        assert O.rel(a_, b_) < tol, (name, O.rel(a_, b_))
    assert device_error_clear()
