"""GPU: the sm_100a kernels against the reference's OWN CUDA kernels (ncaops/nca_step.cuh, compiled unchanged for
sm_100a into oracle/_ref by oracle/build_ref.py) on the same B200: the Philox update mask bit for bit, the forward and
the gradients within TF32 tolerance. Skipped when oracle/_ref was not built (no reference checkout)."""
import pytest
import torch

from oracle import nca_oracle as O
from oracle import ref_kernels as R

pytestmark = [pytest.mark.gpu, pytest.mark.skipif(not R.available(), reason='oracle/_ref not built')]


@pytest.fixture(scope='module')
def ops():
    from ultranca_b200 import nca_ops
    return nca_ops


@pytest.mark.parametrize('n,h,w,seed,rate', [(4, 128, 128, 7, 0.5), (3, 37, 50, 1234, 0.5), (2, 9, 13, 2 ** 62 - 1, 0.3),
                                             (17, 129, 65, 99, 0.5), (1, 8, 16, 5, 1.0)])
def test_mask_equals_reference_mask_kernel(ops, n, h, w, seed, rate):
    ours = ops.update_mask(n, h, w, seed, rate)
    ref = R.update_mask(n, h, w, seed, rate)
    torch.cuda.synchronize()
    assert torch.equal(ours, ref)


@pytest.mark.parametrize('C,HID', [(12, 96), (16, 128)])
@pytest.mark.parametrize('growing', [False, True])
@pytest.mark.parametrize('rate', [0.5, 1.0])
def test_forward_matches_reference_kernel(ops, C, HID, growing, rate):
    for K, B, H, W in ((3, 2, 128, 128), (2, 3, 37, 50), (1, 1, 8, 16)):
        x, w1, b1, w2 = (t.cuda() for t in O.make(K, B, C, HID, H, W, seed=5, growing=growing))
        for fp32 in (False, True):
            ours = ops.step(x, w1, b1, w2, rate, growing, fp32=fp32, seed=1234)
            ref, _ = R.forward(x, w1, b1, w2, rate, 1234, fp32=fp32, growing=growing)
            torch.cuda.synchronize()
            if growing:  # compare away from alive-bit flips (TF32 rounding differs between the two kernels)
                keep = (ours != 0) == (ref != 0)
                ours, ref = ours * keep, ref * keep
            assert O.rel(ours.cpu(), ref.cpu()) < (1e-5 if fp32 else 1e-3), (C, growing, rate, fp32, (K, B, H, W))


@pytest.mark.parametrize('C,HID', [(12, 96), (16, 128)])
def test_gradients_match_reference_kernel(ops, C, HID):
    from test_gpu_parity import unambiguous
    for K, B, H, W in ((3, 2, 64, 64), (2, 3, 37, 50)):
        x, w1, b1, w2 = O.make(K, B, C, HID, H, W, seed=8)
        Rg, _ = unambiguous(x, w1, b1, torch.randn(x.shape, generator=torch.Generator().manual_seed(9)))
        xd, w1d, b1d, w2d, gy = (t.cuda() for t in (x, w1, b1, w2, Rg))
        for fp32 in (False, True):
            params = [t.clone().requires_grad_() for t in (xd, w1d, b1d, w2d)]
            out = ops.step(*params, 0.5, False, fp32=fp32, seed=99)
            ours = torch.autograd.grad((out * gy).sum(), params)
            ref = R.Backward(K, B, C, HID, H, W, 0.5, fp32=fp32)(xd, gy, None, w1d, b1d, w2d, 99)
            torch.cuda.synchronize()
            if fp32:  # fp32 mode: both are checked against the fp32 oracle; ours must be at least as close as the reference
                ref32 = O.step_grads(x, w1, b1, w2, O.mask_for(K, B, H, W, 99, 0.5), Rg)
                for a, b, r32, name in zip(ours, ref, ref32, ('gx', 'dw1', 'db1', 'dw2')):
                    e_ours, e_ref = O.rel(a.cpu(), r32), O.rel(b.cpu(), r32)
                    assert e_ours < 1e-5 and e_ours <= max(e_ref, 1e-6), (name, (K, B, H, W), e_ours, e_ref)
                continue
            for a, b, name in zip(ours, ref, ('gx', 'dw1', 'db1', 'dw2')):
                assert O.rel(a.cpu(), b.cpu()) < 1e-3, (name, fp32, (K, B, H, W))
