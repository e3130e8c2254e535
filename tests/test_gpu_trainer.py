"""GPU: the training iteration's rollout backward (every step adds its weight-gradient partials to the workspace, one
reduce at the end: NCA_STAGE_PARTIAL_ADD) gives the gradient that per-step autograd through nca_ops.step gives. Both run
the same TF32 kernels; only the order of the weight-gradient sums differs. Row-streaming path, tile path (W not a
multiple of 4) and a growing NCA (tile path, alive masks)."""
import pytest
import torch

from oracle import nca_oracle as O

pytestmark = pytest.mark.gpu

CASES = [(2, 2, 12, 96, 24, 32, False), (2, 2, 12, 96, 17, 30, False), (2, 2, 16, 128, 20, 20, True)]


@pytest.mark.parametrize('K,B,C,HID,H,W,growing', CASES)
def test_rollout_trainer_gradient_matches_stepwise_autograd(K, B, C, HID, H, W, growing):
    from ultranca_b200 import nca_ops, training
    steps, rate, seed = 5, 0.5, 321
    x, w1, b1, w2 = (t.cuda() for t in O.make(K, B, C, HID, H, W, seed=4, growing=growing))
    target = (torch.rand(K, 3, H, W, generator=torch.Generator().manual_seed(6)) - 0.5).cuda()
    tr = training.RolloutTrainer(w1.clone(), b1.clone(), w2.clone(), B, H, W, steps, rate, growing=growing)
    tr.states[0].copy_(x)
    tr.forward_steps(seed, steps)
    training.synthetic_loss(tr.states[steps], target, tr.overflow_weight, tr.gy[0], tr.loss, tr.loss_work)
    tr.backward_steps(seed, tr.gy[0], steps)
    got = [g.clone() for g in tr.grads]

    params = [t.clone().requires_grad_() for t in (w1, b1, w2)]
    s = x.clone()
    for i in range(steps):
        s = nca_ops.step(s, *params, rate, growing, fp32=False, seed=nca_ops.step_seed(seed, i))
    _, gy = training.synthetic_loss(s.detach(), target, tr.overflow_weight)
    ref = torch.autograd.grad((s * gy).sum(), params)
    torch.cuda.synchronize()
    assert torch.equal(tr.states[steps], s.detach()), 'the trainer and the operator API run the same forward'
    for a, b, name in zip(got, ref, ('dw1', 'db1', 'dw2')):
        e = O.rel(a.cpu(), b.cpu())
        assert e < 1e-4, (name, (K, B, C, HID, H, W, growing), e)
