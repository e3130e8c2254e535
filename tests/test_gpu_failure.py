"""GPU failure detection without a fault: a bounded device wait that runs out.

Every mbarrier wait of the step kernels is bounded; a kernel whose wait runs out makes the CTA's other warps give up
too (a shared abort word), frees its Tensor Memory, sets the device error word and returns, so the context stays
usable. nca_wait_selftest runs that path on an mbarrier that nothing arrives on: the test checks that the kernel
returns after the short limit, that the second warp followed the abort instead of waiting out its own 2 s limit, that
nca_device_error reports code 1, and that a normal step run afterwards still matches the oracle.
"""
import ctypes

import pytest
import torch

from oracle import nca_oracle as O

pytestmark = pytest.mark.gpu


def test_bounded_wait_runs_out_and_the_context_stays_usable():
    from ultranca_b200 import nca_ops
    from ultranca_b200._lib import check, lib, ptr
    code = ctypes.c_int()
    check(lib.nca_device_error(ctypes.byref(code), 1))  # start from a clear error word
    out = torch.full((4,), -1, dtype=torch.int64, device='cuda')
    st = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    limit_ns = 1_000_000  # 1 ms
    check(lib.nca_wait_selftest(limit_ns, ptr(out), st))
    torch.cuda.synchronize()  # returns: the kernel did not hang
    t0, ok0, t1, ok1 = out.tolist()
    assert ok0 == 0 and ok1 == 0, 'a wait on a barrier nothing arrives on must report failure'
    assert limit_ns <= t0 < 100 * limit_ns, t0  # gave up after its own limit
    assert t1 < 200 * limit_ns, t1  # the other warp followed the abort, not its own 2 s limit
    check(lib.nca_device_error(ctypes.byref(code), 1))
    assert code.value == 1
    check(lib.nca_device_error(ctypes.byref(code), 0))
    assert code.value == 0  # cleared by the read above

    # the context is still usable: a step and its gradients match the oracle
    K, B, C, HID, H, W = 2, 2, 12, 96, 24, 32
    x, w1, b1, w2 = O.make(K, B, C, HID, H, W, seed=12)
    R = torch.randn(x.shape, generator=torch.Generator().manual_seed(13))
    mask = O.mask_for(K, B, H, W, 55, 0.5)
    params = [t.cuda().requires_grad_() for t in (x, w1, b1, w2)]
    y = nca_ops.step(*params, 0.5, seed=55)
    grads = torch.autograd.grad((y * R.cuda()).sum(), params)
    torch.cuda.synchronize()
    assert O.rel(y.detach().cpu(), O.reference_step(x, w1, b1, w2, mask, tf32=True)) < 1e-3
    ref = O.step_backward(x, w1, b1, w2, mask, R, tf32=True)
    for a, b in zip(grads, ref):
        assert O.rel(a.cpu(), b) < 1e-3
    check(lib.nca_device_error(ctypes.byref(code), 0))
    assert code.value == 0

