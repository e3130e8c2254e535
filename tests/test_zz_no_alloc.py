"""GPU: nca_backward_static_scratch (the row-kernel backward whose scratch is a library-owned device array, for callers
that cannot allocate device memory) against nca_backward with a caller-allocated workspace, through the C-ABI.

Two calls in a row on different inputs and shapes: the second call reuses the array the first one left behind, so a
slot that the second call read without writing would show up here. Collected last (file name), and independent of
every other test module, so that it passes in a fresh process as well as after the whole suite."""
import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu

TOL = 1e-3  # TF32 tolerance of the parity tests; both paths run the same kernels, so in practice they agree bitwise


def rel(a, b):
    return float((a - b).abs().max() / b.abs().max().clamp_min(1e-30))


def inputs(K, B, H, W, seed):
    g = torch.Generator().manual_seed(seed)
    C, HID = 12, 96
    x = torch.rand(K * B, C, H, W, generator=g) * 2 - 1
    gy = torch.randn(K * B, C, H, W, generator=g)
    w1 = torch.randn(K, HID, 4 * C, generator=g) * 0.2
    b1 = torch.randn(K, HID, generator=g) * 0.1
    w2 = torch.randn(K, C, HID, generator=g) * 0.1
    return [t.cuda() for t in (x, gy, w1, b1, w2)]


def outputs(x, w1, b1, w2, init):
    """gx (never read by either entry point) and the weight gradients; init: values the weight gradients start from
    (accumulate = 1 adds to them), or None."""
    gx = torch.full_like(x, float('nan'))
    grads = [torch.full_like(t, float('nan')) if init is None else i.clone() for t, i in
             zip((w1, b1, w2), init if init is not None else (None,) * 3)]
    return [gx] + grads


def with_workspace(lib, P, x, gy, w1, b1, w2, K, B, seed, rate, st, offset=0, init=None):
    N, C, H, W = x.shape
    HID = w1.shape[1]
    dpf, pf, ch = ctypes.c_int64(), ctypes.c_int64(), ctypes.c_int64()
    assert lib.nca_backward_workspace(C, HID, 0, N, H, W, K, rate, 0, ctypes.byref(dpf), ctypes.byref(pf),
                                      ctypes.byref(ch)) == 0
    dp, partial = torch.empty(dpf.value, device='cuda'), torch.empty(pf.value, device='cuda')
    out = outputs(x, w1, b1, w2, init)
    assert lib.nca_backward(P(x), P(gy), None, P(w1), P(b1), P(w2), *map(P, out), P(dp), dpf.value, P(partial),
                            pf.value, N, C, H, W, K, HID, B, seed, rate, 0, 0, offset, int(init is not None),
                            st) == 0, lib.nca_last_error()
    return out


def static_scratch(lib, P, x, gy, w1, b1, w2, K, B, seed, rate, st, offset=0, init=None):
    N, C, H, W = x.shape
    out = outputs(x, w1, b1, w2, init)
    assert lib.nca_backward_static_scratch(P(x), P(gy), P(w1), P(b1), P(w2), *map(P, out), N, C, H, W, K, w1.shape[1],
                                           B, seed, rate, offset, int(init is not None), st) == 0, lib.nca_last_error()
    return out


def test_static_scratch_backward_matches_workspace_backward_twice():
    from ultranca_b200._lib import lib, ptr as P
    st = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    # the larger case first, so that the second call finds more stale slots in the array than it writes
    for K, B, H, W, seed, rate in ((5, 3, 96, 128, 7, 0.5), (2, 2, 37, 40, 2 ** 62 + 11, 0.75)):
        x, gy, w1, b1, w2 = inputs(K, B, H, W, seed)
        ref = with_workspace(lib, P, x, gy, w1, b1, w2, K, B, seed, rate, st)
        got = static_scratch(lib, P, x, gy, w1, b1, w2, K, B, seed, rate, st)
        torch.cuda.synchronize()
        for a, b, name in zip(got, ref, ('gx', 'dw1', 'db1', 'dw2')):
            assert torch.isfinite(a).all(), (name, (K, B, H, W))
            assert rel(a, b) < TOL, (name, (K, B, H, W), rel(a, b))


def test_static_scratch_backward_accumulates_and_follows_the_shard_offset():
    """accumulate = 1 adds the step's weight gradients to the values the outputs hold (the autograd accumulation of a
    rollout), and a nonzero image offset (a shard of a multi-GPU job) selects the shard's update masks: both as the
    workspace backward does, with outputs pre-filled with the same values on both paths."""
    from ultranca_b200._lib import lib, ptr as P
    st = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    K, B, H, W, seed, rate, offset = 3, 2, 40, 64, 12345, 0.5, 6
    x, gy, w1, b1, w2 = inputs(K, B, H, W, seed)
    g = torch.Generator().manual_seed(5)
    init = [torch.randn(t.shape, generator=g).cuda() for t in (w1, b1, w2)]
    for off, acc in ((offset, None), (offset, init), (0, init)):
        ref = with_workspace(lib, P, x, gy, w1, b1, w2, K, B, seed, rate, st, off, acc)
        got = static_scratch(lib, P, x, gy, w1, b1, w2, K, B, seed, rate, st, off, acc)
        torch.cuda.synchronize()
        for a, b, name in zip(got, ref, ('gx', 'dw1', 'db1', 'dw2')):
            assert torch.isfinite(a).all(), (name, off, acc is not None)
            assert rel(a, b) < TOL, (name, off, acc is not None, rel(a, b))
    # the offset changes the masks (the case above is not the unsharded one) and accumulation adds the init values
    plain = with_workspace(lib, P, x, gy, w1, b1, w2, K, B, seed, rate, st, 0, None)
    shifted = with_workspace(lib, P, x, gy, w1, b1, w2, K, B, seed, rate, st, offset, None)
    added = with_workspace(lib, P, x, gy, w1, b1, w2, K, B, seed, rate, st, 0, init)
    torch.cuda.synchronize()
    assert not torch.equal(plain[0], shifted[0])
    for a, b, i in zip(added[1:], plain[1:], init):
        assert rel(a - i, b) < 1e-5


def test_static_scratch_backward_rejects_what_it_cannot_hold():
    from ultranca_b200._lib import lib
    bogus = ctypes.c_void_p(256)  # never dereferenced: every case below is rejected before any launch
    args = lambda N, C, H, W, K, HID: (bogus,) * 9 + (N, C, H, W, K, HID, N // K, 1, 0.5, 0, 0, None)
    assert lib.nca_backward_static_scratch(*args(4000, 12, 8, 8, 4000, 96)) == 2  # NCA_ERR_SHAPE: too many NCAs
    assert 'static array holds' in lib.nca_last_error().decode()
    assert lib.nca_backward_static_scratch(*args(4, 16, 8, 8, 2, 128)) == 3  # NCA_ERR_UNSUPPORTED: growing sizes
    assert lib.nca_backward_static_scratch(*args(4, 12, 8, 6, 2, 96)) == 3  # W not a multiple of 4
