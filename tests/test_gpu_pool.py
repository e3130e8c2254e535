"""Device-driven training iteration (train.py:126-142 on the device): pool sampling with seed injection, device-read
step seeds, the fused reduce + Adam launch, pool write-back, and CUDA-graph replay of the whole iteration.

Random draws (pool entries, rollout seeds) are this library's own, so they are checked by their properties (distinct
entries in range, injection on the right iterations) and the rest against the host-driven path on the same draws."""
import pytest
import torch

from oracle import nca_oracle as O

pytestmark = pytest.mark.gpu


def _setup(K=2, B=2, C=12, HID=96, H=16, W=32, steps=3, P=6, seed=5, growing=False):
    from ultranca_b200 import training
    x, w1, b1, w2 = (t.cuda() for t in O.make(K, B, C, HID, H, W, seed=seed))
    g = torch.Generator().manual_seed(seed)
    pool = ((torch.rand(K, P, C, H, W, generator=g) * 2 - 1) * 0.1).cuda()
    target = (torch.rand(K, 3, H, W, generator=g) - 0.5).cuda()
    tr = training.RolloutTrainer(w1.clone(), b1.clone(), w2.clone(), B, H, W, steps, 0.5, growing=growing,
                                 milestones=(2, 4), gamma=0.5)
    return tr, pool, target


def test_pool_sample_distinct_entries_and_injection():
    from ultranca_b200 import training
    from ultranca_b200._lib import check, lib, ptr
    K, P, B, C, H, W = 5, 9, 4, 16, 10, 12
    pool = torch.randn(K, P, C, H, W, device='cuda')
    ctl = torch.zeros(4, dtype=torch.int64, device='cuda')
    ctl[0] = 1234
    idx = torch.empty(K * B, dtype=torch.int64, device='cuda')
    x0 = torch.empty(K, B, C, H, W, device='cuda')
    seen = set()
    for it in range(6):
        st = torch.cuda.current_stream().cuda_stream
        check(lib.nca_control_advance(ptr(ctl), st))
        check(lib.nca_pool_sample(ptr(pool), ptr(x0), ptr(idx), ptr(ctl), K, P, B, C, H, W, 3, training.SEED_GROWING,
                                  0, st))
        if it == 1:  # a shard holding NCAs 2.. draws what the whole job draws for them
            idx2 = torch.empty((K - 2) * B, dtype=torch.int64, device='cuda')
            x2 = torch.empty(K - 2, B, C, H, W, device='cuda')
            check(lib.nca_pool_sample(ptr(pool[2:]), ptr(x2), ptr(idx2), ptr(ctl), K - 2, P, B, C, H, W, 3,
                                      training.SEED_GROWING, 2, st))
            torch.cuda.synchronize()
            assert torch.equal(idx2, idx[2 * B:])
        torch.cuda.synchronize()
        assert int(ctl[2]) == it and int(ctl[1]) == it + 1
        ix = idx.view(K, B).cpu()
        assert ((ix >= 0) & (ix < P)).all()
        for k in range(K):
            assert len(set(ix[k].tolist())) == B  # B distinct entries per NCA
            seen.add(tuple(ix[k].tolist()))
            for b in range(B):
                if b == 0 and it % 3 == 0:  # the growing seed: 1 in channels 3.. at the centre, else 0
                    ref = torch.zeros(C, H, W, device='cuda')
                    ref[3:, H // 2, W // 2] = 1
                    assert torch.equal(x0[k, b], ref)
                else:
                    assert torch.equal(x0[k, b], pool[k, ix[k, b]])
    assert len(seen) > 10  # the draws change between iterations and NCAs


def test_pool_store_writes_back():
    from ultranca_b200._lib import check, lib, ptr
    K, P, B, C, H, W = 3, 7, 2, 12, 8, 8
    pool = torch.randn(K, P, C, H, W, device='cuda')
    before = pool.clone()
    x = torch.randn(K, B, C, H, W, device='cuda')
    idx = torch.tensor([[4, 1], [0, 6], [3, 2]], dtype=torch.int64, device='cuda').view(-1)
    check(lib.nca_pool_store(ptr(pool), ptr(x), ptr(idx), K, P, B, C, H, W, torch.cuda.current_stream().cuda_stream))
    torch.cuda.synchronize()
    expect = before.clone()
    for k in range(K):
        for b in range(B):
            expect[k, idx.view(K, B)[k, b]] = x[k, b]
    assert torch.equal(pool, expect)


def test_device_seed_equals_host_seed():
    """Steps launched with the rollout seed in device memory equal those given the seed by the host."""
    tr, pool, target = _setup()
    seed = 0x1234567890ABCDEF
    x0 = pool[:, :2].contiguous()
    tr.states[0].copy_(x0)
    tr.forward_steps(seed, 3)
    host = tr.states.clone()
    gx_host = tr.backward_steps(seed, host[3] * 0 + 0.5, 3).clone()
    g_host = [g.clone() for g in tr.grads]
    sd = torch.tensor([seed if seed < (1 << 63) else seed - (1 << 64)], dtype=torch.int64, device='cuda')
    tr.states.zero_()
    tr.states[0].copy_(x0)
    tr.forward_steps(None, 3, seed_dev=sd.data_ptr())
    assert torch.equal(tr.states, host)
    gx_dev = tr.backward_steps(None, host[3] * 0 + 0.5, 3, seed_dev=sd.data_ptr())
    assert torch.equal(gx_dev, gx_host)
    for a, b in zip(tr.grads, g_host):
        assert torch.equal(a, b)


@pytest.mark.parametrize('shape', [(2, 2, 12, 96, 16, 32), (2, 2, 12, 96, 20, 36), (2, 1, 16, 128, 12, 12)])
def test_fused_reduce_adam_equals_reduce_then_adam(shape):
    K, B, C, HID, H, W = shape
    growing = C == 16
    a, pool, target = _setup(K, B, C, HID, H, W, growing=growing)
    b, _, _ = _setup(K, B, C, HID, H, W, growing=growing)
    x0 = pool[:, :B].contiguous()
    for it in range(3):
        a.iteration(x0, target, seed=77 + it, fused=True)
        b.iteration(x0, target, seed=77 + it, fused=False)
    torch.cuda.synchronize()
    for p, q in ((a.w1, b.w1), (a.b1, b.b1), (a.w2, b.w2), *zip(a.opt.m + a.opt.v, b.opt.m + b.opt.v)):
        assert torch.equal(p, q)
    assert int(a.opt.iteration) == int(b.opt.iteration) == 3


def test_pool_iteration_equals_host_driven_iteration():
    """One device-driven iteration equals RolloutTrainer.iteration on the batch it sampled and the seed it drew."""
    from ultranca_b200 import training
    a, pool_a, target = _setup()
    b, pool_b, _ = _setup()
    pt = training.PoolTrainer(a, pool_a, target, inject_every=2, key=99, graph=False)
    pool_before = pool_b.clone()
    pt.iteration()
    torch.cuda.synchronize()
    idx = pt.idx.view(a.K, a.B).cpu()
    seed = int(pt.ctl[3]) & (2 ** 64 - 1)
    x0 = torch.stack([pool_before[k, idx[k]] for k in range(a.K)])
    x0[:, 0] = 0.0  # iteration 0 injects the texture seed (zeros)
    b.iteration(x0, target, seed=seed)
    torch.cuda.synchronize()
    for p, q in ((a.w1, b.w1), (a.b1, b.b1), (a.w2, b.w2)):
        assert torch.equal(p, q)
    expect = pool_before.clone()
    for k in range(a.K):
        for j in range(a.B):
            expect[k, idx[k, j]] = b.states[a.steps][k, j]
    assert torch.equal(pool_a, expect)


def test_graph_replay_equals_direct_launches():
    from ultranca_b200 import training
    a, pool_a, target = _setup()
    b, pool_b, _ = _setup()
    direct = training.PoolTrainer(a, pool_a, target, inject_every=3, key=7, graph=False)
    graphed = training.PoolTrainer(b, pool_b, target, inject_every=3, key=7, graph=True)
    for it, n in enumerate((3, 3, 2, 3, 2, 3)):
        la = direct.iteration(n).clone()
        lb = graphed.iteration(n).clone()
        assert torch.equal(la, lb), it
    torch.cuda.synchronize()
    assert sorted(graphed.graphs) == [2, 3]
    for p, q in ((a.w1, b.w1), (a.b1, b.b1), (a.w2, b.w2), (pool_a, pool_b), (direct.ctl, graphed.ctl),
                 *zip(a.opt.m + a.opt.v, b.opt.m + b.opt.v)):
        assert torch.equal(p, q)
    assert graphed.iteration_index() == 5


def test_graph_timers_time_every_step_launch():
    from ultranca_b200 import training
    a, pool, target = _setup()
    b, pool_b, _ = _setup()
    pt = training.PoolTrainer(a, pool, target, key=1, graph=True, timed=1)
    plain = training.PoolTrainer(b, pool_b, target, key=1, graph=True)
    for _ in range(5):  # one direct iteration, then the two timed graph copies in turn
        pt.iteration()
        plain.iteration()
    kt = pt.kernel_times()
    assert sorted(kt) == ['bwd', 'fwd'] and len(kt['fwd']) == len(kt['bwd']) == 5 * a.steps
    assert all(0 < v < 1000 for v in kt['fwd'] + kt['bwd'])
    assert torch.equal(a.w1, b.w1) and torch.equal(pool, pool_b)  # timing changes nothing
    sampled = training.PoolTrainer(a, pool, target, key=1, graph=True, timed=2)
    for _ in range(3):
        sampled.iteration()
    kt = sampled.kernel_times(reset=True)
    assert len(kt['fwd']) == len(kt['bwd']) == 3  # steps 1 of 0..2, every iteration
    assert sampled.kernel_times() == {}
