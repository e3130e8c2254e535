"""Checkpoint I/O. CPU: the per-NCA files have the reference's keys and shapes (train.py:209-210) and load through a
restatement of the reference's reader (train.py:112-114); a group round-trips. GPU: a training group resumed from a
saved state continues bitwise as the uninterrupted run."""
import os

import pytest
import torch

from ultranca_b200 import checkpoint as ck


def reference_reader(files, C, Hd):
    """The reference's init_weights for a directory of files (train.py:112-114), restated."""
    sds = [torch.load(f, map_location='cpu') for f in files]
    return [(s['w1.weight'].reshape(Hd, 4 * C), s['w1.bias'], s['w2.weight'].reshape(C, Hd)) for s in sds]


def test_per_nca_file_is_the_reference_format(tmp_path):
    g = torch.Generator().manual_seed(0)
    K, C, Hd = 3, 12, 96
    w1, b1, w2 = torch.randn(K, Hd, 4 * C, generator=g), torch.randn(K, Hd, generator=g), torch.randn(K, C, Hd, generator=g)
    stems = [f'tex{k}' for k in range(K)]
    ck.save_group(str(tmp_path), stems, w1, b1, w2)
    sd = torch.load(os.path.join(tmp_path, 'tex1.pt'))
    assert set(sd) == {'w1.weight', 'w1.bias', 'w2.weight'}
    assert sd['w1.weight'].shape == (Hd, 4 * C, 1, 1) and sd['w2.weight'].shape == (C, Hd, 1, 1)
    ref = reference_reader([os.path.join(tmp_path, s + '.pt') for s in stems], C, Hd)
    for k in range(K):
        assert torch.equal(ref[k][0], w1[k]) and torch.equal(ref[k][1], b1[k]) and torch.equal(ref[k][2], w2[k])
    back = ck.load_group(str(tmp_path), stems)
    for a, b in zip(back, (w1, b1, w2)):
        assert torch.equal(a, b)


def test_reference_written_file_loads(tmp_path):
    """A file as the reference writes it (conv-shaped weights, train.py:209-210) loads as (w1, b1, w2)."""
    C, Hd = 16, 128
    g = torch.Generator().manual_seed(1)
    w1, b1, w2 = torch.randn(Hd, 4 * C, 1, 1, generator=g), torch.randn(Hd, generator=g), torch.randn(C, Hd, 1, 1, generator=g)
    torch.save({'w1.weight': w1, 'w1.bias': b1, 'w2.weight': w2}, tmp_path / 'grow.pt')
    a, b, c = ck.load_nca(str(tmp_path / 'grow.pt'))
    assert a.shape == (Hd, 4 * C) and c.shape == (C, Hd)
    assert torch.equal(a, w1.reshape(Hd, 4 * C)) and torch.equal(b, b1) and torch.equal(c, w2.reshape(C, Hd))


def test_not_a_checkpoint_is_rejected(tmp_path):
    torch.save({'weight': torch.zeros(2)}, tmp_path / 'x.pt')
    with pytest.raises(KeyError):
        ck.load_nca(str(tmp_path / 'x.pt'))


def _fake_trainer(seed):
    """The attributes of a RolloutTrainer that the group state reads and writes, as CPU tensors."""
    import ctypes
    from types import SimpleNamespace
    g = torch.Generator().manual_seed(seed)
    K, C, Hd = 2, 12, 96
    ws = [torch.randn(K, Hd, 4 * C, generator=g), torch.randn(K, Hd, generator=g), torch.randn(K, C, Hd, generator=g)]
    opt = SimpleNamespace(m=[torch.randn_like(w) for w in ws], v=[torch.rand_like(w) for w in ws],
                          iteration=torch.tensor([5]), lr=1e-3, betas=(0.9, 0.999), eps=1e-8, gamma=0.5,
                          milestones=(ctypes.c_int64 * 8)(256, 512), n_milestones=2)
    return SimpleNamespace(w1=ws[0], b1=ws[1], w2=ws[2], opt=opt)


def test_group_state_with_other_moments_is_rejected_untouched():
    """A group state whose Adam moments differ in number or shape from the trainer's is refused before anything is
    overwritten (weights and moments keep their values)."""
    src, dst = _fake_trainer(1), _fake_trainer(2)
    sd = ck.state_dict(src)
    before = [t.clone() for t in (dst.w1, dst.b1, dst.w2, *dst.opt.m, *dst.opt.v)]
    bad_count = dict(sd, m=sd['m'][:2])
    bad_shape = dict(sd, v=[sd['v'][0], sd['v'][1][:, :-1], sd['v'][2]])
    for bad in (bad_count, bad_shape):
        with pytest.raises(ValueError):
            ck.load_state_dict(dst, bad)
        after = (dst.w1, dst.b1, dst.w2, *dst.opt.m, *dst.opt.v)
        assert all(torch.equal(a, b) for a, b in zip(before, after))
    ck.load_state_dict(dst, sd)  # the matching state restores every tensor
    assert all(torch.equal(a, b) for a, b in zip((dst.w1, *dst.opt.m, *dst.opt.v), (src.w1, *src.opt.m, *src.opt.v)))


@pytest.mark.gpu
def test_resumed_group_continues_bitwise(tmp_path):
    from oracle import nca_oracle as O
    from ultranca_b200 import training
    K, B, C, HID, H, W, steps = 2, 2, 12, 96, 16, 32, 4
    x, w1, b1, w2 = (t.cuda() for t in O.make(K, B, C, HID, H, W, seed=3))
    target = (torch.rand(K, 3, H, W, generator=torch.Generator().manual_seed(2)) - 0.5).cuda()

    def trainer(ws):
        return training.RolloutTrainer(*(t.clone() for t in ws), B, H, W, steps, 0.5, milestones=(1, 3), gamma=0.5)

    a = trainer((w1, b1, w2))
    for it in range(2):
        a.iteration(x, target, seed=100 + it)
    ck.save_state(str(tmp_path / 'state.pt'), a)
    a.iteration(x, target, seed=102)
    a.iteration(x, target, seed=103)

    b = trainer((torch.zeros_like(w1), torch.zeros_like(b1), torch.zeros_like(w2)))
    ck.load_state(str(tmp_path / 'state.pt'), b)
    b.iteration(x, target, seed=102)
    b.iteration(x, target, seed=103)
    torch.cuda.synchronize()
    for p, q in ((a.w1, b.w1), (a.b1, b.b1), (a.w2, b.w2)):
        assert torch.equal(p, q)
    assert int(a.opt.iteration.item()) == int(b.opt.iteration.item()) == 4
