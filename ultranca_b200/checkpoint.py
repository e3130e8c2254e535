"""Checkpoint I/O of trained NCAs and of a training group's state.

Per-NCA files use the reference's format (train.py:209-210 writes, train.py:112-114 reads): a torch.save dict with
`w1.weight` (hidden, 4C, 1, 1), `w1.bias` (hidden,) and `w2.weight` (C, hidden, 1, 1), CPU tensors, one file per NCA,
so weights trained here load in the reference's `init_weights` and the reference's files load here.

The group state adds what a training group needs to resume in the middle (the reference restarts a group from its
initial weights): the stacked weights, the Adam moments, the device iteration counter that drives bias correction and
the MultiStepLR schedule, the schedule's parameters, and optionally the sample pool.
"""
import os

import torch


def save_nca(path, w1, b1, w2):
    """One NCA's weights (w1 (hidden, 4C) or (hidden, 4C, 1, 1), b1 (hidden,), w2 (C, hidden) or (C, hidden, 1, 1))
    -> `path` in the reference's per-NCA format."""
    hidden, pin = w1.shape[0], w1.reshape(w1.shape[0], -1).shape[1]
    C = pin // 4
    torch.save({'w1.weight': w1.detach().reshape(hidden, pin, 1, 1).float().cpu().clone(),
                'w1.bias': b1.detach().reshape(hidden).float().cpu().clone(),
                'w2.weight': w2.detach().reshape(C, hidden, 1, 1).float().cpu().clone()}, path)


def load_nca(path, map_location='cpu'):
    """-> (w1 (hidden, 4C), b1 (hidden,), w2 (C, hidden)) from a per-NCA file of the reference's format."""
    sd = torch.load(path, map_location=map_location)
    missing = [k for k in ('w1.weight', 'w1.bias', 'w2.weight') if k not in sd]
    if missing:
        raise KeyError(f'{path}: not an NCA checkpoint (missing {missing})')
    hidden = sd['w1.bias'].shape[0]
    w1 = sd['w1.weight'].reshape(hidden, -1)
    C = w1.shape[1] // 4
    return w1, sd['w1.bias'].reshape(hidden), sd['w2.weight'].reshape(C, hidden)


def save_group(directory, stems, w1, b1, w2):
    """Stacked weights of K NCAs (w1 (K, hidden, 4C), b1 (K, hidden), w2 (K, C, hidden)) -> `directory`/<stem>.pt, as the
    reference writes a finished group (train.py:206-210)."""
    os.makedirs(directory, exist_ok=True)
    for k, stem in enumerate(stems):
        save_nca(os.path.join(directory, stem + '.pt'), w1[k], b1[k], w2[k])


def load_group(directory, stems, device='cpu'):
    """-> stacked (w1, b1, w2) of the NCAs `directory`/<stem>.pt, in order."""
    ws = [load_nca(os.path.join(directory, stem + '.pt')) for stem in stems]
    return tuple(torch.stack(t).to(device) for t in zip(*ws))


def state_dict(trainer, pool=None):
    """A RolloutTrainer's resumable state: weights, Adam moments and iteration counter, schedule parameters, and the
    pool when given (CPU copies)."""
    opt = trainer.opt
    sd = {'w1': trainer.w1, 'b1': trainer.b1, 'w2': trainer.w2, 'm': list(opt.m), 'v': list(opt.v),
          'iteration': opt.iteration, 'lr': opt.lr, 'betas': tuple(opt.betas), 'eps': opt.eps, 'gamma': opt.gamma,
          'milestones': [int(opt.milestones[i]) for i in range(opt.n_milestones)]}
    if pool is not None:
        sd['pool'] = pool
    out = {}
    for k, v in sd.items():
        if torch.is_tensor(v):
            out[k] = v.detach().cpu().clone()
        elif isinstance(v, list) and v and torch.is_tensor(v[0]):
            out[k] = [t.detach().cpu().clone() for t in v]
        else:
            out[k] = v
    return out


def load_state_dict(trainer, sd, pool=None):
    """Restore `sd` (from state_dict) into `trainer` in place (and into `pool` when both have one). The schedule
    parameters must match the trainer's: a resumed group continues the same schedule."""
    opt = trainer.opt
    mine = [int(opt.milestones[i]) for i in range(opt.n_milestones)]
    if list(sd['milestones']) != mine or float(sd['lr']) != float(opt.lr) or float(sd['gamma']) != float(opt.gamma):
        raise ValueError('checkpoint schedule (lr, gamma, milestones) differs from the trainer\'s')
    for name, mine_t in (('m', opt.m), ('v', opt.v)):
        if len(sd[name]) != len(mine_t):
            raise ValueError(f'checkpoint holds {len(sd[name])} Adam {name} tensors, the trainer {len(mine_t)}')
    pairs = [(trainer.w1, sd['w1']), (trainer.b1, sd['b1']), (trainer.w2, sd['w2'])]
    pairs += list(zip(opt.m + opt.v, list(sd['m']) + list(sd['v'])))
    for dst, src in pairs:  # every shape checked before anything is overwritten
        if dst.shape != src.shape:
            raise ValueError(f'checkpoint shape {tuple(src.shape)} != trainer shape {tuple(dst.shape)}')
    with torch.no_grad():
        for dst, src in pairs:
            dst.copy_(src)
        opt.iteration.copy_(sd['iteration'])
        if pool is not None and 'pool' in sd:
            pool.copy_(sd['pool'])


def save_state(path, trainer, pool=None):
    torch.save(state_dict(trainer, pool), path)


def load_state(path, trainer, pool=None):
    load_state_dict(trainer, torch.load(path, map_location='cpu'), pool)
