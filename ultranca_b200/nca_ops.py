"""PyTorch operator API of the fused NCA step on B200 -- a drop-in for the reference's ncaops/nca_ops.py.

Same names, signatures, argument meaning and error behaviour as the reference (ncaops/nca_ops.py:1-84):
x (K, B, C, H, W), w1 (K, hidden, 4C), b1 (K, hidden), w2 (K, C, hidden), fp32 CUDA tensors; update_rate >= 1 updates
every cell; growing=True applies the alive mask of a growing NCA (alpha = channel 3); fp32=False runs the MLP on TF32
tensor cores, fp32=True in fp32. The update mask is generated in the kernels from a per-call seed drawn from torch's
CPU generator (reproducible under torch.manual_seed), and regenerated, never stored, in the backward.

Additions (keyword-only, defaulted so existing callers are unaffected): `image_offset`, the global index of the first
image when a multi-GPU job shards the NCAs (the Philox counter uses the global image index, so a shard reproduces the
single-GPU masks).

The calls go through the C-ABI of libultranca_b200.so (ultranca_b200/_lib.py); there is no CPU or eager fallback.
"""
import ctypes

import torch

from ._lib import check, lib, ptr

__all__ = ['step', 'rollout', 'update_mask', 'new_seed', 'CHUNK', 'backward_workspace', 'step_seed']

CHUNK = None  # images per backward chunk; accepted for compatibility and ignored (one launch covers all images)


def _check(name, t, dims, dtype=torch.float32):
    if not isinstance(t, torch.Tensor):
        raise TypeError(f'{name} must be a torch.Tensor')
    if t.device.type != 'cuda':
        raise RuntimeError(f'{name} must be a CUDA tensor (there is no CPU path), got {t.device}')
    if t.dtype != dtype:
        raise TypeError(f'{name} must be {dtype}, got {t.dtype}')
    if t.dim() != dims:
        raise RuntimeError(f'{name} must have {dims} dimensions, got shape {tuple(t.shape)}')


def _stream(dev):
    return ctypes.c_void_p(torch.cuda.current_stream(dev).cuda_stream)


def _shapes(x, w1, b1, w2):
    _check('x', x, 5); _check('w1', w1, 3); _check('b1', b1, 2); _check('w2', w2, 3)
    K, B, C, H, W = x.shape
    HID = w1.shape[1]
    if tuple(w1.shape) != (K, HID, 4 * C):
        raise RuntimeError(f'w1 must have shape {(K, HID, 4 * C)}, got {tuple(w1.shape)}')
    if tuple(b1.shape) != (K, HID):
        raise RuntimeError(f'b1 must have shape {(K, HID)}, got {tuple(b1.shape)}')
    if tuple(w2.shape) != (K, C, HID):
        raise RuntimeError(f'w2 must have shape {(K, C, HID)}, got {tuple(w2.shape)}')
    for name, t in (('w1', w1), ('b1', b1), ('w2', w2)):
        if t.device != x.device:
            raise RuntimeError(f'{name} is on {t.device}, x on {x.device}')
    return K, B, C, H, W, HID


def _forward(x, w1, b1, w2, update_rate, seed, fp32, growing, image_offset=0):
    """-> y, alive mask (growing; empty otherwise) for the backward (nca_ops.py:13-20)."""
    K, B, C, H, W, HID = _shapes(x, w1, b1, w2)
    y = torch.empty_like(x)
    n = (K * B, H, W) if growing else (0, 0, 0)
    alive = torch.empty(n, dtype=torch.uint8, device=x.device)
    with torch.cuda.device(x.device):
        check(lib.nca_forward(ptr(x), ptr(w1), ptr(b1), ptr(w2), ptr(y), None, ptr(alive) if growing else None, K * B, C, H, W, K, HID, B, seed & (2 ** 64 - 1),
                              float(update_rate), int(bool(fp32)), int(bool(growing)), int(image_offset),
                              _stream(x.device)))
    return y, alive


def backward_workspace(C, hidden, fp32, N, H, W, K, update_rate, growing, device=None):
    """(dp floats, partial floats, images per chunk) of the backward on `device` (the reference's tuple,
    nca_cuda.cu:235-254, held (packed bytes per NCA, partial floats per image, chunk))."""
    dp, part, chunk = ctypes.c_int64(), ctypes.c_int64(), ctypes.c_int64()
    with torch.cuda.device(device if device is not None else torch.cuda.current_device()):
        check(lib.nca_backward_workspace(C, hidden, int(bool(fp32)), N, H, W, K, float(update_rate), int(bool(growing)),
                                         ctypes.byref(dp), ctypes.byref(part), ctypes.byref(chunk)))
    return dp.value, part.value, chunk.value


def launch_info(C, hidden, fp32, N, H, W, K, growing=False, device=None):
    """The launch configuration of the step kernels for this shape (diagnostic): dict of path, grids, threads."""
    info = (ctypes.c_int32 * 12)()
    with torch.cuda.device(device if device is not None else torch.cuda.current_device()):
        check(lib.nca_launch_info(C, hidden, int(bool(fp32)), int(bool(growing)), N, H, W, K, info))
    keys = ('rows_path', 'fwd_grid', 'fwd_threads', 'bwd_grid', 'bwd_threads', 'sms', 'tile_fwd_ctas_per_sm',
            'tile_bwd_grid', 'rows_fwd_occupancy', 'rows_fwd_regs', 'rows_fwd_max_dyn_smem', 'rows_fwd_carveout')
    return dict(zip(keys, list(info)))


def _backward(x, gy, alive, w1, b1, w2, update_rate, seed, fp32, growing, image_offset=0, grads=None):
    K, B, C, H, W, HID = _shapes(x, w1, b1, w2)
    N = K * B
    dp_floats, partial_floats, _ = backward_workspace(C, HID, fp32, N, H, W, K, update_rate, growing, x.device)
    dp = torch.empty(dp_floats, device=x.device)
    partial = torch.empty(partial_floats, device=x.device)
    gx = torch.empty_like(x)
    if grads is None:
        dw1, db1, dw2, acc = torch.empty_like(w1), torch.empty_like(b1), torch.empty_like(w2), 0
    else:
        (dw1, db1, dw2), acc = grads, 1
    _check('gy', gy, 5, dtype=gy.dtype)
    if gy.shape != x.shape or gy.device != x.device:
        raise RuntimeError(f'gy must have the shape and device of x {tuple(x.shape)} on {x.device}, got '
                           f'{tuple(gy.shape)} on {gy.device}')
    gy = gy.float().contiguous()  # an upstream gradient in another precision (e.g. under autocast) is read as fp32
    with torch.cuda.device(x.device):
        check(lib.nca_backward(ptr(x), ptr(gy), ptr(alive) if growing else None, ptr(w1), ptr(b1), ptr(w2), ptr(gx),
                               ptr(dw1), ptr(db1), ptr(dw2), ptr(dp), dp_floats, ptr(partial), partial_floats, N, C, H, W,
                               K, HID, B, seed & (2 ** 64 - 1), float(update_rate), int(bool(fp32)), int(bool(growing)),
                               int(image_offset), acc, _stream(x.device)))
    return gx, dw1, db1, dw2


class _Step(torch.autograd.Function):
    """nca_ops.py:23-45: saves (x, w1, b1, w2, alive); the backward regenerates the mask from the saved seed."""

    @staticmethod
    def forward(ctx, x, w1, b1, w2, update_rate, seed, fp32, growing, image_offset=0):
        y, alive = _forward(x, w1, b1, w2, update_rate, seed, fp32, growing, image_offset)
        ctx.save_for_backward(x, w1, b1, w2, alive)
        ctx.update_rate, ctx.seed, ctx.fp32, ctx.growing, ctx.image_offset = update_rate, seed, fp32, growing, image_offset
        return y

    @staticmethod
    def backward(ctx, gy):
        x, w1, b1, w2, alive = ctx.saved_tensors
        gx, dw1, db1, dw2 = _backward(x, gy, alive, w1, b1, w2, ctx.update_rate, ctx.seed, ctx.fp32, ctx.growing,
                                      ctx.image_offset)
        return gx, dw1, db1, dw2, None, None, None, None, None


def new_seed():
    """A step seed drawn from torch's CPU generator (nca_ops.py:51-52)."""
    return int(torch.randint(0, 2 ** 62, (1,)).item())


def step_seed(seed, i):
    """splitmix64 seed of rollout step i (nca_cuda.cu:157-164), as rollout() derives it."""
    return int(lib.nca_step_seed(seed & (2 ** 64 - 1), i))


def step(x, w1, b1, w2, update_rate, growing=False, fp32=False, seed=None, *, image_offset=0):
    """One NCA step (nca_ops.py:55-60); differentiable with respect to x, w1, b1, w2."""
    seed = new_seed() if seed is None else seed
    args = (x.contiguous(), w1.contiguous(), b1.contiguous(), w2.contiguous(), float(update_rate), seed, fp32, growing,
            image_offset)
    if torch.is_grad_enabled() and (x.requires_grad or w1.requires_grad or b1.requires_grad or w2.requires_grad):
        return _Step.apply(*args)
    return _forward(*args)[0]  # inference: no autograd bookkeeping


@torch.no_grad()
def rollout(x, w1, b1, w2, update_rate, steps, growing=False, fp32=False, seed=None, *, image_offset=0):
    """`steps` steps of step() without gradients in one call (nca_ops.py:63-77); step seeds derived from `seed`."""
    seed = new_seed() if seed is None else seed
    x, w1, b1, w2 = x.contiguous(), w1.contiguous(), b1.contiguous(), w2.contiguous()
    K, B, C, H, W, HID = _shapes(x, w1, b1, w2)
    y = torch.empty_like(x)
    tmp = torch.empty(K * B if steps > 1 else 0, C, H, W, device=x.device)
    # growing: one alive map per ping-pong buffer (the reference's (2N, H, W), nca_cuda.cu:166-188)
    alive = torch.empty((2 * K * B, H, W) if growing else (0, 0, 0), dtype=torch.uint8, device=x.device)
    with torch.cuda.device(x.device):
        check(lib.nca_rollout(ptr(x), ptr(w1), ptr(b1), ptr(w2), ptr(y), ptr(tmp) if steps > 1 else None,
                              None, ptr(alive) if growing else None, K * B, C, H, W, K, HID,
                              int(steps), B, seed & (2 ** 64 - 1), float(update_rate), int(bool(fp32)),
                              int(bool(growing)), int(image_offset), _stream(x.device)))
    return y


def update_mask(n, h, w, seed, update_rate, device='cuda', *, image_offset=0):
    """The mask the kernels use for `seed`: (n, h, w) of {0, 1} (nca_ops.py:80-84)."""
    m = torch.empty(n, h, w, device=device)
    with torch.cuda.device(m.device):
        check(lib.nca_update_mask(ptr(m), n, h, w, seed & (2 ** 64 - 1), float(update_rate), int(image_offset),
                                  _stream(m.device)))
    return m
