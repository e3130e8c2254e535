"""One warm-up and one measured fwd + bwd NCA step, for Nsight Compute (the reference's
ncaops/testing/profile_one_step.py runs one fwd + bwd step at K = 24, B = 2, 128 x 128 for the same purpose).

    python -m ultranca_b200.profile_step [--K 32] [--B 2] [--size 128] [--growing] [--fp32] [--rate 0.5]
    ncu --set full --clock-control none -k regex:bwd_kernel_tc -s 1 -c 1 -o prof python -m ultranca_b200.profile_step

Default: BASELINE configuration 1's step (32 texture NCAs, batch 2, 128 x 128), whose state (50 MB) plus dp scratch
(201 MB) exceed the L2, so DRAM counters are representative. Launches per step: forward (growing: with the alive mask),
backward main, adjoint, reduce; the warm-up step comes first (skip its launches with ncu -s).
"""
import argparse

import torch


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument('--K', type=int, default=32)
    ap.add_argument('--B', type=int, default=2)
    ap.add_argument('--size', type=int, default=128)
    ap.add_argument('--rate', type=float, default=0.5)
    ap.add_argument('--growing', action='store_true')
    ap.add_argument('--fp32', action='store_true')
    a = ap.parse_args()
    from ultranca_b200 import nca_ops
    C, HID = (16, 128) if a.growing else (12, 96)
    g = torch.Generator(device='cuda').manual_seed(0)
    x = 0.3 * torch.randn(a.K, a.B, C, a.size, a.size, device='cuda', generator=g)
    w1 = 0.1 * torch.randn(a.K, HID, 4 * C, device='cuda', generator=g)
    b1 = 0.05 * torch.randn(a.K, HID, device='cuda', generator=g)
    w2 = 0.05 * torch.randn(a.K, C, HID, device='cuda', generator=g)
    if a.growing:
        x[:, :, 3] = x[:, :, 3].abs()
    params = [t.requires_grad_() for t in (x, w1, b1, w2)]
    R = torch.randn_like(x)
    for _ in range(2):
        y = nca_ops.step(*params, a.rate, a.growing, a.fp32, seed=1234)
        torch.autograd.grad((y * R).sum(), params)
    torch.cuda.synchronize()
    print('profile_step done', flush=True)


if __name__ == '__main__':
    main()
