"""TEST INFRASTRUCTURE ONLY: ctypes access to the reference's own CUDA kernels (oracle/_ref/libncaref.so, built from
the reference checkout by oracle/build_ref.py through the launcher oracle/ref_shim.cu).

Used by the GPU tests (the update mask bitwise, the forward within TF32 tolerance) and by bench.py to time the
reference's step kernels on the same B200. `available()` is False when the library was not built (no checkout).
"""
import ctypes
import os

import torch

HERE = os.path.dirname(os.path.abspath(__file__))
LIB = os.path.join(HERE, '_ref', 'libncaref.so')
_lib = None


def available():
    return os.path.exists(LIB)


def lib():
    global _lib
    if _lib is None:
        l = ctypes.CDLL(LIB)
        vp, i, u64, f = ctypes.c_void_p, ctypes.c_int, ctypes.c_uint64, ctypes.c_float
        l.ref_update_mask.argtypes = [vp, i, i, i, u64, f, vp]
        l.ref_forward.argtypes = [vp, vp, vp, vp, vp, vp, vp, i, i, i, i, i, i, u64, f, i, i, vp]
        l.ref_backward_workspace.argtypes = [i, i, i, i, i, i, f, i, i] + [ctypes.POINTER(ctypes.c_int64)] * 4
        l.ref_backward.argtypes = [vp] * 14 + [i] * 7 + [u64, f, i, i, vp]
        for fn in (l.ref_update_mask, l.ref_forward, l.ref_backward_workspace, l.ref_backward):
            fn.restype = ctypes.c_int
        _lib = l
    return _lib


def _p(t):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def _stream():
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


def _check(status):
    if status != 0:
        raise RuntimeError(f'reference kernel launch failed: cuda error {status}')


def update_mask(n, h, w, seed, rate):
    m = torch.empty(n, h, w, device='cuda')
    _check(lib().ref_update_mask(_p(m), n, h, w, seed, float(rate), _stream()))
    return m


def forward(x, w1, b1, w2, rate, seed, fp32=False, growing=False):
    K, B, C, H, W = x.shape
    HID = w1.shape[1]
    y = torch.empty_like(x)
    alpha = torch.empty(K * B, H, W, device=x.device) if growing else None
    alive = torch.empty(K * B, H, W, dtype=torch.uint8, device=x.device) if growing else None
    _check(lib().ref_forward(_p(x), _p(w1), _p(b1), _p(w2), _p(y), _p(alpha), _p(alive), K * B, C, HID, H, W, B, seed,
                             float(rate), int(fp32), int(growing), _stream()))
    return y, alive


class Backward:
    """Workspaces of the reference backward for one shape, reused across calls."""

    def __init__(self, K, B, C, HID, H, W, rate, fp32=False, growing=False):
        self.K, self.B, self.C, self.HID, self.H, self.W = K, B, C, HID, H, W
        self.rate, self.fp32, self.growing = float(rate), int(fp32), int(growing)
        vals = [ctypes.c_int64() for _ in range(4)]
        _check(lib().ref_backward_workspace(K * B, K, C, HID, H, W, self.rate, self.fp32, self.growing,
                                            *[ctypes.byref(v) for v in vals]))
        packed, partial, dp, updating = (v.value for v in vals)
        self.packed = torch.empty(packed, dtype=torch.uint8, device='cuda')
        self.partial = torch.empty(partial, device='cuda')
        self.dp = torch.empty(dp, device='cuda')
        self.updating = torch.empty(updating, dtype=torch.uint8, device='cuda')

    def __call__(self, x, gy, alive, w1, b1, w2, seed, out=None):
        gx, dw1, db1, dw2 = out if out is not None else (torch.empty_like(x), torch.empty_like(w1), torch.empty_like(b1),
                                                          torch.empty_like(w2))
        _check(lib().ref_backward(_p(x), _p(gy), _p(alive), _p(w1), _p(b1), _p(w2), _p(gx), _p(dw1), _p(db1), _p(dw2),
                                  _p(self.packed), _p(self.dp), _p(self.updating), _p(self.partial), self.K * self.B,
                                  self.K, self.C, self.HID, self.H, self.W, self.B, seed, self.rate, self.fp32,
                                  self.growing, _stream()))
        return gx, dw1, db1, dw2
