"""ctypes binding of libultranca_b200.so (the C-ABI in include/ultranca_b200.h).

There is no fallback: if the library is missing or cannot be loaded, importing this module raises ImportError with
the build command, and every failed call raises RuntimeError with the library's message (the reference's nanobind
layer raises RuntimeError the same way, ncaops/nca_cuda.cu:23-33).
"""
import ctypes
import os

PKG = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(PKG, 'libultranca_b200.so')

c_f32p = ctypes.c_void_p
c_u8p = ctypes.c_void_p
c_i64 = ctypes.c_int64
c_u32 = ctypes.c_uint32
c_u64 = ctypes.c_uint64
c_int = ctypes.c_int
c_float = ctypes.c_float
c_vp = ctypes.c_void_p

# name -> (restype, argtypes); every function the header declares
SIGNATURES = {
    'nca_last_error': (ctypes.c_char_p, []),
    'nca_version': (c_int, []),
    'nca_forward': (c_int, [c_f32p, c_f32p, c_f32p, c_f32p, c_f32p, c_f32p, c_u8p, c_i64, c_i64, c_i64, c_i64, c_i64,
                            c_i64, c_u32, c_u64, c_float, c_int, c_int, c_i64, c_vp]),
    'nca_rollout': (c_int, [c_f32p, c_f32p, c_f32p, c_f32p, c_f32p, c_f32p, c_f32p, c_u8p, c_i64, c_i64, c_i64, c_i64,
                            c_i64, c_i64, c_u32, c_u32, c_u64, c_float, c_int, c_int, c_i64, c_vp]),
    'nca_step_seed': (c_u64, [c_u64, c_u64]),
    'nca_backward_workspace': (c_int, [c_i64, c_i64, c_int, c_i64, c_i64, c_i64, c_i64, c_float, c_int,
                                       ctypes.POINTER(c_i64), ctypes.POINTER(c_i64), ctypes.POINTER(c_i64)]),
    'nca_backward': (c_int, [c_f32p, c_f32p, c_u8p, c_f32p, c_f32p, c_f32p, c_f32p, c_f32p, c_f32p, c_f32p, c_f32p,
                             c_i64, c_f32p, c_i64, c_i64, c_i64, c_i64, c_i64, c_i64, c_i64, c_u32, c_u64, c_float,
                             c_int, c_int, c_i64, c_int, c_vp]),
    'nca_backward_stages': (c_int, [c_f32p, c_f32p, c_u8p, c_f32p, c_f32p, c_f32p, c_f32p, c_f32p, c_f32p, c_f32p,
                                    c_f32p, c_i64, c_f32p, c_i64, c_i64, c_i64, c_i64, c_i64, c_i64, c_i64, c_u32,
                                    c_u64, c_float, c_int, c_int, c_i64, c_int, c_int, c_vp]),
    'nca_backward_static_scratch': (c_int, [c_f32p, c_f32p, c_f32p, c_f32p, c_f32p, c_f32p, c_f32p, c_f32p, c_f32p,
                                            c_i64, c_i64, c_i64, c_i64, c_i64, c_i64, c_u32, c_u64, c_float, c_i64,
                                            c_int, c_vp]),
    'nca_update_mask': (c_int, [c_f32p, c_i64, c_i64, c_i64, c_u64, c_float, c_i64, c_vp]),
    'nca_synthetic_loss': (c_int, [c_f32p, c_f32p, c_f32p, c_f32p, c_f32p, c_i64, c_i64, c_i64, c_i64, c_i64, c_float,
                                   c_vp]),
    'nca_task_loss': (c_int, [c_f32p, c_f32p, c_f32p, c_f32p, c_f32p, c_i64, c_i64, c_i64, c_i64, c_i64, c_i64,
                              c_float, c_vp]),
    'nca_adam_step': (c_int, [c_f32p, c_f32p, c_f32p, c_f32p, c_f32p, c_f32p, c_f32p, c_f32p, c_f32p, c_f32p, c_f32p,
                              c_f32p, c_i64, c_i64, c_i64, c_i64, c_vp, c_float, c_float, c_float, c_float, c_float,
                              ctypes.POINTER(c_i64), c_int, c_vp]),
    'nca_launch_info': (c_int, [c_i64, c_i64, c_int, c_int, c_i64, c_i64, c_i64, c_i64, ctypes.POINTER(ctypes.c_int32)]),
    'nca_device_error': (c_int, [ctypes.POINTER(c_int), c_int]),
    'nca_umma_selftest': (c_int, [c_int, c_int, c_int, c_f32p, c_f32p, c_f32p, c_vp]),
    'nca_wait_selftest': (c_int, [c_i64, c_vp, c_vp]),
    'nca_forward_dseed': (c_int, [c_f32p, c_f32p, c_f32p, c_f32p, c_f32p, c_f32p, c_u8p, c_i64, c_i64, c_i64, c_i64,
                                  c_i64, c_i64, c_u32, c_vp, c_i64, c_float, c_int, c_int, c_i64, c_vp]),
    'nca_backward_stages_dseed': (c_int, [c_f32p, c_f32p, c_u8p, c_f32p, c_f32p, c_f32p, c_f32p, c_f32p, c_f32p,
                                          c_f32p, c_f32p, c_i64, c_f32p, c_i64, c_i64, c_i64, c_i64, c_i64, c_i64,
                                          c_i64, c_u32, c_vp, c_i64, c_float, c_int, c_int, c_i64, c_int, c_int, c_vp]),
    'nca_reduce_adam_step': (c_int, [c_f32p, c_i64, c_i64, c_i64, c_i64, c_i64, c_i64, c_i64, c_u32, c_int, c_int,
                                     c_f32p, c_f32p, c_f32p, c_f32p, c_f32p, c_f32p, c_f32p, c_f32p, c_f32p, c_f32p,
                                     c_f32p, c_f32p, c_vp, c_float, c_float, c_float, c_float, c_float,
                                     ctypes.POINTER(c_i64), c_int, c_vp]),
    'nca_control_advance': (c_int, [c_vp, c_vp]),
    'nca_pool_sample': (c_int, [c_f32p, c_f32p, c_vp, c_vp, c_i64, c_i64, c_i64, c_i64, c_i64, c_i64, c_i64, c_int,
                                c_i64, c_vp]),
    'nca_pool_store': (c_int, [c_f32p, c_f32p, c_vp, c_i64, c_i64, c_i64, c_i64, c_i64, c_i64, c_vp]),
}


def _load():
    if not os.path.exists(LIB_PATH):
        raise ImportError(f'{LIB_PATH} is missing: build it with `python -m ultranca_b200.build` '
                          '(there is no CPU or PyTorch fallback for the NCA step)')
    lib = ctypes.CDLL(LIB_PATH)
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    return lib


lib = _load()


def check(status):
    if status != 0:
        raise RuntimeError(lib.nca_last_error().decode(errors='replace'))


def ptr(t):
    """Device pointer of a tensor (None -> NULL)."""
    return None if t is None else ctypes.c_void_p(t.data_ptr())
