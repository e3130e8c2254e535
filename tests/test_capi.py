"""CPU: the C-ABI library loads, exports every symbol include/ultranca_b200.h declares, and its host-side validation
rejects bad arguments with the reference's error behaviour before any device work (no compute calls here)."""
import ctypes
import json
import os
import re

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, 'include', 'ultranca_b200.h')


def declared_functions():
    text = re.sub(r'/\*.*?\*/', '', open(HEADER).read(), flags=re.S)
    return sorted(set(re.findall(r'^\s*(?:const\s+)?[a-z_0-9]+\s*\*?\s*(nca_[a-z_0-9]+)\s*\(', text, flags=re.M)))


def test_library_exports_every_declared_symbol():
    from ultranca_b200 import _lib
    names = declared_functions()
    assert len(names) >= 12, names
    raw = ctypes.CDLL(_lib.LIB_PATH)
    for name in names:
        assert hasattr(raw, name), f'{name} declared in the header but not exported'
        assert name in _lib.SIGNATURES, f'{name} has no ctypes signature'
    assert _lib.lib.nca_version() == 1


def test_step_seed_matches_reference_splitmix64():
    from ultranca_b200 import nca_ops
    s = json.load(open(os.path.join(ROOT, 'tests', 'golden', 'step_seeds.json')))
    assert [nca_ops.step_seed(s['seed'], i) for i in range(8)] == [int(v) for v in s['step_seeds']]


def _forward(**over):
    from ultranca_b200._lib import lib
    args = dict(x=1, w1=1, b1=1, w2=1, y=1, alpha=None, alive=None, N=4, C=12, H=8, W=16, K=2, hidden=96, B=2, seed=0,
                rate=0.5, fp32=0, growing=0, off=0, stream=None)
    args.update(over)
    p = lambda v: None if v is None else ctypes.c_void_p(v)
    st = lib.nca_forward(p(args['x']), p(args['w1']), p(args['b1']), p(args['w2']), p(args['y']), p(args['alpha']),
                         p(args['alive']), args['N'], args['C'], args['H'], args['W'], args['K'], args['hidden'],
                         args['B'], args['seed'], args['rate'], args['fp32'], args['growing'], args['off'], args['stream'])
    return st, lib.nca_last_error().decode()


@pytest.mark.parametrize('over, code, text', [
    (dict(N=5), 2, 'number of NCAs'),                 # nca_cuda.cu:132-133
    (dict(C=8, hidden=64, N=4), 3, 'no kernel instantiated'),  # nca_cuda.cu:75
    (dict(growing=1, C=3, hidden=96), 2, 'at least 4 channels'),  # nca_cuda.cu:140-141
    (dict(x=None), 1, 'x must not be null'),
    (dict(growing=1), 1, 'alive must not be null'),  # alpha is unused: the alive mask is computed in the step
    (dict(H=0), 2, 'positive'),
])
def test_forward_validation_errors(over, code, text):
    st, msg = _forward(**over)
    assert st == code and text in msg, (st, msg)


def test_python_api_rejects_cpu_tensors():
    import torch
    from ultranca_b200 import nca_ops
    x = torch.zeros(1, 1, 12, 8, 16)
    w1, b1, w2 = torch.zeros(1, 96, 48), torch.zeros(1, 96), torch.zeros(1, 12, 96)
    with pytest.raises(RuntimeError, match='CUDA tensor'):
        nca_ops.step(x, w1, b1, w2, 0.5, seed=1)


def test_ncaops_import_path_is_the_same_module():
    import ncaops
    from ncaops import nca_ops
    import ultranca_b200.nca_ops as impl
    assert nca_ops is impl and ncaops.step is impl.step
    nca_ops.CHUNK = 3
    assert impl.CHUNK == 3
    nca_ops.CHUNK = None


def test_partial_add_stage_requires_main():
    """NCA_STAGE_PARTIAL_ADD (8) modifies NCA_STAGE_MAIN: on its own it is an argument error, found before any device
    work."""
    from ultranca_b200._lib import lib
    p = ctypes.c_void_p(256)
    st = lib.nca_backward_stages(p, p, None, p, p, p, p, p, p, p, p, 1 << 30, p, 1 << 30, 4, 12, 8, 16, 2, 96, 2, 0, 0.5,
                                 0, 0, 0, 0, 8, None)
    assert st == 1 and 'PARTIAL_ADD' in lib.nca_last_error().decode()


@pytest.mark.parametrize('stages', [0, 16, 32, 16 | 32])
def test_stage_mask_needs_a_stage_and_known_bits(stages):
    """NCA_STAGE_X_STABLE (16) qualifies the stages; a mask without a stage bit or with an unknown bit is rejected
    before any device work."""
    from ultranca_b200._lib import lib
    p = ctypes.c_void_p(256)
    st = lib.nca_backward_stages(p, p, None, p, p, p, p, p, p, p, p, 1 << 30, p, 1 << 30, 4, 12, 8, 16, 2, 96, 2, 0, 0.5,
                                 0, 0, 0, 0, stages, None)
    assert st == 1 and 'stage' in lib.nca_last_error().decode()


def test_wait_selftest_validates_its_arguments():
    """The failure-detection self-test refuses a limit outside (0, 1 s] and a null output before any launch."""
    from ultranca_b200._lib import lib
    assert lib.nca_wait_selftest(0, ctypes.c_void_p(256), None) == 1
    assert lib.nca_wait_selftest(2_000_000_000, ctypes.c_void_p(256), None) == 1
    assert lib.nca_wait_selftest(1000, None, None) == 1
    assert 'out must not be null' in lib.nca_last_error().decode()
