"""Build the CUDA library in-tree: ultranca_b200/csrc/*.cu -> ultranca_b200/libultranca_b200.so (sm_100a only).

    python -m ultranca_b200.build [--verbose] [--force]

The shared library exports the C-ABI declared in include/ultranca_b200.h; ultranca_b200/_lib.py loads it with ctypes.
"""
import argparse
import glob
import os
import subprocess
import sys

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
LIB = os.path.join(PKG, 'libultranca_b200.so')
NVCC = os.environ.get('NVCC', '/usr/local/cuda/bin/nvcc')
FLAGS = ['-gencode', 'arch=compute_100a,code=sm_100a', '-lineinfo', '-O3', '-std=c++17', '--expt-relaxed-constexpr',
         '-Xcompiler', '-fPIC', '-shared', '-cudart', 'shared']


def sources():
    return sorted(glob.glob(os.path.join(PKG, 'csrc', '*.cu')))


def deps():
    return sources() + sorted(glob.glob(os.path.join(PKG, 'csrc', '*.cuh'))) + [os.path.join(ROOT, 'include', 'ultranca_b200.h')]


def up_to_date():
    return os.path.exists(LIB) and all(os.path.getmtime(LIB) >= os.path.getmtime(d) for d in deps())


def build(verbose=False, force=False, ptxas_verbose=False):
    if not force and up_to_date():
        return LIB
    cmd = [NVCC] + FLAGS + (['-Xptxas', '-v'] if ptxas_verbose else []) + ['-I', os.path.join(ROOT, 'include')] + \
        sources() + ['-o', LIB + '.tmp']
    if verbose:
        print(' '.join(cmd), flush=True)
    subprocess.check_call(cmd)
    os.replace(LIB + '.tmp', LIB)
    return LIB


if __name__ == '__main__':
    ap = argparse.ArgumentParser()
    ap.add_argument('--verbose', action='store_true')
    ap.add_argument('--force', action='store_true')
    ap.add_argument('--ptxas', action='store_true', help='print registers / spills / shared memory per kernel')
    a = ap.parse_args()
    print(build(a.verbose, a.force, a.ptxas))
    sys.exit(0)
