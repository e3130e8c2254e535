"""Build recipe of oracle/_ref/libncaref.so: the reference's own CUDA kernels (UltraNCA ncaops/nca_step.cuh, used
unchanged from the reference checkout) behind the test-only launcher oracle/ref_shim.cu, for sm_100a.

    python -m oracle.build_ref [/path/to/UltraNCA]

Flags follow the reference's build (ncaops/CMakeLists.txt:1-35, build.sh:1-21): -O3 --use_fast_math -lineinfo, and
NCA_SMEM_PER_SM_KB=228, the value build.sh derives for compute capability 10.0. The output stays out of git
(.gitignore: oracle/_ref/) but travels to the GPU box, where the reference checkout itself is absent. If the checkout
is missing, nothing is built (and tests that need the library skip).
"""
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
OUT_DIR = os.path.join(HERE, '_ref')
OUT = os.path.join(OUT_DIR, 'libncaref.so')
DEFAULT_REF = '/root/reference'
NVCC = os.environ.get('NVCC', '/usr/local/cuda/bin/nvcc')


def build_ref(ref_root=None, verbose=False):
    ref_root = ref_root or os.environ.get('ULTRANCA_REFERENCE', DEFAULT_REF)
    header = os.path.join(ref_root, 'ncaops', 'nca_step.cuh')
    if not os.path.exists(header):
        if verbose:
            print(f'reference checkout not found at {ref_root}: oracle/_ref not built', flush=True)
        return None
    src = os.path.join(HERE, 'ref_shim.cu')
    if os.path.exists(OUT) and os.path.getmtime(OUT) >= max(os.path.getmtime(src), os.path.getmtime(header)):
        return OUT
    os.makedirs(OUT_DIR, exist_ok=True)
    cmd = [NVCC, '-gencode', 'arch=compute_100a,code=sm_100a', '-O3', '--use_fast_math', '-lineinfo', '-std=c++17',
           '-DNCA_SMEM_PER_SM_KB=228', '-Xcompiler', '-fPIC', '-shared', '-cudart', 'shared',
           '-I', os.path.join(ref_root, 'ncaops'), src, '-o', OUT + '.tmp']
    if verbose:
        print(' '.join(cmd), flush=True)
    subprocess.check_call(cmd)
    os.replace(OUT + '.tmp', OUT)
    return OUT


if __name__ == '__main__':
    print(build_ref(sys.argv[1] if len(sys.argv) > 1 else None, verbose=True))
