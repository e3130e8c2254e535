"""Build recipe of the CPU oracle (test infrastructure): oracle/philox_mask.c -> oracle/libnca_oracle.so with gcc.

python -m oracle.build     (also run by __graft_entry__.build())
No fast-math: the mask restatement relies on IEEE fp32 rounding of one add, exactly as written in the reference.
"""
import os
import subprocess

HERE = os.path.dirname(os.path.abspath(__file__))


def build_oracle(verbose=False):
    src = os.path.join(HERE, 'philox_mask.c')
    out = os.path.join(HERE, 'libnca_oracle.so')
    if os.path.exists(out) and os.path.getmtime(out) >= os.path.getmtime(src):
        return out
    cmd = ['gcc', '-O2', '-std=c11', '-fPIC', '-shared', '-fno-fast-math', '-ffp-contract=off', src, '-o', out + '.tmp',
           '-lm']
    if verbose:
        print(' '.join(cmd), flush=True)
    subprocess.check_call(cmd)
    os.replace(out + '.tmp', out)
    return out


if __name__ == '__main__':
    print(build_oracle(verbose=True))
