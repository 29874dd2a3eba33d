"""Build the yanchor_b200 CUDA library in place (sm_100a).

    python -m yanchor_b200.build            # -> yanchor_b200/libyanchor_b200.so

The library is a plain shared object with the C ABI of include/yanchor_b200.h;
nvcc cross-compiles it on a machine without a GPU.  Object files go to
yanchor_b200/_build/ and are reused when their source and the shared headers
are older than the object.
"""
from __future__ import annotations

import os
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, 'csrc')
BUILD = os.path.join(HERE, '_build')
LIB = os.path.join(HERE, 'libyanchor_b200.so')
INCLUDE = os.path.join(os.path.dirname(HERE), 'include')

ARCH = ['-gencode', 'arch=compute_100a,code=sm_100a']
FLAGS = ['-O3', '-std=c++17', '-lineinfo', '-Xcompiler', '-fPIC', '--expt-relaxed-constexpr',
         '-Xptxas', '-v', '-I', INCLUDE]


def nvcc():
    for cand in (os.environ.get('NVCC'), '/usr/local/cuda/bin/nvcc', 'nvcc'):
        if cand and (os.path.sep not in cand or os.path.exists(cand)):
            return cand
    raise RuntimeError('nvcc not found')


def _headers():
    out = [os.path.join(INCLUDE, 'yanchor_b200.h')]
    out += [os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith(('.cuh', '.h'))]
    return out


def _compile(src, obj, verbose):
    cmd = [nvcc(), *ARCH, *FLAGS, '-c', src, '-o', obj]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f'nvcc failed on {os.path.basename(src)}:\n{res.stderr}')
    if verbose:
        print(res.stderr, file=sys.stderr)
    return obj


def build(verbose: bool = False, force: bool = False) -> str:
    os.makedirs(BUILD, exist_ok=True)
    sources = sorted(f for f in os.listdir(CSRC) if f.endswith('.cu'))
    newest_header = max(os.path.getmtime(h) for h in _headers())
    jobs = []
    objs = []
    for f in sources:
        src = os.path.join(CSRC, f)
        obj = os.path.join(BUILD, f[:-3] + '.o')
        objs.append(obj)
        if force or not os.path.exists(obj) or os.path.getmtime(obj) < max(os.path.getmtime(src), newest_header):
            jobs.append((src, obj))
    with ThreadPoolExecutor(max_workers=min(8, max(1, len(jobs)))) as ex:
        list(ex.map(lambda j: _compile(*j, verbose), jobs))
    if jobs or not os.path.exists(LIB) or os.path.getmtime(LIB) < max(os.path.getmtime(o) for o in objs):
        cmd = [nvcc(), *ARCH, '-shared', '-o', LIB, *objs, '-lcudart']
        res = subprocess.run(cmd, capture_output=True, text=True)
        if res.returncode != 0:
            raise RuntimeError(f'link failed:\n{res.stderr}')
    return LIB


TEST_CSRC = os.path.join(os.path.dirname(HERE), 'tests', 'csrc')
TEST_LIB = os.path.join(os.path.dirname(HERE), 'tests', '_build', 'libyb_tc_debug.so')


def build_test_lib(force: bool = False) -> str:
    """Test-only library: the tensor-core chunk kernel with its stage dumps
    enabled (tests/csrc/tc_debug.cu).  Never loaded by the package."""
    src = os.path.join(TEST_CSRC, 'tc_debug.cu')
    deps = [src, os.path.join(CSRC, 'gdn_chunk_tc.cu')] + _headers()
    os.makedirs(os.path.dirname(TEST_LIB), exist_ok=True)
    if force or not os.path.exists(TEST_LIB) or os.path.getmtime(TEST_LIB) < max(os.path.getmtime(d) for d in deps):
        cmd = [nvcc(), *ARCH, *FLAGS, '-shared', src, '-o', TEST_LIB, '-lcudart']
        res = subprocess.run(cmd, capture_output=True, text=True)
        if res.returncode != 0:
            raise RuntimeError(f'nvcc failed on tc_debug.cu:\n{res.stderr}')
    return TEST_LIB


if __name__ == '__main__':
    print(build(verbose='-v' in sys.argv, force='-f' in sys.argv))
    print(build_test_lib(force='-f' in sys.argv))
