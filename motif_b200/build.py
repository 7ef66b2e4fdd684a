"""Build `libmotif_b200.so` (all CUDA kernels + the C ABI) in-tree for sm_100a.

    python -m motif_b200.build [--force] [--jobs N]

Each `csrc/*.cu` is compiled to an object in `_build/` with
`-gencode arch=compute_100a,code=sm_100a`, then linked into
`motif_b200/libmotif_b200.so` next to this file.  Rebuilds only when a source or
header is newer than the library.
"""

import argparse
import concurrent.futures as cf
import glob
import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, 'csrc')
BUILD = os.path.join(ROOT, '_build')
LIB = os.path.join(HERE, 'libmotif_b200.so')
HEADER = os.path.join(ROOT, 'include', 'motif_b200.h')

ARCH = ['-gencode', 'arch=compute_100a,code=sm_100a']
NVCC_FLAGS = ['-O3', '-std=c++17', '-lineinfo', '-Xcompiler', '-fPIC', '-Xcompiler', '-fvisibility=hidden',
              '--expt-relaxed-constexpr', f'-I{os.path.join(ROOT, "include")}']


def nvcc() -> str:
    for cand in (os.environ.get('NVCC'), shutil.which('nvcc'), '/usr/local/cuda/bin/nvcc'):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError('nvcc not found: set NVCC or put the CUDA toolkit on PATH')


def sources():
    return sorted(glob.glob(os.path.join(CSRC, '*.cu')))


def _stale() -> bool:
    if not os.path.exists(LIB):
        return True
    t = os.path.getmtime(LIB)
    deps = sources() + glob.glob(os.path.join(CSRC, '*.cuh')) + [HEADER]
    return any(os.path.getmtime(p) > t for p in deps)


def _compile(src: str) -> str:
    obj = os.path.join(BUILD, os.path.basename(src) + '.o')
    cmd = [nvcc(), *ARCH, *NVCC_FLAGS, '-c', src, '-o', obj]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f'nvcc failed on {src}:\n{r.stderr}')
    return obj


def build(force: bool = False, jobs: int = 0, verbose: bool = False) -> str:
    """Compile every kernel and link the shared library; returns its path."""
    if not force and not _stale():
        return LIB
    os.makedirs(BUILD, exist_ok=True)
    srcs = sources()
    jobs = jobs or min(len(srcs), os.cpu_count() or 4)
    with cf.ThreadPoolExecutor(max_workers=jobs) as ex:
        objs = list(ex.map(_compile, srcs))
    tmp = LIB + '.tmp'
    cmd = [nvcc(), *ARCH, '-shared', '-Xcompiler', '-fPIC', *objs, '-o', tmp, '-lcudart']
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f'link failed:\n{r.stderr}')
    os.replace(tmp, LIB)
    if verbose:
        print(f'built {LIB}')
    return LIB


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument('--force', action='store_true')
    ap.add_argument('--jobs', type=int, default=0)
    a = ap.parse_args()
    build(force=a.force, jobs=a.jobs, verbose=True)


if __name__ == '__main__':
    sys.exit(main())
