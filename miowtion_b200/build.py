"""Builds the in-tree CUDA library `miowtion_b200/libveda_b200.so` for sm_100a.

    python -m miowtion_b200.build [--verbose]

Each `csrc/*.cu` is compiled separately (in parallel) and linked into one
shared library with the CUDA runtime linked statically, so the library
loads next to any PyTorch build. Rebuilds only when a source or header is
newer than the library.
"""

from __future__ import annotations

import argparse
import concurrent.futures
import glob
import os
import shutil
import subprocess
import sys

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
CSRC = os.path.join(PKG, 'csrc')
INCLUDE = os.path.join(ROOT, 'include')
BUILD = os.path.join(ROOT, '_build')
LIB = os.path.join(PKG, 'libveda_b200.so')

ARCH = ['-gencode', 'arch=compute_100a,code=sm_100a']
FLAGS = ['-O3', '-lineinfo', '-std=c++17', '-Xcompiler', '-fPIC',
         '--expt-relaxed-constexpr', f'-I{INCLUDE}', f'-I{CSRC}']


def nvcc() -> str:
    path = shutil.which('nvcc') or '/usr/local/cuda/bin/nvcc'
    if not os.path.exists(path):
        raise RuntimeError('nvcc not found; the CUDA toolkit is required to '
                           'build the library')
    return path


def sources() -> list[str]:
    return sorted(glob.glob(os.path.join(CSRC, '*.cu')))


def _stale() -> bool:
    if not os.path.exists(LIB):
        return True
    newest = max(os.path.getmtime(p) for p in
                 sources() + glob.glob(os.path.join(CSRC, '*.cuh')) +
                 glob.glob(os.path.join(INCLUDE, '*.h')) + [__file__])
    return newest > os.path.getmtime(LIB)


def _compile(src: str, verbose: bool) -> str:
    obj = os.path.join(BUILD, os.path.basename(src)[:-3] + '.o')
    cmd = [nvcc(), *ARCH, *FLAGS, '-c', src, '-o', obj]
    if verbose:
        cmd += ['-Xptxas', '-v']
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f'nvcc failed on {src}:\n{res.stderr}')
    if verbose and res.stderr:
        print(res.stderr, file=sys.stderr)
    return obj


def build(force: bool = False, verbose: bool = False) -> str:
    """Compiles and links the library; returns its path."""
    if not force and not _stale():
        return LIB
    os.makedirs(BUILD, exist_ok=True)
    with concurrent.futures.ThreadPoolExecutor(max_workers=8) as pool:
        objs = list(pool.map(lambda s: _compile(s, verbose), sources()))
    tmp = LIB + '.tmp'
    cmd = [nvcc(), *ARCH, '-shared', '-cudart', 'static', '-o', tmp, *objs]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f'link failed:\n{res.stderr}')
    os.replace(tmp, LIB)
    return LIB


if __name__ == '__main__':
    ap = argparse.ArgumentParser()
    ap.add_argument('--verbose', action='store_true')
    ap.add_argument('--force', action='store_true')
    args = ap.parse_args()
    print(build(force=args.force or args.verbose, verbose=args.verbose))
