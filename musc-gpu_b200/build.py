"""Build the sm_100a C-ABI library ``musc_b200/libmusc_b200.so`` with nvcc.

Usage: ``python musc-gpu_b200/build.py [--force] [--verbose]``.  Each ``.cu``
file under ``csrc/`` is compiled to an object for
``-gencode arch=compute_100a,code=sm_100a`` and linked into one shared
library with the CUDA runtime linked statically (so the library shares the
process's primary CUDA context with torch without depending on torch's
runtime build).  Objects are rebuilt only when a source or header is newer.
"""
from __future__ import annotations

import argparse
import os
import shutil
import subprocess
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parent
CSRC = ROOT / 'csrc'
INCLUDE = ROOT.parent / 'include'
OUT_DIR = ROOT / 'musc_b200'
BUILD = ROOT / '_build'
LIB = OUT_DIR / 'libmusc_b200.so'

ARCH = ['-gencode', 'arch=compute_100a,code=sm_100a']
NVCC_FLAGS = ['-O3', '-lineinfo', '-std=c++17', '-Xcompiler', '-fPIC', '--expt-relaxed-constexpr',
              '-Xptxas', '-warn-spills']


def nvcc() -> str:
    for cand in (os.environ.get('NVCC'), '/usr/local/cuda/bin/nvcc', shutil.which('nvcc')):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError('nvcc not found')


def _newest_header() -> float:
    hdrs = list(CSRC.glob('*.cuh')) + list(INCLUDE.glob('*.h'))
    return max((h.stat().st_mtime for h in hdrs), default=0.0)


def build(force: bool = False, verbose: bool = False, ptxas_info: bool = False) -> Path:
    BUILD.mkdir(exist_ok=True)
    compiler = nvcc()
    newest_hdr = _newest_header()
    objs = []
    for src in sorted(CSRC.glob('*.cu')):
        obj = BUILD / (src.stem + '.o')
        objs.append(obj)
        if (not force and obj.exists() and obj.stat().st_mtime >= src.stat().st_mtime
                and obj.stat().st_mtime >= newest_hdr and not ptxas_info):
            continue
        cmd = [compiler, *ARCH, *NVCC_FLAGS, '-I', str(INCLUDE), '-c', str(src), '-o', str(obj)]
        if ptxas_info:
            cmd[1:1] = ['-Xptxas', '-v']
        if verbose:
            print(' '.join(cmd), flush=True)
        subprocess.run(cmd, check=True)
    if force or not LIB.exists() or any(o.stat().st_mtime > LIB.stat().st_mtime for o in objs):
        cmd = [compiler, *ARCH, '-shared', '-cudart', 'static', '-o', str(LIB), *map(str, objs)]
        if verbose:
            print(' '.join(cmd), flush=True)
        subprocess.run(cmd, check=True)
    return LIB


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument('--force', action='store_true')
    ap.add_argument('--verbose', action='store_true')
    ap.add_argument('--ptxas-info', action='store_true', help='print registers / spills / smem per kernel')
    args = ap.parse_args()
    lib = build(args.force, args.verbose, args.ptxas_info)
    print(lib)


if __name__ == '__main__':
    sys.exit(main())
