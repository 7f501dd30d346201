"""Build libhla_s6.so (every CUDA source under csrc/) in-tree for sm_100a with nvcc.

The library is a plain C-ABI shared object (include/hla_s6.h); Python binds it with ctypes.
Incremental: sources are recompiled only when a .cu/.cuh/.h under csrc/ or include/ is newer
than the library; the translation units compile in parallel.  ``python build.py [--force] [-v]``.
"""
from __future__ import annotations

import argparse
import os
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / 'csrc'
LIB = PKG / 'libhla_s6.so'
ARCH = ['-gencode', 'arch=compute_100a,code=sm_100a']
NVCC = os.environ.get('NVCC', '/usr/local/cuda/bin/nvcc')


def sources():
    return sorted(CSRC.glob('*.cu'))


def _stale(target: Path) -> bool:
    if not target.exists():
        return True
    mtime = target.stat().st_mtime
    deps = list(CSRC.glob('*')) + list((ROOT / 'include').glob('*.h'))
    return any(p.stat().st_mtime > mtime for p in deps)


def build(force: bool = False, verbose: bool = False) -> Path:
    """Compile csrc/*.cu into libhla_s6.so next to this file; returns its path."""
    if not force and not _stale(LIB):
        return LIB
    objdir = PKG / '_build'
    objdir.mkdir(exist_ok=True)
    flags = ARCH + ['-O3', '-lineinfo', '-std=c++17', '-Xcompiler', '-fPIC', '--expt-relaxed-constexpr',
                    '-I', str(CSRC), '-I', str(ROOT / 'include')]
    if verbose:
        flags += ['-Xptxas', '-v']
    def compile_one(src):
        obj = objdir / (src.stem + '.o')
        proc = subprocess.run([NVCC, *flags, '-c', str(src), '-o', str(obj)], capture_output=True, text=True)
        return src, obj, proc

    objs = []
    with ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 1)) as pool:
        for src, obj, proc in pool.map(compile_one, sources()):
            if proc.returncode != 0:
                sys.stderr.write(proc.stdout + proc.stderr)
                raise RuntimeError(f'nvcc failed on {src.name}')
            if verbose:
                sys.stderr.write(proc.stderr)
            objs.append(str(obj))
    tmp = LIB.with_suffix('.so.tmp')
    cmd = [NVCC, *ARCH, '-shared', '-o', str(tmp), *objs, '-lcudart']
    proc = subprocess.run(cmd, capture_output=True, text=True)
    if proc.returncode != 0:
        sys.stderr.write(proc.stdout + proc.stderr)
        raise RuntimeError('nvcc link failed')
    os.replace(tmp, LIB)
    return LIB


if __name__ == '__main__':
    ap = argparse.ArgumentParser()
    ap.add_argument('--force', action='store_true')
    ap.add_argument('-v', '--verbose', action='store_true')
    args = ap.parse_args()
    print(build(args.force, args.verbose))
