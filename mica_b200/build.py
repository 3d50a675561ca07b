"""Builds libmica_w8a8.so in-tree for sm_100a (nvcc cross-compiles without a GPU).

    python -m mica_b200.build          # or mica_b200.build.build()

The library is one translation unit (csrc/mica_w8a8.cu) linked against the static CUDA
runtime, so it does not depend on which libcudart torch happens to load.
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
SRC = HERE / 'csrc' / 'mica_w8a8.cu'
OUT = HERE / 'libmica_w8a8.so'
ARCH = ['-gencode', 'arch=compute_100a,code=sm_100a']
FLAGS = ['-O3', '-lineinfo', '-std=c++17', '-shared', '-Xcompiler', '-fPIC,-O2', '--expt-relaxed-constexpr']


def nvcc() -> str:
    for cand in (os.environ.get('NVCC'), shutil.which('nvcc'), '/usr/local/cuda/bin/nvcc'):
        if cand and Path(cand).exists():
            return cand
    raise FileNotFoundError('nvcc not found')


def sources():
    return sorted((HERE / 'csrc').glob('*.cu*')) + sorted((HERE.parent / 'include').glob('*.h'))


def up_to_date() -> bool:
    if not OUT.is_file():
        return False
    t = OUT.stat().st_mtime
    return all(p.stat().st_mtime <= t for p in sources())


def build(force: bool = False, verbose: bool = False) -> Path:
    if not force and up_to_date():
        return OUT
    tmp = OUT.with_suffix('.so.tmp')
    cmd = [nvcc(), *ARCH, *FLAGS, '-o', str(tmp), str(SRC)]
    if verbose:
        cmd.insert(1, '-Xptxas=-v')
        print(' '.join(cmd), file=sys.stderr)
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f'nvcc failed ({r.returncode}):\n{r.stdout}\n{r.stderr}')
    if verbose:
        print(r.stderr, file=sys.stderr)
    os.replace(tmp, OUT)
    return OUT


if __name__ == '__main__':
    print(build(force='--force' in sys.argv, verbose='-v' in sys.argv))
