"""Build the sm_100a kernels into the in-tree shared library ``bdm_b200/libbdm_b200.so``.

    python -m bdm_b200.build            # incremental
    python -m bdm_b200.build --force    # rebuild everything

Each ``csrc/*.cu`` compiles separately with nvcc for ``sm_100a`` only (no
PTX fallback, no other architectures); the objects link into one shared
library with the CUDA runtime linked statically, so the library depends on
nothing but the driver.  No GPU is needed to build.
"""
from __future__ import annotations

import argparse
import concurrent.futures as cf
import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, 'csrc')
BUILD = os.path.join(HERE, '_build')
LIB = os.path.join(HERE, 'libbdm_b200.so')
HEADER = os.path.join(ROOT, 'include', 'bdm_b200.h')

ARCH = ['-gencode', 'arch=compute_100a,code=sm_100a']
NVCC_FLAGS = ['-O3', '-std=c++17', '-lineinfo', '-Xcompiler', '-fPIC', '-Xcompiler', '-fvisibility=hidden',
              '--expt-relaxed-constexpr', f'-I{os.path.join(ROOT, "include")}']


def nvcc() -> str:
    cand = os.environ.get('NVCC') or shutil.which('nvcc') or '/usr/local/cuda/bin/nvcc'
    if not os.path.exists(cand):
        raise RuntimeError('nvcc not found; set NVCC or put /usr/local/cuda/bin on PATH')
    return cand


def sources() -> list[str]:
    return sorted(os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith('.cu'))


def _deps_mtime() -> float:
    deps = [os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith(('.cuh', '.h'))] + [HEADER]
    return max(os.path.getmtime(d) for d in deps)


def _compile(src: str, force: bool, verbose: bool) -> str:
    obj = os.path.join(BUILD, os.path.basename(src)[:-3] + '.o')
    if not force and os.path.exists(obj) and os.path.getmtime(obj) >= max(os.path.getmtime(src), _deps_mtime()):
        return obj
    cmd = [nvcc(), *ARCH, *NVCC_FLAGS, '-c', src, '-o', obj]
    if verbose:
        cmd.insert(1, '-Xptxas=-v')
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f'nvcc failed for {src}:\n{res.stdout}\n{res.stderr}')
    if verbose:
        sys.stderr.write(res.stderr)
    return obj


def build(force: bool = False, verbose: bool = False) -> str:
    """Compile every kernel for sm_100a and link the shared library; returns its path."""
    os.makedirs(BUILD, exist_ok=True)
    srcs = sources()
    with cf.ThreadPoolExecutor(max_workers=min(8, len(srcs))) as pool:
        objs = list(pool.map(lambda s: _compile(s, force, verbose), srcs))
    if force or not os.path.exists(LIB) or os.path.getmtime(LIB) < max(os.path.getmtime(o) for o in objs):
        tmp = LIB + '.tmp'
        cmd = [nvcc(), *ARCH, '-shared', '-cudart', 'static', '-o', tmp, *objs]
        res = subprocess.run(cmd, capture_output=True, text=True)
        if res.returncode != 0:
            raise RuntimeError(f'link failed:\n{res.stdout}\n{res.stderr}')
        os.replace(tmp, LIB)
    return LIB


if __name__ == '__main__':
    ap = argparse.ArgumentParser()
    ap.add_argument('--force', action='store_true')
    ap.add_argument('--verbose', action='store_true', help='print ptxas register / spill reports')
    a = ap.parse_args()
    print(build(force=a.force, verbose=a.verbose))
