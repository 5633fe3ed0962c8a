"""Builds ``libspmm_b200.so`` (the C-ABI library) from ``spmm_b200/csrc`` with nvcc.

Every translation unit is compiled for sm_100a only
(``-gencode arch=compute_100a,code=sm_100a``) and linked in-tree into
``spmm_b200/libspmm_b200.so``; the library depends on the CUDA runtime only.
Usage: ``python -m spmm_b200.build [--force] [-v]``.
"""

from __future__ import annotations

import argparse
import concurrent.futures as cf
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, 'csrc')
BUILD = os.path.join(HERE, '_build')
LIB = os.path.join(HERE, 'libspmm_b200.so')
INCLUDE = os.path.join(os.path.dirname(HERE), 'include')
NVCC = os.environ.get('NVCC', '/usr/local/cuda/bin/nvcc')
ARCH = ['-gencode', 'arch=compute_100a,code=sm_100a']
FLAGS = ['-O3', '-std=c++17', '-lineinfo', '-Xcompiler', '-fPIC', '--expt-relaxed-constexpr',
         '-Xptxas', '-warn-spills']


def sources():
    return sorted(os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith('.cu'))


def _deps():
    files = [os.path.join(CSRC, f) for f in os.listdir(CSRC)]
    files.append(os.path.join(INCLUDE, 'spmm_b200.h'))
    return files


def _stale(target, deps):
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps)


def build(force: bool = False, verbose: bool = False) -> str:
    os.makedirs(BUILD, exist_ok=True)
    deps = _deps()
    objs = []
    jobs = []
    for src in sources():
        obj = os.path.join(BUILD, os.path.basename(src)[:-3] + '.o')
        objs.append(obj)
        if force or _stale(obj, deps):
            cmd = [NVCC, *ARCH, *FLAGS, '-I', INCLUDE, '-c', src, '-o', obj]
            if verbose:
                cmd += ['-Xptxas', '-v']
            jobs.append(cmd)

    def run(cmd):
        r = subprocess.run(cmd, capture_output=True, text=True)
        return cmd, r

    with cf.ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 1)) as ex:
        for cmd, r in ex.map(run, jobs):
            if verbose or r.returncode:
                sys.stderr.write(r.stdout + r.stderr)
            if r.returncode:
                raise RuntimeError(f'nvcc failed: {" ".join(cmd)}')
    if force or jobs or _stale(LIB, objs):
        tmp = LIB + f'.{os.getpid()}.tmp'
        subprocess.check_call([NVCC, *ARCH, '-shared', '-o', tmp, *objs, '-lcudart'])
        os.replace(tmp, LIB)
    return LIB


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument('--force', action='store_true')
    ap.add_argument('-v', '--verbose', action='store_true')
    args = ap.parse_args()
    print(build(args.force, args.verbose))


if __name__ == '__main__':
    main()
