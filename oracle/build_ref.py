"""Build the reference's own CPU core (``torch_fast_spdmm_core``) into ``oracle/_ref/``.

Test infrastructure only.  The reference's BOO/PBR builders and CPU SpMM live in
three C++ files of the reference project:

* ``torch_fast_spdmm/bindings/bindings.cpp`` (pybind11 module; its CUDA part is
  compiled out because ``CUDA_ENABLED`` is not defined, bindings.cpp:13-19, 225-231)
* ``torch_fast_spdmm/boo_matrix/boo_matrix.cpp`` (csr_to_boo, boo_to_csr,
  boo_batched_matmul_cpu)
* ``torch_fast_spdmm/pbr_matrix/pbr_matrix.cpp`` (csr_to_pbr, pbr_to_csr,
  pbr_batched_matmul_cpu, pbr_analyze_csr)

They are compiled where they lie (nothing is copied into this repository) with
``torch.utils.cpp_extension.load``; the only output is the extension module in
``oracle/_ref/``.  That directory is git-ignored but travels with the repository
snapshot, so the built module can serve as the CPU baseline on a machine that
does not have the reference sources.

Usage: ``python oracle/build_ref.py [--reference PATH]``.  Exits 0 and prints the
module path; exits 2 if the reference sources are absent.
"""

from __future__ import annotations

import argparse
import os
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
REF_OUT = os.path.join(HERE, '_ref')
# the reference checkout next to this repository, unless SPMM_REFERENCE_ROOT names one
DEFAULT_REFERENCE = os.environ.get('SPMM_REFERENCE_ROOT',
                                   os.path.abspath(os.path.join(HERE, '..', '..', 'reference')))
MODULE = 'torch_fast_spdmm_core'


def built_module_path() -> str | None:
    """Path of an already-built reference module in oracle/_ref/, or None."""
    if not os.path.isdir(REF_OUT):
        return None
    for name in sorted(os.listdir(REF_OUT)):
        if name.startswith(MODULE) and name.endswith('.so'):
            return os.path.join(REF_OUT, name)
    return None


def build(reference_root: str = DEFAULT_REFERENCE, verbose: bool = False) -> str:
    pkg = os.path.join(reference_root, 'torch_fast_spdmm')
    sources = [os.path.join(pkg, 'bindings', 'bindings.cpp'),
               os.path.join(pkg, 'pbr_matrix', 'pbr_matrix.cpp'),
               os.path.join(pkg, 'boo_matrix', 'boo_matrix.cpp')]
    missing = [s for s in sources if not os.path.isfile(s)]
    if missing:
        raise FileNotFoundError(f'reference sources not found: {missing}')
    import torch  # noqa: F401  (loads libc10 before the extension)
    from torch.utils.cpp_extension import load
    os.makedirs(REF_OUT, exist_ok=True)
    load(name=MODULE, sources=sources, extra_include_paths=[pkg],
         extra_cflags=['-O3', '-std=c++20', '-w'], build_directory=REF_OUT,
         verbose=verbose, is_python_module=True)
    path = built_module_path()
    if path is None:
        raise RuntimeError('reference build produced no module')
    return path


def load_reference():
    """Import the built reference module from oracle/_ref/ (None if absent)."""
    path = built_module_path()
    if path is None:
        return None
    import importlib.util
    import torch  # noqa: F401
    spec = importlib.util.spec_from_file_location(MODULE, path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def main() -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument('--reference', default=DEFAULT_REFERENCE)
    ap.add_argument('--verbose', action='store_true')
    args = ap.parse_args()
    if not os.path.isdir(args.reference):
        print(f'reference not present at {args.reference}; nothing built', file=sys.stderr)
        return 2
    print(build(args.reference, args.verbose))
    return 0


if __name__ == '__main__':
    sys.exit(main())
