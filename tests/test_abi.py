"""The C-ABI library loads and exports exactly what include/spmm_b200.h
declares; host-only entry points answer without a GPU."""

import ctypes as C
import os
import re
import subprocess

import pytest

from spmm_b200 import _lib

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, 'include', 'spmm_b200.h')


def declared():
    text = open(HEADER).read()
    text = re.sub(r'/\*.*?\*/', '', text, flags=re.S)
    return sorted(set(re.findall(r'\b(spmm_[a-z0-9_]+)\s*\(', text)))


def exported():
    out = subprocess.run(['nm', '-D', '--defined-only', _lib.LIB_PATH], capture_output=True,
                         text=True, check=True).stdout
    return sorted({line.split()[-1] for line in out.splitlines() if ' T spmm_' in line})


def test_library_exports_every_declared_symbol():
    decl = declared()
    assert decl, 'no declarations parsed'
    L = _lib.lib()
    for name in decl:
        assert hasattr(L, name), name
    assert exported() == decl
    assert set(decl) == set(_lib.EXPORTS)


def test_host_only_entry_points():
    L = _lib.lib()
    assert L.spmm_abi_version() == 2
    assert 'uint16' in _lib.status_string(_lib.SPMM_EOVERFLOW_U16)
    assert 'wait expired' in _lib.status_string(_lib.SPMM_ETIMEOUT)
    assert 'collective' in _lib.status_string(_lib.SPMM_ENCCL)
    assert L.spmm_hem_level_slots(32) == 8 * 5 + 16 + 1
    assert L.spmm_hem_level_slots(1) == 8 + 16 + 1
    assert _lib.status_string(12345) == 'unknown status'
    for fn in (L.spmm_boo_build_workspace_size, L.spmm_pbr_build_workspace_size):
        small = fn(10, 10, 10)
        big = fn(1000, 1000, 100000)
        assert 0 < small < big
        assert fn(-1, 0, 0) == 0


def test_launch_cfg_layout():
    """spmm_launch_cfg as the header lays it out (64-bit): version 2 adds the
    status word after the workspace."""
    assert C.sizeof(_lib.LaunchCfg) == 56 and _lib.LaunchCfg.plan.offset == 48
    assert _lib.LaunchCfg.workspace.offset == 16 and _lib.LaunchCfg.status.offset == 32
    assert _lib.LaunchCfg.flags.offset == 40
    cfg = _lib.launch_cfg('tensor_cores', wait_us=5)
    assert (cfg.version, cfg.engine, cfg.wait_us, cfg.status, cfg.flags) == (2, 2, 5, None, 0)


def test_null_arguments_are_rejected_without_touching_a_gpu():
    L = _lib.lib()
    assert L.spmm_boo_matmul(None, None, None, 1, 1, None, None) == _lib.SPMM_EINVAL
    assert L.spmm_pbr_matmul(None, None, None, 1, 1, None, None) == _lib.SPMM_EINVAL
    sizes = _lib.BooDev()
    assert L.spmm_boo_build_analyze(None, None, None, 2, 4, 0, None, 0, C.byref(sizes),
                                    None) == _lib.SPMM_EINVAL
    a = _lib.CsrDev()
    a.rows, a.cols, a.nnz, a.index_type, a.scalar_type = 2, 2, 0, 0, 0
    a.indptr = 1  # never dereferenced: the merge policy is rejected first
    assert L.spmm_boo_build_analyze(C.byref(a), 1, 1, 1, 4, 0, 1, 1 << 20, C.byref(sizes),
                                    None) == _lib.SPMM_EINVAL
    p = _lib.PbrDev()
    assert L.spmm_pbr_build_analyze(C.byref(a), 8, 9, 4, 1, 1 << 20, C.byref(p),
                                    None) == _lib.SPMM_EINVAL
