"""ctypes binding of ``libspmm_b200.so`` (declared in ``include/spmm_b200.h``).

The library is the only compute path of this package: there is no CPU
fallback.  Importing this module never touches a GPU; ``lib()`` raises
``ImportError`` when the shared library has not been built
(``python -m spmm_b200.build``).
"""

from __future__ import annotations

import ctypes as C
import os

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, 'libspmm_b200.so')

SPMM_OK = 0
SPMM_EINVAL = 1
SPMM_ELABEL = 2
SPMM_EOVERFLOW_U16 = 3
SPMM_EDUPLICATE = 4
SPMM_ECUDA = 5
SPMM_EWORKSPACE = 6
SPMM_EUNSUPPORTED = 7
SPMM_EALIGN = 8

I32, I64 = 0, 1
F32, F64 = 0, 1

SPMM_ESCRATCH = 9
SPMM_ETIMEOUT = 10
SPMM_ENCCL = 11

EXPORTS = ('spmm_status_string', 'spmm_abi_version', 'spmm_boo_build_workspace_size',
           'spmm_boo_build_analyze', 'spmm_boo_build_emit', 'spmm_boo_build_noalloc',
           'spmm_pbr_build_workspace_size',
           'spmm_pbr_build_analyze', 'spmm_pbr_build_emit', 'spmm_boo_matmul', 'spmm_pbr_matmul',
           'spmm_tc_status', 'spmm_boo_matmul_workspace_size', 'spmm_product_launches',
           'spmm_boo_to_csr_workspace_size', 'spmm_boo_to_csr', 'spmm_pbr_to_csr_workspace_size',
           'spmm_pbr_to_csr', 'spmm_hem_labels', 'spmm_hem_level_slots', 'spmm_hem_hierarchy',
           'spmm_boo_matmul_groups', 'spmm_boo_plan_size', 'spmm_boo_plan_workspace_size',
           'spmm_boo_plan_build')


class CsrDev(C.Structure):
    _fields_ = [('rows', C.c_int64), ('cols', C.c_int64), ('nnz', C.c_int64),
                ('indptr', C.c_void_p), ('indices', C.c_void_p), ('values', C.c_void_p),
                ('index_type', C.c_int32), ('scalar_type', C.c_int32)]


BOO_PTR_FIELDS = ('row_grp_ptr', 'row_ids', 'col_grp_ptr', 'col_ids', 'blk_row_grp', 'blk_col_grp',
                  'blk_nz_ptr', 'blk_shift', 'nz_idx', 'nz_val', 'rem_indptr', 'rem_col_ind',
                  'rem_vals', 'tail_row', 'tail_col', 'tail_val')
BOO_SIZE_FIELDS = ('rows', 'cols', 'total_nnz', 'n_rg', 'n_cg', 'nb', 'nnz_c', 'rem_nnz', 'tail_nnz',
                   'max_nr', 'max_nc', 'max_nnz_blk')


class BooDev(C.Structure):
    _fields_ = ([(n, C.c_int64) for n in BOO_SIZE_FIELDS]
                + [('nz_order', C.c_int32), ('scalar_type', C.c_int32)]
                + [(n, C.c_void_p) for n in BOO_PTR_FIELDS])


PBR_PTR_FIELDS = ('codes', 'coords', 'offsets', 'data', 'rem_indptr', 'rem_col_ind', 'rem_vals')
PBR_SIZE_FIELDS = ('rows', 'cols', 'block_rows', 'block_cols', 'total_nnz', 'nb', 'nnz_c', 'rem_nnz')


class PbrDev(C.Structure):
    _fields_ = ([(n, C.c_int64) for n in PBR_SIZE_FIELDS]
                + [('index_type', C.c_int32), ('scalar_type', C.c_int32)]
                + [(n, C.c_void_p) for n in PBR_PTR_FIELDS])


class LaunchCfg(C.Structure):
    _fields_ = [('version', C.c_int32), ('slab_features', C.c_int32), ('engine', C.c_int32),
                ('wait_us', C.c_int32), ('workspace', C.c_void_p), ('workspace_bytes', C.c_uint64),
                ('status', C.c_void_p), ('flags', C.c_int32), ('reserved', C.c_int32), ('plan', C.c_void_p)]


SPMM_CFG_EXPIRE_FIRST_WAIT = 1


ENGINES = {'auto': 0, 'cuda_cores': 1, 'tensor_cores': 2, 'tensor_cores_tf32': 3}


def launch_cfg(engine: str = 'auto', workspace: int = 0, workspace_bytes: int = 0,
               slab_features: int = 0, status: int = 0, wait_us: int = 0, flags: int = 0,
               plan: int = 0) -> 'LaunchCfg':
    """spmm_launch_cfg (version 2): engine, remainder slab setting, workspace
    and the call's device status word (0 / None: none)."""
    if engine not in ENGINES:
        raise ValueError(f"engine must be one of {sorted(ENGINES)}, got {engine!r}")
    return LaunchCfg(2, int(slab_features), ENGINES[engine], int(wait_us), workspace or None, workspace_bytes,
                     status or None, int(flags), 0, plan or None)


class SpmmError(RuntimeError):
    """A non-OK status from the C ABI."""

    def __init__(self, status: int, where: str):
        self.status = status
        super().__init__(f'{where}: {status_string(status)} (status {status})')


_LIB = None


def lib() -> C.CDLL:
    global _LIB
    if _LIB is None:
        if not os.path.exists(LIB_PATH):
            raise ImportError(f'{LIB_PATH} is missing: build it with `python -m spmm_b200.build`')
        L = C.CDLL(LIB_PATH)
        L.spmm_status_string.restype = C.c_char_p
        L.spmm_status_string.argtypes = [C.c_int]
        L.spmm_abi_version.restype = C.c_int
        for n in ('spmm_boo_build_workspace_size', 'spmm_pbr_build_workspace_size'):
            getattr(L, n).restype = C.c_size_t
            getattr(L, n).argtypes = [C.c_int64, C.c_int64, C.c_int64]
        L.spmm_boo_build_analyze.argtypes = [C.POINTER(CsrDev), C.c_void_p, C.c_void_p, C.c_int,
                                             C.c_int64, C.c_int, C.c_void_p, C.c_size_t,
                                             C.POINTER(BooDev), C.c_void_p]
        L.spmm_boo_build_emit.argtypes = L.spmm_boo_build_analyze.argtypes
        L.spmm_boo_build_noalloc.argtypes = [C.POINTER(CsrDev), C.c_void_p, C.c_void_p, C.c_int,
                                             C.c_int64, C.c_int, C.POINTER(BooDev), C.c_void_p]
        L.spmm_boo_build_noalloc.restype = C.c_int
        L.spmm_pbr_build_analyze.argtypes = [C.POINTER(CsrDev), C.c_int64, C.c_int64, C.c_int,
                                             C.c_void_p, C.c_size_t, C.POINTER(PbrDev), C.c_void_p]
        L.spmm_pbr_build_emit.argtypes = L.spmm_pbr_build_analyze.argtypes
        L.spmm_boo_matmul.argtypes = [C.POINTER(BooDev), C.c_void_p, C.c_void_p, C.c_int64, C.c_int64,
                                      C.POINTER(LaunchCfg), C.c_void_p]
        L.spmm_pbr_matmul.argtypes = [C.POINTER(PbrDev), C.c_void_p, C.c_void_p, C.c_int64, C.c_int64,
                                      C.POINTER(LaunchCfg), C.c_void_p]
        L.spmm_boo_matmul_groups.argtypes = [C.POINTER(BooDev), C.c_void_p, C.c_void_p, C.c_int64, C.c_int64,
                                             C.c_int64, C.c_int64, C.POINTER(LaunchCfg), C.c_void_p]
        L.spmm_boo_matmul_groups.restype = C.c_int
        for n in ('spmm_boo_plan_size', 'spmm_boo_plan_workspace_size'):
            getattr(L, n).argtypes = [C.POINTER(BooDev)]
            getattr(L, n).restype = C.c_size_t
        L.spmm_boo_plan_build.argtypes = [C.POINTER(BooDev), C.c_void_p, C.c_size_t, C.c_void_p, C.c_size_t,
                                          C.c_void_p]
        L.spmm_boo_plan_build.restype = C.c_int
        L.spmm_boo_matmul_workspace_size.argtypes = [C.POINTER(BooDev), C.c_int64, C.c_int64,
                                                     C.POINTER(LaunchCfg)]
        L.spmm_boo_matmul_workspace_size.restype = C.c_size_t
        L.spmm_tc_status.argtypes = [C.c_int]
        L.spmm_tc_status.restype = C.c_int
        L.spmm_product_launches.argtypes = []
        L.spmm_product_launches.restype = C.c_uint64
        L.spmm_boo_to_csr_workspace_size.argtypes = [C.POINTER(BooDev)]
        L.spmm_boo_to_csr_workspace_size.restype = C.c_size_t
        L.spmm_pbr_to_csr_workspace_size.argtypes = [C.POINTER(PbrDev)]
        L.spmm_pbr_to_csr_workspace_size.restype = C.c_size_t
        L.spmm_boo_to_csr.argtypes = [C.POINTER(BooDev), C.c_void_p, C.c_void_p, C.c_void_p, C.c_int,
                                      C.c_void_p, C.c_size_t, C.c_void_p]
        L.spmm_pbr_to_csr.argtypes = [C.POINTER(PbrDev), C.c_void_p, C.c_void_p, C.c_void_p, C.c_int,
                                      C.c_void_p, C.c_size_t, C.c_void_p]
        L.spmm_boo_to_csr.restype = C.c_int
        L.spmm_hem_labels.argtypes = [C.c_int64, C.c_int64, C.c_void_p, C.c_void_p, C.c_int64, C.c_int64,
                                      C.c_int64, C.c_int64, C.c_int64, C.c_int32, C.c_int32, C.c_void_p,
                                      C.c_void_p]
        L.spmm_hem_labels.restype = C.c_int
        L.spmm_hem_level_slots.argtypes = [C.c_int64]
        L.spmm_hem_level_slots.restype = C.c_int64
        L.spmm_hem_hierarchy.argtypes = [C.c_int64, C.c_int64, C.c_void_p, C.c_void_p, C.c_int64, C.c_int64,
                                         C.c_int64, C.c_int64, C.c_int64, C.c_int32, C.c_int32, C.c_void_p,
                                         C.c_void_p, C.c_int64, C.POINTER(C.c_int64), C.c_void_p]
        L.spmm_hem_hierarchy.restype = C.c_int
        L.spmm_pbr_to_csr.restype = C.c_int
        for n in ('spmm_boo_build_analyze', 'spmm_boo_build_emit', 'spmm_pbr_build_analyze',
                  'spmm_pbr_build_emit', 'spmm_boo_matmul', 'spmm_pbr_matmul'):
            getattr(L, n).restype = C.c_int
        _LIB = L
    return _LIB


def status_string(status: int) -> str:
    try:
        return lib().spmm_status_string(int(status)).decode()
    except ImportError:
        return f'status {status}'


def check(status: int, where: str) -> None:
    if status != SPMM_OK:
        raise SpmmError(status, where)
