"""ctypes front end of the C oracle (oracle/spmm_oracle.c).

TEST INFRASTRUCTURE ONLY.  The product (``spmm_b200``) never imports this
module; tests, ``__graft_entry__.smoke()`` and ``bench.py``'s ``cpu_baseline``
leg use it as the checker.  Array names and semantics follow the reference's
``boo_matrix_t`` (torch_fast_spdmm/boo_matrix/boo_matrix.hpp:56-138) and
``pbr_matrix_t`` (torch_fast_spdmm/pbr_matrix/pbr_matrix.hpp:98-167).

All index arrays come back as int64; values keep the input's float dtype.
"""

from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, 'liboracle.so')
SOURCES = [os.path.join(HERE, n) for n in ('spmm_oracle.c', 'spmm_oracle.h', 'spmm_oracle_body.h',
                                            'hem_oracle.c')]

POLICY_CODE = {'keep': 0, 'merge': 1, 'remainder': 2, 'tail_batch': 3}
ORDER_CODE = {'rowmajor': 0, 'colmajor': 1}
ERRORS = {1: 'cluster label out of range', 2: 'block local index space exceeds uint16',
          3: "'merge' policy is a clustering-level column relabel",
          4: 'unknown small_block_policy', 5: 'unknown nz_order',
          6: 'label array length must match matrix dims', 7: 'out of memory'}

BOO_FIELDS = ('row_grp_ptr', 'row_ids', 'col_grp_ptr', 'col_ids', 'blk_row_grp', 'blk_col_grp',
              'blk_nz_ptr', 'blk_shift', 'nz_idx', 'nz_val', 'rem_indptr', 'rem_col_ind',
              'rem_vals', 'tail_row', 'tail_col', 'tail_val')
PBR_FIELDS = ('block_codes', 'block_coords', 'block_offsets', 'block_data',
              'remainder_indptr', 'remainder_col_ind', 'remainder_data')


class OracleError(ValueError):
    def __init__(self, code: int):
        super().__init__(f'oracle: {ERRORS.get(code, code)}')
        self.code = code


def build_lib(force: bool = False) -> str:
    """Compile liboracle.so with gcc (no -march: plain SSE2 arithmetic, no FMA)."""
    stale = (not os.path.exists(LIB_PATH) or
             any(os.path.getmtime(s) > os.path.getmtime(LIB_PATH) for s in SOURCES))
    if force or stale:
        tmp = LIB_PATH + f'.{os.getpid()}.tmp'
        subprocess.check_call(['gcc', '-O2', '-std=c11', '-fPIC', '-shared', '-o', tmp,
                               os.path.join(HERE, 'spmm_oracle.c'), os.path.join(HERE, 'hem_oracle.c')])
        os.replace(tmp, LIB_PATH)
    return LIB_PATH


class _Boo(C.Structure):
    _fields_ = ([(n, C.c_int64) for n in ('rows', 'cols', 'total_nnz', 'n_rg', 'n_cg', 'nb', 'nnz_c',
                                           'rem_nnz', 'tail_nnz', 'max_nr', 'max_nc', 'max_nnz_blk')]
                + [('nz_order', C.c_int32), ('scalar_size', C.c_int32)]
                + [(n, C.c_void_p) for n in BOO_FIELDS])


class _Pbr(C.Structure):
    _fields_ = ([(n, C.c_int64) for n in ('rows', 'cols', 'block_rows', 'block_cols', 'total_nnz',
                                           'nb', 'nnz_c', 'rem_nnz')]
                + [('scalar_size', C.c_int32)]
                + [(n, C.c_void_p) for n in ('codes', 'coords', 'offsets', 'data', 'rem_indptr',
                                             'rem_col_ind', 'rem_vals')])


_LIB = None


def lib():
    global _LIB
    if _LIB is None:
        _LIB = C.CDLL(build_lib())
        for sfx in ('f32', 'f64'):
            getattr(_LIB, f'oracle_csr_to_boo_{sfx}').restype = C.c_int
            getattr(_LIB, f'oracle_csr_to_pbr_{sfx}').restype = C.c_int
            getattr(_LIB, f'oracle_pbr_to_csr_{sfx}').restype = C.c_int
        _LIB.oracle_hem_labels.restype = C.c_int
        _LIB.oracle_hem_level_slots.restype = C.c_int64
        _LIB.oracle_hem_level_slots.argtypes = [C.c_int64]
        _LIB.oracle_enforce_caps.restype = C.c_int
    return _LIB


def _p(a):
    return a.ctypes.data_as(C.c_void_p)


def _sfx(dtype) -> str:
    dtype = np.dtype(dtype)
    if dtype == np.float32:
        return 'f32'
    if dtype == np.float64:
        return 'f64'
    raise TypeError(f'oracle supports float32/float64, got {dtype}')


def _copy(ptr, n, dtype):
    if n == 0:
        return np.zeros(0, dtype=dtype)
    buf = (C.c_char * (n * np.dtype(dtype).itemsize)).from_address(ptr)
    return np.frombuffer(buf, dtype=dtype).copy()


def _csr_args(indptr, indices, data):
    indptr = np.ascontiguousarray(indptr, dtype=np.int64)
    indices = np.ascontiguousarray(indices, dtype=np.int64)
    data = np.ascontiguousarray(data)
    _sfx(data.dtype)
    return indptr, indices, data


# ----------------------------------------------------------------------------
# BOO
# ----------------------------------------------------------------------------

def boo_build(indptr, indices, data, rows, cols, row_labels, col_labels,
              policy='remainder', threshold=4, nz_order='rowmajor') -> dict:
    """csr_to_boo (boo_matrix.cpp:53-274).  Returns a dict of numpy arrays + scalars."""
    indptr, indices, data = _csr_args(indptr, indices, data)
    rl = np.ascontiguousarray(row_labels, dtype=np.int32)
    cl = np.ascontiguousarray(col_labels, dtype=np.int32)
    pol = POLICY_CODE[policy] if isinstance(policy, str) else int(policy)
    order = ORDER_CODE[nz_order] if isinstance(nz_order, str) else int(nz_order)
    out = _Boo()
    fn = getattr(lib(), f'oracle_csr_to_boo_{_sfx(data.dtype)}')
    rc = fn(C.c_int64(rows), C.c_int64(cols), C.c_int64(data.size), _p(indptr), _p(indices),
            _p(data), _p(rl), C.c_int64(rl.size), _p(cl), C.c_int64(cl.size), C.c_int(pol),
            C.c_int64(threshold), C.c_int(order), C.byref(out))
    if rc:
        lib().oracle_boo_free(C.byref(out))
        raise OracleError(rc)
    sd = data.dtype
    res = {k: int(getattr(out, k)) for k in ('rows', 'cols', 'total_nnz', 'n_rg', 'n_cg', 'nb', 'nnz_c',
                                              'rem_nnz', 'tail_nnz', 'max_nr', 'max_nc', 'max_nnz_blk')}
    res['nz_order'] = int(out.nz_order)
    sizes = {'row_grp_ptr': (res['n_rg'] + 1, np.int64), 'row_ids': (rows, np.int64),
             'col_grp_ptr': (res['n_cg'] + 1, np.int64), 'col_ids': (cols, np.int64),
             'blk_row_grp': (res['nb'], np.int64), 'blk_col_grp': (res['nb'], np.int64),
             'blk_nz_ptr': (res['nb'] + 1, np.int64), 'blk_shift': (res['nb'], np.uint8),
             'nz_idx': (res['nnz_c'], np.uint16), 'nz_val': (res['nnz_c'], sd),
             'rem_indptr': (rows + 1, np.int64), 'rem_col_ind': (res['rem_nnz'], np.int64),
             'rem_vals': (res['rem_nnz'], sd), 'tail_row': (res['tail_nnz'], np.int64),
             'tail_col': (res['tail_nnz'], np.int64), 'tail_val': (res['tail_nnz'], sd)}
    for name, (n, dt) in sizes.items():
        res[name] = _copy(getattr(out, name), n, dt)
    lib().oracle_boo_free(C.byref(out))
    return res


def _x3(x):
    x = np.asarray(x)
    return (x[None] if x.ndim == 2 else x), x.ndim == 2


def boo_matmul(b: dict, x) -> np.ndarray:
    """boo_batched_matmul_cpu (boo_matrix.cpp:336-396): blocks, remainder, tail,
    accumulated serially in the value dtype."""
    x3, squeeze = _x3(x)
    sd = np.asarray(b['nz_val']).dtype
    x3 = np.ascontiguousarray(x3, dtype=sd)
    bt, _, k = x3.shape
    rows = int(b['rows'])
    y = np.empty((bt, rows, k), dtype=sd)
    a = {n: np.ascontiguousarray(b[n], dtype=(np.int64 if n not in ('blk_shift', 'nz_idx', 'nz_val',
                                                                     'rem_vals', 'tail_val') else None))
         for n in BOO_FIELDS}
    a['blk_shift'] = np.ascontiguousarray(b['blk_shift'], dtype=np.uint8)
    a['nz_idx'] = np.ascontiguousarray(b['nz_idx'], dtype=np.uint16)
    for n in ('nz_val', 'rem_vals', 'tail_val'):
        a[n] = np.ascontiguousarray(b[n], dtype=sd)
    fn = getattr(lib(), f'oracle_boo_matmul_{_sfx(sd)}')
    fn(C.c_int64(rows), C.c_int64(int(b['cols'])), C.c_int64(a['blk_row_grp'].size),
       _p(a['row_grp_ptr']), _p(a['row_ids']), _p(a['col_grp_ptr']), _p(a['col_ids']),
       _p(a['blk_row_grp']), _p(a['blk_col_grp']), _p(a['blk_nz_ptr']), _p(a['blk_shift']),
       _p(a['nz_idx']), _p(a['nz_val']), _p(a['rem_indptr']), _p(a['rem_col_ind']),
       _p(a['rem_vals']), C.c_int64(a['tail_val'].size), _p(a['tail_row']), _p(a['tail_col']),
       _p(a['tail_val']), _p(x3), C.c_int64(bt), C.c_int64(k), _p(y))
    return y[0] if squeeze else y


def boo_to_csr(b: dict):
    """boo_to_csr (boo_matrix.cpp:277-333) -> (indptr, indices, data)."""
    sd = np.asarray(b['nz_val']).dtype
    st = _Boo()
    keep = {}
    for k in ('rows', 'cols', 'total_nnz', 'nb', 'tail_nnz'):
        setattr(st, k, int(b[k]))
    for n in BOO_FIELDS:
        dt = {'blk_shift': np.uint8, 'nz_idx': np.uint16, 'nz_val': sd, 'rem_vals': sd,
              'tail_val': sd}.get(n, np.int64)
        keep[n] = np.ascontiguousarray(b[n], dtype=dt)
        setattr(st, n, keep[n].ctypes.data)
    total = int(b['total_nnz'])
    indptr = np.zeros(int(b['rows']) + 1, np.int64)
    indices = np.zeros(total, np.int64)
    data = np.zeros(total, sd)
    getattr(lib(), f'oracle_boo_to_csr_{_sfx(sd)}')(C.byref(st), _p(indptr), _p(indices), _p(data))
    return indptr, indices, data


# ----------------------------------------------------------------------------
# PBR
# ----------------------------------------------------------------------------

def pbr_build(indptr, indices, data, rows, cols, block_rows=8, block_cols=8,
              min_nnz_per_block=4) -> dict:
    """csr_to_pbr (pbr_matrix.cpp:333-448) with blocks in canonical (stripe, column) order."""
    indptr, indices, data = _csr_args(indptr, indices, data)
    out = _Pbr()
    fn = getattr(lib(), f'oracle_csr_to_pbr_{_sfx(data.dtype)}')
    rc = fn(C.c_int64(rows), C.c_int64(cols), C.c_int64(data.size), _p(indptr), _p(indices),
            _p(data), C.c_int64(block_rows), C.c_int64(block_cols),
            C.c_uint8(int(min_nnz_per_block) & 0xFF), C.byref(out))
    if rc:
        lib().oracle_pbr_free(C.byref(out))
        raise OracleError(rc)
    sd = data.dtype
    nb, nnz_c, rem = int(out.nb), int(out.nnz_c), int(out.rem_nnz)
    res = dict(rows=rows, cols=cols, block_rows=block_rows, block_cols=block_cols,
               total_nnz=int(data.size), nb=nb, nnz_c=nnz_c, rem_nnz=rem)
    res['block_codes'] = _copy(out.codes, nb, np.uint64)
    res['block_coords'] = _copy(out.coords, 2 * nb, np.int64)
    res['block_offsets'] = _copy(out.offsets, nb + 1, np.int64)
    res['block_data'] = _copy(out.data, nnz_c, sd)
    res['remainder_indptr'] = _copy(out.rem_indptr, rows + 1, np.int64)
    res['remainder_col_ind'] = _copy(out.rem_col_ind, rem, np.int64)
    res['remainder_data'] = _copy(out.rem_vals, rem, sd)
    lib().oracle_pbr_free(C.byref(out))
    return res


def pbr_matmul(p: dict, x) -> np.ndarray:
    """pbr_batched_matmul_cpu (pbr_matrix.cpp:17-68), blocks in the order given."""
    x3, squeeze = _x3(x)
    sd = np.asarray(p['block_data']).dtype
    x3 = np.ascontiguousarray(x3, dtype=sd)
    bt, _, k = x3.shape
    rows = int(p['rows'])
    y = np.empty((bt, rows, k), dtype=sd)
    codes = np.ascontiguousarray(p['block_codes'], dtype=np.uint64)
    coords = np.ascontiguousarray(p['block_coords'], dtype=np.int64)
    data = np.ascontiguousarray(p['block_data'], dtype=sd)
    ri = np.ascontiguousarray(p['remainder_indptr'], dtype=np.int64)
    rc = np.ascontiguousarray(p['remainder_col_ind'], dtype=np.int64)
    rv = np.ascontiguousarray(p['remainder_data'], dtype=sd)
    getattr(lib(), f'oracle_pbr_matmul_{_sfx(sd)}')(
        C.c_int64(rows), C.c_int64(int(p['cols'])), C.c_int64(int(p['block_rows'])),
        C.c_int64(int(p['block_cols'])), C.c_int64(codes.size), _p(codes), _p(coords), _p(data),
        _p(ri), _p(rc), _p(rv), _p(x3), C.c_int64(bt), C.c_int64(k), _p(y))
    return y[0] if squeeze else y


def pbr_to_csr(p: dict):
    """pbr_to_csr (pbr_matrix.cpp:279-331) -> (indptr, indices, data)."""
    sd = np.asarray(p['block_data']).dtype
    st = _Pbr()
    for k in ('rows', 'cols', 'block_rows', 'block_cols', 'total_nnz'):
        setattr(st, k, int(p[k]))
    st.nb = int(np.asarray(p['block_codes']).size)
    keep = dict(codes=np.ascontiguousarray(p['block_codes'], dtype=np.uint64),
                coords=np.ascontiguousarray(p['block_coords'], dtype=np.int64),
                offsets=np.ascontiguousarray(p['block_offsets'], dtype=np.int64),
                data=np.ascontiguousarray(p['block_data'], dtype=sd),
                rem_indptr=np.ascontiguousarray(p['remainder_indptr'], dtype=np.int64),
                rem_col_ind=np.ascontiguousarray(p['remainder_col_ind'], dtype=np.int64),
                rem_vals=np.ascontiguousarray(p['remainder_data'], dtype=sd))
    for n, a in keep.items():
        setattr(st, n, a.ctypes.data)
    total = int(p['total_nnz'])
    indptr = np.zeros(int(p['rows']) + 1, np.int64)
    indices = np.zeros(total, np.int64)
    data = np.zeros(total, sd)
    rc = getattr(lib(), f'oracle_pbr_to_csr_{_sfx(sd)}')(C.byref(st), _p(indptr), _p(indices), _p(data))
    if rc:
        raise RuntimeError('Block has a nonzero past the last matrix row.')
    return indptr, indices, data


# ----------------------------------------------------------------------------
# helpers for comparing against the reference's own objects
# ----------------------------------------------------------------------------

def reference_boo_arrays(obj) -> dict:
    """Arrays + scalars of a reference BOOMatrix* object as a plain dict."""
    res = {n: np.asarray(getattr(obj, n)).copy() for n in BOO_FIELDS}
    res.update(rows=int(obj.rows), cols=int(obj.cols), total_nnz=int(obj.total_nnz),
               max_nr=int(obj.max_nr), max_nc=int(obj.max_nc), max_nnz_blk=int(obj.max_nnz_blk),
               nz_order=int(obj.nz_order), nb=int(obj.num_blocks()),
               n_rg=int(obj.num_row_groups()), n_cg=int(obj.num_col_groups()),
               nnz_c=int(obj.compressed_nnz()), rem_nnz=int(obj.remainder_nnz()),
               tail_nnz=int(obj.tail_nnz()))
    return res


def reference_pbr_arrays(obj) -> dict:
    res = {n: np.asarray(getattr(obj, n)).copy() for n in PBR_FIELDS}
    res.update(rows=int(obj.rows), cols=int(obj.cols), block_rows=int(obj.block_rows),
               block_cols=int(obj.block_cols), total_nnz=int(obj.total_nnz),
               nb=int(obj.accounted_blocks()), nnz_c=int(obj.compressed_nnz()),
               rem_nnz=int(obj.remainder_nnz()))
    return res


def pbr_canonical(p: dict) -> dict:
    """Re-sort PBR blocks by (row, col) of their top-left corner, carrying each
    block's code, data segment and offsets along.  The reference emits blocks
    of a stripe in std::unordered_map order (pbr_matrix.cpp:396); this puts any
    PBR array set into the canonical order the GPU builder emits."""
    coords = np.asarray(p['block_coords'], dtype=np.int64).reshape(-1, 2)
    nb = coords.shape[0]
    order = np.lexsort((coords[:, 1], coords[:, 0]))
    offsets = np.asarray(p['block_offsets'], dtype=np.int64)
    data = np.asarray(p['block_data'])
    out = dict(p)
    out['block_codes'] = np.asarray(p['block_codes'], dtype=np.uint64)[order]
    out['block_coords'] = coords[order].reshape(-1)
    if nb:
        seg = [data[offsets[b]:offsets[b + 1]] for b in order]
        out['block_data'] = np.concatenate(seg) if seg else data[:0]
        lens = np.diff(offsets)[order]
        out['block_offsets'] = np.concatenate([[0], np.cumsum(lens)]).astype(np.int64)
    return out


# ----------------------------------------------------------------------------
# clustering (hem_oracle.c)
# ----------------------------------------------------------------------------

def binary_pattern(mat):
    """Canonical binary CSR pattern of `mat` (rows sorted, duplicates merged)."""
    import scipy.sparse as sp
    a = sp.csr_matrix(mat, copy=True)
    a.sum_duplicates()
    a.sort_indices()
    a.data = np.ones(a.nnz, dtype=np.int8)
    return a


def hem_labels(pat, target, max_size=None, max_nnz=None, hub_degree=1024, topk=32,
               residual_rounds=3, feasible_first=False, hierarchy: bool = False):
    """HEM labels of the rows of a canonical binary pattern, before cap
    enforcement (clustering.py:128-351).  With ``hierarchy``, returns
    (labels, [identity, labels after level 1, ...])."""
    n, m = pat.shape
    indptr = np.ascontiguousarray(pat.indptr, dtype=np.int64)
    indices = np.ascontiguousarray(pat.indices, dtype=np.int64)
    labels = np.empty(n, dtype=np.int64)
    slots = int(lib().oracle_hem_level_slots(int(target)))
    hier = np.empty((slots, max(n, 1)), dtype=np.int64) if hierarchy else None
    nlev = C.c_int64(0)
    neg = lambda v: -1 if v is None else int(v)  # noqa: E731
    rc = lib().oracle_hem_labels(
        C.c_int64(n), C.c_int64(m), _p(indptr), _p(indices), C.c_int64(int(target)), C.c_int64(neg(max_size)),
        C.c_int64(neg(max_nnz)), C.c_int64(int(hub_degree)), C.c_int64(neg(topk)), C.c_int32(residual_rounds),
        C.c_int32(1 if feasible_first else 0), _p(labels), _p(hier) if hier is not None else None,
        C.byref(nlev))
    if rc:
        raise OracleError(7)
    if hierarchy:
        return labels, [hier[k, :n].copy() for k in range(nlev.value)]
    return labels


def enforce_caps(labels, row_nnz, max_size=None, max_nnz=None):
    """Cap enforcement + consecutive relabelling (clustering.py:83-121)."""
    lab = np.ascontiguousarray(labels, dtype=np.int64).copy()
    nz = np.ascontiguousarray(row_nnz, dtype=np.int64)
    if lab.size and lib().oracle_enforce_caps(C.c_int64(lab.size), _p(lab), _p(nz),
                                              C.c_int64(-1 if max_size is None else int(max_size)),
                                              C.c_int64(-1 if max_nnz is None else int(max_nnz))):
        raise OracleError(7)
    return lab


def hem_cluster(mat, target, max_size=None, max_nnz=None, hub_degree=1024, topk=32, feasible_first=False):
    """int32 HEM group label per row of `mat`: the reference's
    cluster_axis(method='hem') (clustering.py:454-509)."""
    pat = binary_pattern(mat)
    if pat.shape[0] == 0:
        return np.zeros(0, dtype=np.int32)
    lab = hem_labels(pat, target, max_size, max_nnz, hub_degree, topk, feasible_first=feasible_first)
    return enforce_caps(lab, np.diff(pat.indptr), max_size, max_nnz).astype(np.int32)
