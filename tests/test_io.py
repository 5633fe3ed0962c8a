"""On-disk BOO / PBR formats (CPU): save -> load gives the same class, sizes
and arrays bit for bit; wrong files are rejected."""

import numpy as np
import pytest
import scipy.sparse as sp

from oracle import oracle as O
from spmm_b200 import boo as B
from spmm_b200 import io
from spmm_b200 import pbr as P


def _boo_from_oracle(mat, cls):
    rows, cols = mat.shape
    ob = O.boo_build(mat.indptr, mat.indices, mat.data, rows, cols, np.arange(rows) // 8, np.arange(cols) // 8,
                     'tail_batch', 3, 'rowmajor')
    sizes = {k: int(ob[k]) for k in ('rows', 'cols', 'total_nnz', 'max_nr', 'max_nc', 'max_nnz_blk')}
    sizes.update(n_rg=len(ob['row_grp_ptr']) - 1, n_cg=len(ob['col_grp_ptr']) - 1, nb=len(ob['blk_shift']),
                 nnz_c=len(ob['nz_val']), rem_nnz=len(ob['rem_vals']), tail_nnz=len(ob['tail_val']), nz_order=0)
    obj = cls(sizes, None)
    idt, sdt = B._BOO_TYPE_MAP[cls.__name__]
    obj._host = {n: np.asarray(ob[n]).astype({'nz_idx': np.uint16, 'blk_shift': np.uint8}.get(
        n, sdt if B._DEV_DTYPES[n] is None else idt)) for n in B._DEV_DTYPES}
    return obj


@pytest.mark.parametrize('cls', [B.BOOMatrixInt32Float, B.BOOMatrixInt64Double])
def test_boo_roundtrip(tmp_path, cls):
    mat = sp.random(100, 90, density=0.08, format='csr', random_state=1,
                    dtype=np.float32 if 'Float' in cls.__name__ else np.float64)
    obj = _boo_from_oracle(mat, cls)
    path = tmp_path / 'm.npz'
    io.save_boo(path, obj)
    back = io.load_boo(path)
    assert type(back) is cls and back._sizes == obj._sizes
    for n in B._DEV_DTYPES:
        a, b = obj._host[n], getattr(back, n)
        assert a.dtype == b.dtype and np.array_equal(a, b), n
    with pytest.raises(ValueError):
        io.load_pbr(path)


def test_pbr_roundtrip(tmp_path):
    mat = sp.random(64, 80, density=0.1, format='csr', random_state=2, dtype=np.float32)
    op = O.pbr_build(mat.indptr, mat.indices, mat.data, 64, 80, 8, 8, 2)
    sizes = dict(rows=64, cols=80, block_rows=8, block_cols=8, total_nnz=mat.nnz, nb=len(op['block_codes']),
                 nnz_c=len(op['block_data']), rem_nnz=len(op['remainder_data']))
    obj = P.PBRMatrixInt32Float(sizes, None)
    obj._host = {n: np.asarray(op[n]) for n in io._PBR_ARRAYS}
    obj._host['block_codes'] = obj._host['block_codes'].astype(np.uint64)
    for n in ('block_coords', 'block_offsets', 'remainder_indptr', 'remainder_col_ind'):
        obj._host[n] = obj._host[n].astype(np.int32)
    path = tmp_path / 'p.npz'
    io.save_pbr(path, obj)
    back = io.load_pbr(path)
    assert type(back) is P.PBRMatrixInt32Float and back._sizes == sizes
    for n in io._PBR_ARRAYS:
        assert np.array_equal(obj._host[n], getattr(back, n)), n
    with pytest.raises(TypeError):
        io.save_boo(path, obj)
