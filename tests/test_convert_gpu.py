"""GPU inverse conversions (spmm_boo_to_csr / spmm_pbr_to_csr, behind
boo_to_csr / pbr_to_csr) against the oracle's restatement of the
reference's boo_to_csr / pbr_to_csr (boo_matrix.cpp:277-333,
pbr_matrix.cpp:279-331): indptr, indices and values bit for bit, each row
ordered by (column, value) -- duplicates, blocks, remainder and tail."""

import numpy as np
import pytest
import scipy.sparse as sp

import spmm_b200 as S
from oracle import oracle as O

pytestmark = pytest.mark.gpu


def _dup_csr(rows, cols, per_row, rng, dtype, index_dtype):
    """A non-canonical CSR: unsorted columns, repeated (row, col) entries with
    different values, some empty rows."""
    lens = rng.integers(0, per_row + 1, rows)
    lens[rng.random(rows) < 0.1] = 0
    indptr = np.concatenate([[0], np.cumsum(lens)]).astype(index_dtype)
    indices = rng.integers(0, cols, indptr[-1]).astype(index_dtype)
    dup = rng.random(indptr[-1]) < 0.2                       # copy the previous entry's column
    dup[0:1] = False
    indices[dup] = np.roll(indices, 1)[dup]
    data = rng.choice([-1.5, -0.25, 0.0, 0.5, 2.0, 3.0], indptr[-1]).astype(dtype)
    mat = sp.csr_matrix((rows, cols), dtype=dtype)
    mat.indptr, mat.indices, mat.data = indptr, indices, data
    return mat


def _oracle_boo_csr(boo):
    d = {f: getattr(boo, f) for f in O.BOO_FIELDS}
    d.update(rows=boo.rows, cols=boo.cols, total_nnz=boo.total_nnz, nb=boo.num_blocks(),
             tail_nnz=len(boo.tail_row))
    return O.boo_to_csr(d)


def _assert_csr(got, ref, index_dtype, dtype):
    """Values bit for bit; the index dtype is scipy's choice, as for the
    reference's own csr_matrix((data, indices, indptr)) construction."""
    ip, ix, dv = ref
    assert got.data.dtype == dtype
    del index_dtype
    np.testing.assert_array_equal(got.indptr, ip)
    np.testing.assert_array_equal(got.indices, ix)
    np.testing.assert_array_equal(got.data, dv)


@pytest.mark.parametrize('seed', range(8))
def test_boo_to_csr_matches_oracle(cuda, seed):
    rng = np.random.default_rng(300 + seed)
    dtype = (np.float32, np.float64)[seed % 2]
    index_dtype = (np.int32, np.int64)[(seed // 2) % 2]
    rows, cols = int(rng.integers(1, 700)), int(rng.integers(1, 700))
    mat = _dup_csr(rows, cols, 12, rng, dtype, index_dtype)
    policy = ('keep', 'remainder', 'tail_batch')[seed % 3]
    order = ('rowmajor', 'colmajor')[seed % 2]
    boo = S.csr_to_boo(mat, row_labels=rng.integers(0, max(1, rows // 16), rows),
                       col_labels=rng.integers(0, max(1, cols // 16), cols), small_block_policy=policy,
                       small_block_threshold=int(rng.integers(1, 6)), nz_order=order)
    got = S.boo_to_csr(boo)
    _assert_csr(got, _oracle_boo_csr(boo), index_dtype, dtype)
    got_dev = S.boo_to_csr(boo.to('cuda'))                  # from the device-resident object too
    _assert_csr(got_dev, _oracle_boo_csr(boo), index_dtype, dtype)


def test_boo_to_csr_large_and_empty(cuda):
    rng = np.random.default_rng(9)
    mat = sp.random(20000, 15000, density=0.002, format='csr', random_state=3, dtype=np.float32)
    boo = S.csr_to_boo(mat, cluster='identity', target_nr=32, target_nc=32, small_block_policy='tail_batch',
                       small_block_threshold=3)
    _assert_csr(S.boo_to_csr(boo), _oracle_boo_csr(boo), np.int32, np.float32)
    empty = sp.csr_matrix((5, 7), dtype=np.float64)
    be = S.csr_to_boo(empty, cluster='identity')
    out = S.boo_to_csr(be)
    assert out.shape == (5, 7) and out.nnz == 0 and np.array_equal(out.indptr, np.zeros(6))
    del rng


@pytest.mark.parametrize('seed', range(6))
def test_pbr_to_csr_matches_oracle(cuda, seed):
    rng = np.random.default_rng(500 + seed)
    dtype = (np.float32, np.float64)[seed % 2]
    index_dtype = (np.int32, np.int64)[(seed // 2) % 2]
    rows, cols = int(rng.integers(1, 900)), int(rng.integers(1, 900))
    mat = sp.random(rows, cols, density=float(rng.uniform(0.005, 0.1)), format='csr', random_state=seed,
                    dtype=np.float64)
    mat.data = rng.choice([-2.0, -0.5, 0.0, 1.0, 4.0], mat.nnz)
    mat = mat.astype(dtype)
    mat.indptr, mat.indices = mat.indptr.astype(index_dtype), mat.indices.astype(index_dtype)
    br, bc = [(2, 2), (4, 4), (8, 8), (3, 5)][seed % 4]
    pbr = S.csr_to_pbr(mat, br, bc, int(rng.integers(1, 5)))
    ref = dict(rows=pbr.rows, cols=pbr.cols, block_rows=br, block_cols=bc, total_nnz=pbr.total_nnz,
               **{f: getattr(pbr, f) for f in O.PBR_FIELDS})
    _assert_csr(S.pbr_to_csr(pbr), O.pbr_to_csr(ref), index_dtype, dtype)
