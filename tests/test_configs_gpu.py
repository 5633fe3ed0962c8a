"""The five benchmark configurations on the GPU.

Reduced sizes: every format array bit-exact against the oracle, Y within
tol * (|A||X|) of the oracle's CPU SpMM.  Full sizes (C1 bit-exact; C2, C3 with
HEM grouping as configured, C4, C5 by properties): the oracle would take
minutes, so size-independent properties are checked instead --
exact agreement of the builder's counts with a host recount, linearity of the
product, and a float64 recomputation of a random sample of output rows."""

import numpy as np
import pytest
import torch

import spmm_b200 as S
from oracle import oracle as O
from spmm_b200 import workloads as W
from tests.conftest import TOL, abs_bound, assert_spmm_close

pytestmark = pytest.mark.gpu


def _eq(a, b):
    a, b = np.asarray(a), np.asarray(b)
    return a.shape == b.shape and np.array_equal(a.astype(b.dtype) if a.dtype != b.dtype else a, b)


SMALL = {
    'c1_laplacian2d': (lambda: W.laplacian2d(64), 'boo', 32, 128),
    'c2_fem3d': (lambda: W.fem3d(10), 'boo', 32, 128),
    'c3_powerlaw': (lambda: W.powerlaw(2500), 'boo', 32, 256),
    'c4_blockdiag': (lambda: W.blockdiag(64, 64), 'boo', 64, 512),
    'c5_uniform': (lambda: W.uniform(50000), 'pbr', 32, 64),
}


@pytest.mark.parametrize('name', list(SMALL))
def test_reduced_config(cuda, name):
    gen, fmt, target, K = SMALL[name]
    mat = gen()
    x = W.dense_x(mat.shape[1], K, seed=0)
    bound = abs_bound(mat.indptr, mat.indices, mat.data, x.numpy())
    cluster = 'hem' if name == 'c3_powerlaw' else 'identity'
    if fmt == 'boo' or name == 'c5_uniform':
        boo = S.csr_to_boo(mat, cluster=cluster, target_nr=target, target_nc=target)
        rl, cl = S.cluster_axes(mat, method=cluster, target_nr=target, target_nc=target,
                                max_nr=target, max_nc=target, feasible_first=True)
        ob = O.boo_build(mat.indptr, mat.indices, mat.data, mat.shape[0], mat.shape[1], rl, cl,
                         'remainder', 4, 'rowmajor')
        for f in O.BOO_FIELDS:
            assert _eq(getattr(boo, f), ob[f]), f
        y = S.boo_matmul(boo.to('cuda'), x.cuda()).cpu().numpy()
        assert_spmm_close(y, O.boo_matmul(ob, x.numpy()), bound, TOL[np.dtype(np.float32)])
    if fmt == 'pbr' or name == 'c2_fem3d':
        pbr = S.csr_to_pbr(mat, 8, 8, 4)
        op = O.pbr_build(mat.indptr, mat.indices, mat.data, mat.shape[0], mat.shape[1], 8, 8, 4)
        for f in O.PBR_FIELDS:
            assert _eq(getattr(pbr, f), op[f]), f
        y = S.pbr_matmul(pbr.to('cuda'), x.cuda()).cpu().numpy()
        assert_spmm_close(y, O.pbr_matmul(op, x.numpy()), bound, TOL[np.dtype(np.float32)])


def _sample_rows_f64(mat, x, rows):
    """Exact-ish float64 recomputation of a sample of output rows."""
    xd = x.double().numpy()
    out = np.zeros((rows.size, x.shape[1]))
    for i, r in enumerate(rows):
        s, e = mat.indptr[r], mat.indptr[r + 1]
        out[i] = mat.data[s:e].astype(np.float64) @ xd[mat.indices[s:e]]
    return out


def _properties(mat, matmul, K, seed=0):
    x1 = W.dense_x(mat.shape[1], K, seed=seed).cuda()
    x2 = W.dense_x(mat.shape[1], K, seed=seed + 1).cuda()
    y1, y2, y3 = matmul(x1), matmul(x2), matmul(x1 + 2 * x2)
    # linearity within the fp32 tolerance
    xa = (x1.abs() + 2 * x2.abs()).cpu().numpy()
    rows = np.random.default_rng(seed).choice(mat.shape[0], size=2000, replace=False)
    sub = mat[rows]
    bound = abs_bound(sub.indptr, sub.indices, sub.data, xa)
    lin = (y3 - y1 - 2 * y2)[torch.from_numpy(rows).cuda()].cpu().numpy()
    assert_spmm_close(lin, np.zeros_like(lin), bound, 3 * TOL[np.dtype(np.float32)])
    # sampled rows against a float64 recomputation
    ref = _sample_rows_f64(mat, x1.cpu(), rows)
    b1 = abs_bound(sub.indptr, sub.indices, sub.data, x1.abs().cpu().numpy())
    assert_spmm_close(y1[torch.from_numpy(rows).cuda()].cpu().numpy(), ref, b1, TOL[np.dtype(np.float32)])
    # every output row written (no stale memory): y of a zero X is exactly zero
    assert torch.count_nonzero(matmul(torch.zeros_like(x1))) == 0


def test_c1_full_size_bit_exact_build(cuda):
    mat = W.laplacian2d(256)
    assert mat.nnz == 326_656
    boo = S.csr_to_boo(mat, cluster='identity', target_nr=32, target_nc=32)
    rl = np.arange(mat.shape[0], dtype=np.int32) // 32
    ob = O.boo_build(mat.indptr, mat.indices, mat.data, mat.shape[0], mat.shape[1], rl, rl,
                     'remainder', 4, 'rowmajor')
    for f in O.BOO_FIELDS:
        assert _eq(getattr(boo, f), ob[f]), f
    assert (boo.num_blocks(), boo.compressed_nnz(), boo.remainder_nnz(), boo.max_nnz_blk) == \
        (ob['nb'], ob['nnz_c'], ob['rem_nnz'], ob['max_nnz_blk'])
    x = W.dense_x(mat.shape[1], 128, seed=0)
    y = S.boo_matmul(boo.to('cuda'), x.cuda()).cpu().numpy()
    bound = abs_bound(mat.indptr, mat.indices, mat.data, x.numpy())
    assert_spmm_close(y, O.boo_matmul(ob, x.numpy()), bound, TOL[np.dtype(np.float32)])


def test_c2_full_size_properties(cuda):
    mat = W.fem3d(64)
    assert mat.nnz == 61_731_000
    boo = S.csr_to_boo(mat, cluster='identity', target_nr=32, target_nc=32).to('cuda')
    assert boo.compressed_nnz() + boo.remainder_nnz() == mat.nnz
    assert boo.num_row_groups() == mat.shape[0] // 32
    _properties(mat, lambda x: S.boo_matmul(boo, x), 128)
    pbr = S.csr_to_pbr(mat, 8, 8, 4).to('cuda')
    assert pbr.compressed_nnz() + pbr.remainder_nnz() == mat.nnz
    _properties(mat, lambda x: S.pbr_matmul(pbr, x), 128, seed=5)


def test_c5_full_size_properties(cuda):
    mat = W.uniform()
    assert mat.nnz == 67_108_864
    pbr = S.csr_to_pbr(mat, 8, 8, 4).to('cuda')
    assert pbr.compressed_nnz() + pbr.remainder_nnz() == mat.nnz
    _properties(mat, lambda x: S.pbr_matmul(pbr, x), 64)


def test_c3_full_size_hem_properties(cuda):
    """C3 as the configuration names it: 2 M power-law rows grouped by HEM
    (labels on the GPU), remainder-major with scattered blocks -- the plan's
    row-ordered pass.  Also the same matrix with identity grouping."""
    mat = W.powerlaw()
    boo = S.csr_to_boo(mat, cluster='hem', target_nr=32, target_nc=32).to('cuda')
    s = boo._sizes
    assert boo.compressed_nnz() + boo.remainder_nnz() + boo.tail_nnz() == mat.nnz
    assert 2 * s['rem_nnz'] >= s['total_nnz'] and s['nnz_c'] > 0
    counts = np.bincount(boo.row_grp_ptr[1:] - boo.row_grp_ptr[:-1])
    assert counts.size <= 33                         # groups capped at the target
    _properties(mat, lambda x: S.boo_matmul(boo, x), 256)
    ident = S.csr_to_boo(mat, cluster='identity', target_nr=32, target_nc=32).to('cuda')
    _properties(mat, lambda x: S.boo_matmul(ident, x), 256, seed=3)


def test_c4_full_size_properties(cuda):
    """C4 at full size (4,096 dense 64 x 64 blocks + noise, K = 512) on the
    tensor cores and on CUDA cores."""
    mat = W.blockdiag()
    boo = S.csr_to_boo(mat, cluster='identity', target_nr=64, target_nc=64).to('cuda')
    assert boo.num_row_groups() == 4096
    assert boo.compressed_nnz() + boo.remainder_nnz() == mat.nnz
    _properties(mat, lambda x: S.boo_matmul(boo, x, engine='tensor_cores'), 512)
    _properties(mat, lambda x: S.boo_matmul(boo, x, engine='cuda_cores'), 512, seed=7)
