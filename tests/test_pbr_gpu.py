"""PBR on the GPU against the oracle and the reference's golden fixtures.

Format arrays bit-exact (blocks in canonical (stripe, column) order; the
reference's fixtures are re-sorted that way); Y within tol * (|A||X|).
Cases follow the reference's tests/torch_fast_spdmm/test_pbr.py."""

import json
import os

import numpy as np
import pytest
import scipy.sparse as sp
import torch

import spmm_b200 as S
from oracle import oracle as O
from tests.conftest import TOL, abs_bound, assert_spmm_close

pytestmark = pytest.mark.gpu

GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), 'golden')
MANIFEST = json.load(open(os.path.join(GOLD, 'manifest.json')))
PBR = np.load(os.path.join(GOLD, 'pbr_golden.npz'))


def _eq(a, b):
    a, b = np.asarray(a), np.asarray(b)
    return a.shape == b.shape and np.array_equal(a.astype(b.dtype) if a.dtype != b.dtype else a, b)


def _arrays(p):
    return {f: getattr(p, f) for f in O.PBR_FIELDS}


def _check_product(mat, pbr, x):
    got = S.pbr_matmul(pbr, x)
    xn = x.detach().cpu().numpy()
    ref = O.pbr_matmul(dict(_arrays(pbr), rows=pbr.rows, cols=pbr.cols, block_rows=pbr.block_rows,
                            block_cols=pbr.block_cols), xn)
    bound = abs_bound(mat.indptr, mat.indices, mat.data, xn)
    assert_spmm_close(got.cpu().numpy(), ref, bound, TOL[np.dtype(mat.dtype)])
    return got


@pytest.mark.parametrize('case', MANIFEST['pbr'], ids=lambda c: f"pbr{c['case']}")
def test_gpu_build_and_product_match_reference_fixture(cuda, case):
    p = f"p{case['case']}/"
    g = {k[len(p):]: PBR[k] for k in PBR.files if k.startswith(p)}
    mat = sp.csr_matrix((g['data'], g['indices'], g['indptr']), shape=(case['rows'], case['cols']))
    mat.indptr, mat.indices = g['indptr'], g['indices']   # keep the fixture's index dtype
    pbr = S.csr_to_pbr(mat, case['block_rows'], case['block_cols'], case['min_nnz'])
    ref = dict(rows=case['rows'], cols=case['cols'], block_rows=case['block_rows'],
               block_cols=case['block_cols'], **{f: g[f] for f in O.PBR_FIELDS})
    canon = O.pbr_canonical(ref)
    for f in O.PBR_FIELDS:
        assert _eq(getattr(pbr, f), canon[f]), f
    y = S.pbr_matmul(pbr.to('cuda'), torch.from_numpy(g['x']).to(cuda)).cpu().numpy()
    bound = abs_bound(g['indptr'], g['indices'], g['data'], g['x'])
    assert_spmm_close(y, g['y'], bound, TOL[g['data'].dtype])
    out = S.pbr_to_csr(pbr)
    assert _eq(out.indptr, g['csr_indptr']) and _eq(out.indices, g['csr_indices'])
    assert _eq(out.data, g['csr_data'])


def _fixture(kind, n, dtype):
    rng = np.random.default_rng(n)
    if kind == 'identity':
        return sp.eye(n, dtype=dtype, format='csr')
    if kind == 'permutation':
        return sp.csr_matrix((np.ones(n, dtype=dtype), (np.arange(n), rng.permutation(n))), shape=(n, n))
    return sp.random(n, n, density=0.9, format='csr', random_state=n, dtype=dtype)


@pytest.mark.parametrize('kind', ['identity', 'permutation', 'dense_random'])
@pytest.mark.parametrize('index_dtype', [np.int32, np.int64])
@pytest.mark.parametrize('data_dtype', [np.float32, np.float64])
@pytest.mark.parametrize('system_size', [8, 16])
@pytest.mark.parametrize('block_size', [4, 8])
@pytest.mark.parametrize('min_nnz', [1, 7])
def test_roundtrip_and_meta(cuda, kind, index_dtype, data_dtype, system_size, block_size, min_nnz):
    mat = _fixture(kind, system_size, data_dtype)
    mat.indptr, mat.indices = mat.indptr.astype(index_dtype), mat.indices.astype(index_dtype)
    pbr = S.csr_to_pbr(mat, block_rows=block_size, block_cols=block_size, min_nnz_per_block=min_nnz)
    out = S.pbr_to_csr(pbr)
    np.testing.assert_array_equal(out.indptr, mat.indptr)
    np.testing.assert_array_equal(out.indices, mat.indices)
    np.testing.assert_allclose(out.data, mat.data)
    meta = pbr.to('cuda')._gpu_meta
    it = torch.int32 if index_dtype == np.int32 else torch.int64
    st = torch.float32 if data_dtype == np.float32 else torch.float64
    for name in ('coords', 'offsets', 'rem_indptr', 'rem_col_ind'):
        assert getattr(meta, name).dtype == it, name
    assert meta.data.dtype == st and meta.rem_vals.dtype == st and meta.codes.dtype == torch.int64
    x = torch.randn((1, system_size, 8), dtype=st, device='cuda')
    _check_product(mat, pbr, x)


@pytest.mark.parametrize('rows', [1, 9, 13, 17, 1001])
@pytest.mark.parametrize('block', [(4, 4), (8, 8), (2, 32), (3, 5)])
@pytest.mark.parametrize('min_nnz', [1, 4, 64])
def test_partial_last_stripe(cuda, rows, block, min_nnz):
    rng = np.random.default_rng(0)
    mat = sp.random(rows, rows, density=0.3, format='lil', dtype=np.float32, random_state=rng)
    mat[rows - 1, rng.integers(0, rows, size=min(3, rows))] = 1.0
    mat = mat.tocsr()
    mat.sort_indices()
    pbr = S.csr_to_pbr(mat, block_rows=block[0], block_cols=block[1], min_nnz_per_block=min_nnz)
    ob = O.pbr_build(mat.indptr, mat.indices, mat.data, rows, rows, block[0], block[1], min_nnz)
    for f in O.PBR_FIELDS:
        assert _eq(getattr(pbr, f), ob[f]), f
    out = S.pbr_to_csr(pbr)
    np.testing.assert_array_equal(out.indices, mat.indices)
    _check_product(mat, pbr.to('cuda'), torch.randn((1, rows, 32), device='cuda'))


@pytest.mark.parametrize('K', [1, 3, 8, 32, 100, 127, 200, 520, 1000])
def test_any_feature_count(cuda, K):
    """The reference's block kernel is only right when K is a power-of-two
    multiple of its shared-memory tile (pbr_kernel.cu:81-87); every K works here."""
    mat = sp.random(300, 280, density=0.05, format='csr', random_state=2, dtype=np.float32)
    pbr = S.csr_to_pbr(mat, 8, 8, 2).to('cuda')
    _check_product(mat, pbr, torch.randn((2, 280, K), device='cuda'))


def test_unsorted_input_matches_reference_semantics(cuda):
    """Columns out of order within rows (no duplicates): block values keep CSR
    order and a spilled block's k-th set bit takes its k-th value, as in the
    reference (pbr_matrix.cpp:389, 407-416); the oracle restates that."""
    rng = np.random.default_rng(3)
    rows, cols = 120, 90
    ind, dat, ptr = [], [], [0]
    for r in range(rows):
        c = list(rng.choice(cols, size=int(rng.integers(0, 15)), replace=False))
        rng.shuffle(c)
        ind += c
        dat += list(rng.standard_normal(len(c)))
        ptr.append(len(ind))
    mat = sp.csr_matrix((np.array(dat, np.float64), np.array(ind, np.int32), np.array(ptr, np.int32)),
                        shape=(rows, cols))
    for mn in (1, 3, 9):
        pbr = S.csr_to_pbr(mat, 8, 8, mn)
        ob = O.pbr_build(mat.indptr, mat.indices, mat.data, rows, cols, 8, 8, mn)
        for f in O.PBR_FIELDS:
            assert _eq(getattr(pbr, f), ob[f]), (mn, f)


def test_duplicates_rejected(cuda):
    mat = sp.csr_matrix((np.array([1., 2., 3.]), np.array([1, 1, 0]), np.array([0, 2, 3])), shape=(2, 2))
    with pytest.raises(ValueError, match='duplicate'):
        S.csr_to_pbr(mat, 2, 2, 1)


def test_staging_cpu_x_and_errors(cuda):
    mat = sp.random(50, 40, density=0.2, format='csr', random_state=4, dtype=np.float32)
    pbr = S.csr_to_pbr(mat, 8, 8, 2)
    x = torch.randn(40, 7)
    y_cpu = S.pbr_matmul(pbr, x)            # host operands, GPU product
    assert y_cpu.device.type == 'cpu' and y_cpu.shape == (50, 7)
    with pytest.raises(RuntimeError, match="to\\('cuda'\\)"):
        S.pbr_matmul(pbr, x.cuda())
    pbr.to('cuda')
    assert pbr.to('cuda') is pbr
    y = S.pbr_matmul(pbr, x.cuda(), kernel='nnzflat')
    torch.testing.assert_close(y.cpu(), y_cpu, rtol=0, atol=0)
    with pytest.raises(ValueError, match='2D or 3D'):
        S.pbr_matmul(pbr, torch.zeros(40, device='cuda'))
    info = S.pbr_info(pbr)
    assert info.total_nnz == mat.nnz and info.num_blocks == pbr.accounted_blocks()
    pbr.to('cpu')
    assert pbr._gpu_meta is None
    torch.testing.assert_close(S.pbr_matmul(pbr, x), y_cpu, rtol=0, atol=0)


@pytest.mark.parametrize('dtype', [np.float32, np.float64])
@pytest.mark.parametrize('bs', [8, 4, 2])
@pytest.mark.parametrize('k', [128, 192, 256])
def test_block_major_stripe_path(cuda, dtype, bs, k):
    """Block-major matrices (most entries in blocks: a mesh stiffness pattern)
    take the warp-per-stripe kernel: every shape the reference launches, a
    partial last feature slab (K = 192), a batch of two, a partial last
    stripe (rows not a multiple of the block size) and rows with remainder
    entries next to blocks."""
    from spmm_b200 import workloads
    mat = workloads.fem3d(n=7).astype(dtype)[:1027]          # 1027 rows: a partial last stripe
    mat = sp.csr_matrix(mat)
    extra = sp.random(1027, mat.shape[1], density=0.002, format='csr', random_state=bs, dtype=dtype)
    mat = (mat + extra).tocsr()
    mat.sum_duplicates()
    mat.sort_indices()
    pbr = S.csr_to_pbr(mat, bs, bs, 4)
    assert 2 * pbr.compressed_nnz() >= pbr.total_nnz and pbr.remainder_nnz() > 0
    tdt = torch.float32 if dtype == np.float32 else torch.float64
    x = torch.from_numpy(np.random.default_rng(k + bs).standard_normal((2, mat.shape[1], k))).to(tdt)
    _check_product(mat, pbr.to('cuda'), x.cuda())
