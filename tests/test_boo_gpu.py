"""BOO on the GPU against the oracle and the reference's golden fixtures.

Format arrays must be bit-exact; Y within max|dY| <= tol * (|A||X|)
elementwise (tol 1e-5 fp32, 1e-12 fp64).  Edge cases follow the reference's
tests/torch_fast_spdmm/test_boo_edges.py and test_boo.py."""

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
BOO = np.load(os.path.join(GOLD, 'boo_golden.npz'))
POLICIES = ['keep', 'remainder', 'tail_batch']
PCODE = {'keep': 0, 'remainder': 2, 'tail_batch': 3}


def _eq(a, b):
    a, b = np.asarray(a), np.asarray(b)
    return a.shape == b.shape and np.array_equal(a.astype(b.dtype) if a.dtype != b.dtype else a, b)


def _check_arrays(boo, ref: dict):
    for f in O.BOO_FIELDS:
        assert _eq(getattr(boo, f), ref[f]), f
    for f, m in (('nb', 'num_blocks'), ('nnz_c', 'compressed_nnz'), ('rem_nnz', 'remainder_nnz'),
                 ('tail_nnz', 'tail_nnz'), ('n_rg', 'num_row_groups'), ('n_cg', 'num_col_groups')):
        if f in ref:
            assert getattr(boo, m)() == ref[f], f
    for f in ('max_nr', 'max_nc', 'max_nnz_blk', 'total_nnz'):
        if f in ref:
            assert getattr(boo, f) == ref[f], f


def _build(mat, rl, cl, policy='keep', order='rowmajor', threshold=4):
    return S.csr_to_boo(mat, row_labels=rl, col_labels=cl, small_block_policy=policy,
                        small_block_threshold=threshold, nz_order=order)


def _x(shape, dtype=torch.float32, seed=123):
    return torch.randn(shape, dtype=dtype, generator=torch.Generator().manual_seed(seed))


def _check_product(mat, boo, x, **kw):
    """GPU product vs the oracle's CPU SpMM (the reference's algorithm)."""
    got = S.boo_matmul(boo, x, **kw)
    assert got.dtype == x.dtype and got.device == x.device
    xn = x.detach().cpu().numpy()
    ref = O.boo_matmul(_oracle_arrays(boo), xn)
    bound = abs_bound(mat.indptr, mat.indices, mat.data, xn)
    assert got.shape == ref.shape
    assert_spmm_close(got.cpu().numpy(), ref, bound, TOL[np.dtype(mat.dtype)])
    return got


def _labels_of(boo):
    rl = np.empty(boo.rows, np.int32)
    rgp = boo.row_grp_ptr
    for g in range(len(rgp) - 1):
        rl[boo.row_ids[rgp[g]:rgp[g + 1]]] = g
    cl = np.empty(boo.cols, np.int32)
    cgp = boo.col_grp_ptr
    for g in range(len(cgp) - 1):
        cl[boo.col_ids[cgp[g]:cgp[g + 1]]] = g
    return rl, cl


def _oracle_arrays(boo):
    d = {f: getattr(boo, f) for f in O.BOO_FIELDS}
    d.update(rows=boo.rows, cols=boo.cols)
    return d


def _example(dtype=np.float32, index_dtype=np.int32):
    entries = [(0, 0, 2), (0, 2, -1), (2, 6, 3), (2, 0, 1), (0, 1, 4), (1, 1, 2), (1, 4, -3),
               (4, 7, 1), (4, 9, 2), (4, 3, -2), (3, 5, 1)]
    r, c, v = zip(*entries)
    mat = sp.csr_matrix((np.array(v, dtype=dtype), (r, c)), shape=(7, 11))
    mat.indptr = mat.indptr.astype(index_dtype)
    mat.indices = mat.indices.astype(index_dtype)
    return mat, np.array([0, 1, 0, 2, 1, 0, 2]), np.array([0, 1, 0, 2, 1, 2, 0, 1, 2, 1, 2])


# ---------------------------------------------------------------------------
# against the reference's own outputs
# ---------------------------------------------------------------------------

@pytest.mark.parametrize('case', MANIFEST['boo'], ids=lambda c: f"boo{c['case']}")
def test_gpu_build_and_product_match_reference_fixture(cuda, case):
    p = f"b{case['case']}/"
    g = {k[len(p):]: BOO[k] for k in BOO.files if k.startswith(p)}
    mat = sp.csr_matrix((g['data'], g['indices'], g['indptr']), shape=(case['rows'], case['cols']))
    mat.indptr, mat.indices = g['indptr'], g['indices']   # keep the fixture's index dtype
    policy = {0: 'keep', 2: 'remainder', 3: 'tail_batch'}[case['policy']]
    order = ('rowmajor', 'colmajor')[case['order']]
    boo = _build(mat, g['row_labels'], g['col_labels'], policy, order, case['threshold'])
    assert type(boo).__name__.startswith('BOOMatrixInt' + ('32' if g['indptr'].dtype == np.int32 else '64'))
    _check_arrays(boo, dict(g, **{k: case[k] for k in ('max_nr', 'max_nc', 'max_nnz_blk', 'total_nnz')}))
    y = S.boo_matmul(boo.to('cuda'), torch.from_numpy(g['x']).to(cuda)).cpu().numpy()
    bound = abs_bound(g['indptr'], g['indices'], g['data'], g['x'])
    assert_spmm_close(y, g['y'], bound, TOL[g['data'].dtype])
    ip = S.boo_to_csr(boo)
    assert _eq(ip.indptr, g['csr_indptr']) and _eq(ip.indices, g['csr_indices'])
    assert _eq(ip.data, g['csr_data'])


# ---------------------------------------------------------------------------
# seeded sweep against the oracle
# ---------------------------------------------------------------------------

@pytest.mark.parametrize('seed', range(24))
def test_seeded_sweep(cuda, seed):
    rng = np.random.default_rng(1000 + seed)
    rows, cols = int(rng.integers(1, 400)), int(rng.integers(1, 400))
    dtype = np.float32 if seed % 2 == 0 else np.float64
    idt = np.int32 if seed % 3 else np.int64
    mat = sp.random(rows, cols, density=float(rng.uniform(0.005, 0.3)), format='csr',
                    random_state=seed, dtype=np.float64)
    mat.data = rng.standard_normal(mat.nnz)
    mat = mat.astype(dtype)
    mat.indptr, mat.indices = mat.indptr.astype(idt), mat.indices.astype(idt)
    rl = rng.integers(0, max(1, rows // int(rng.integers(1, 40))), size=rows)
    cl = rng.integers(0, max(1, cols // int(rng.integers(1, 40))), size=cols)
    policy = POLICIES[seed % 3]
    order = ('rowmajor', 'colmajor')[(seed // 3) % 2]
    thr = int(rng.integers(0, 10))
    boo = _build(mat, rl, cl, policy, order, thr)
    ob = O.boo_build(mat.indptr, mat.indices, mat.data, rows, cols, rl, cl, policy, thr, order)
    _check_arrays(boo, ob)
    k = int(rng.choice([1, 3, 4, 17, 32, 64, 100, 128, 200, 256, 520]))
    x = _x((int(rng.integers(1, 3)), cols, k), torch.float32 if dtype == np.float32 else torch.float64,
           seed)
    _check_product(mat, boo.to('cuda'), x.cuda())


# ---------------------------------------------------------------------------
# edge contract (test_boo_edges.py)
# ---------------------------------------------------------------------------

@pytest.mark.parametrize('order', ['rowmajor', 'colmajor'])
@pytest.mark.parametrize('policy', POLICIES)
@pytest.mark.parametrize('index_dtype', [np.int32, np.int64])
def test_explicit_format(cuda, order, policy, index_dtype):
    mat, rl, cl = _example(np.float64, index_dtype)
    boo = _build(mat, rl, cl, policy, order)
    assert f'Int{np.dtype(index_dtype).itemsize * 8}' in type(boo).__name__
    np.testing.assert_array_equal(S.boo_to_csr(boo).toarray(), mat.toarray())
    assert boo.compressed_nnz() == (11 if policy == 'keep' else 8)
    assert boo.remainder_nnz() == (3 if policy == 'remainder' else 0)
    assert boo.tail_nnz() == (3 if policy == 'tail_batch' else 0)
    _check_product(mat, boo.to('cuda'), _x((3, 11, 9), torch.float64).cuda())


@pytest.mark.parametrize('order', ['rowmajor', 'colmajor'])
@pytest.mark.parametrize('features', [1, 7, 8, 9, 31, 32, 33, 63, 64, 65, 127, 128, 129, 255, 256,
                                      257, 511, 512, 513, 1025])
@pytest.mark.parametrize('dtype', [torch.float32, torch.float64])
def test_feature_boundaries(cuda, order, features, dtype):
    mat, rl, cl = _example(np.float32 if dtype == torch.float32 else np.float64)
    boo = _build(mat, rl, cl, order=order).to('cuda')
    _check_product(mat, boo, _x((2, 11, features), dtype).cuda())


@pytest.mark.parametrize('policy,threshold', [('remainder', 4), ('tail_batch', 4),
                                              ('remainder', 100), ('tail_batch', 100)])
def test_mixed_and_all_spilled(cuda, policy, threshold):
    mat, rl, cl = _example()
    boo = _build(mat, rl, cl, policy, 'rowmajor', threshold).to('cuda')
    assert boo.compressed_nnz() == (8 if threshold == 4 else 0)
    spill = boo.remainder_nnz() if policy == 'remainder' else boo.tail_nnz()
    assert spill == (3 if threshold == 4 else mat.nnz)
    for csr_mode in (0, 2):
        _check_product(mat, boo, _x((2, 11, 65)).cuda(), csr_mode=csr_mode)


@pytest.mark.parametrize('device', ['cpu', 'cuda'])
@pytest.mark.parametrize('shape', [(0, 0), (0, 5), (5, 0), (5, 7)])
@pytest.mark.parametrize('policy', POLICIES)
def test_empty_matrix(cuda, device, shape, policy):
    mat = sp.csr_matrix(shape, dtype=np.float32)
    boo = S.csr_to_boo(mat, cluster='identity', small_block_policy=policy).to(device)
    assert boo.num_blocks() == boo.total_nnz == 0
    np.testing.assert_array_equal(S.boo_to_csr(boo).toarray(), mat.toarray())
    for row_seg in (True, False):
        y = S.boo_matmul(boo, _x((2, shape[1], 9)).to(device), row_seg=row_seg)
        assert y.shape == (2, shape[0], 9) and y.device.type == device
        assert torch.count_nonzero(y) == 0


@pytest.mark.parametrize('device', ['cpu', 'cuda'])
@pytest.mark.parametrize('x_shape', [(11, 0), (0, 11, 9), (2, 11, 0)])
def test_empty_dense_dimensions(cuda, device, x_shape):
    mat, rl, cl = _example()
    boo = _build(mat, rl, cl, 'remainder').to(device)
    y = S.boo_matmul(boo, _x(x_shape).to(device))
    exp = (7, 0) if len(x_shape) == 2 else (x_shape[0], 7, x_shape[2])
    assert tuple(y.shape) == exp


@pytest.mark.parametrize('order', ['rowmajor', 'colmajor'])
@pytest.mark.parametrize('shape', [(1, 1), (1, 17), (19, 1)])
def test_singleton_axes(cuda, order, shape):
    mat = sp.csr_matrix(np.arange(1, np.prod(shape) + 1, dtype=np.float32).reshape(shape))
    boo = _build(mat, np.zeros(shape[0], int), np.zeros(shape[1], int), order=order).to('cuda')
    _check_product(mat, boo, _x((shape[1], 33)).cuda())


@pytest.mark.parametrize('order', ['rowmajor', 'colmajor'])
def test_many_blocks_accumulate_exactly(cuda, order):
    mat = sp.csr_matrix(np.ones((3, 257), dtype=np.float32))
    boo = _build(mat, np.zeros(3, int), np.arange(257), order=order).to('cuda')
    assert boo.num_blocks() == 257
    x = torch.ones(257, 17, device='cuda')
    for _ in range(3):
        got = S.boo_matmul(boo, x)
        torch.testing.assert_close(got.cpu(), torch.full((3, 17), 257.), rtol=0, atol=0)


@pytest.mark.parametrize('device', ['cpu', 'cuda'])
@pytest.mark.parametrize('layout', ['transpose', 'slice', 'expand', 'batch_transpose'])
def test_noncontiguous_x(cuda, device, layout):
    mat, rl, cl = _example()
    boo = _build(mat, rl, cl, 'remainder').to(device)
    if layout == 'transpose':
        x = _x((13, 11)).to(device).T
    elif layout == 'slice':
        x = _x((11, 26)).to(device)[:, 1::2]
    elif layout == 'expand':
        x = _x((11, 1)).to(device).expand(11, 13)
    else:
        x = _x((3, 13, 11)).to(device).transpose(1, 2)
    assert not x.is_contiguous()
    saved = x.clone()
    _check_product(mat, boo, x)
    torch.testing.assert_close(x, saved, rtol=0, atol=0)


@pytest.mark.parametrize('order', ['rowmajor', 'colmajor'])
def test_uint16_high_bit_and_last_coordinate(cuda, order):
    mat = sp.csr_matrix((np.array([2, -3, 4], np.float64), ([0, 128, 255], [0, 1, 255])),
                        shape=(256, 256))
    labels = np.zeros(256, dtype=np.int32)
    boo = _build(mat, labels, labels, order=order).to('cuda')
    assert max(boo.nz_idx) == 65535
    _check_product(mat, boo, _x((256, 9), torch.float64).cuda())


@pytest.mark.parametrize('order', ['rowmajor', 'colmajor'])
@pytest.mark.parametrize('shape', [(32, 64), (256, 256), (300, 7)])
def test_large_blocks_are_tiled(cuda, order, shape):
    """A block larger than the CTA's staging buffer (65,536 nonzeros here) is
    processed in pieces; the reference raises RuntimeError('CUDA...') there
    because its shared-memory arena cannot hold it."""
    mat = sp.csr_matrix(np.random.default_rng(0).standard_normal(shape))
    boo = _build(mat, np.zeros(shape[0], int), np.zeros(shape[1], int), order=order).to('cuda')
    _check_product(mat, boo, _x((2, shape[1], 129), torch.float64).cuda())


@pytest.mark.parametrize('order', ['rowmajor', 'colmajor'])
def test_coordinate_overflow_rejected(cuda, order):
    mat = sp.csr_matrix(([1.0], ([256], [255])), shape=(257, 256), dtype=np.float32)
    with pytest.raises(ValueError, match='uint16'):
        _build(mat, np.zeros(257, int), np.zeros(256, int), order=order)


@pytest.mark.parametrize('seed', range(12))
def test_seeded_randomized_product(cuda, seed):
    rng = np.random.default_rng(seed)
    rows, cols = int(rng.integers(2, 40)), int(rng.integers(2, 50))
    dtype = np.float32 if seed % 2 else np.float64
    tdt = torch.float32 if seed % 2 else torch.float64
    dense = rng.normal(size=(rows, cols))
    dense[rng.random((rows, cols)) > (0.05 + 0.07 * seed)] = 0
    mat = sp.csr_matrix(dense.astype(dtype))
    rl = rng.integers(0, min(rows, 5), size=rows)
    cl = rng.integers(0, min(cols, 6), size=cols)
    features = [1, 17, 65, 129, 513, 1025][seed % 6]
    for order in ('rowmajor', 'colmajor'):
        boo = _build(mat, rl, cl, POLICIES[seed % 3], order).to('cuda')
        _check_product(mat, boo, _x((2, cols, features), tdt, seed).cuda())


@pytest.mark.parametrize('device', ['cpu', 'cuda'])
@pytest.mark.parametrize('order', ['rowmajor', 'colmajor'])
def test_unsorted_duplicates_and_explicit_zeros(cuda, device, order):
    mat = sp.csr_matrix((np.array([2., -2., 0., 3., 4.]), np.array([3, 3, 1, 0, 2]),
                         np.array([0, 4, 5, 5])), shape=(3, 5))
    assert not mat.has_canonical_format
    for policy, thr in (('keep', 0), ('remainder', 9), ('tail_batch', 9)):
        boo = _build(mat, np.zeros(3, int), np.zeros(5, int), policy, order, thr)
        ob = O.boo_build(mat.indptr, mat.indices, mat.data, 3, 5, np.zeros(3), np.zeros(5), policy,
                         thr, order)
        _check_arrays(boo, ob)
        np.testing.assert_array_equal(S.boo_to_csr(boo).toarray(), mat.toarray())
        _check_product(mat, boo.to(device), _x((5, 17), torch.float64).to(device))


def test_unsorted_remainder_order_matches_oracle(cuda):
    """Rows with shuffled columns and duplicate entries spilled to the
    remainder: rows sorted by (col, value) exactly as the reference does."""
    rng = np.random.default_rng(5)
    rows, cols = 200, 300
    ind, dat, ptr = [], [], [0]
    for r in range(rows):
        c = list(rng.choice(cols, size=int(rng.integers(0, 12)), replace=False))
        c += [c[0]] * int(rng.integers(0, 3)) if c else []
        rng.shuffle(c)
        ind += c
        dat += list(rng.standard_normal(len(c)))
        ptr.append(len(ind))
    mat = sp.csr_matrix((np.array(dat, np.float32), np.array(ind, np.int32), np.array(ptr, np.int32)),
                        shape=(rows, cols))
    rl = rng.integers(0, 20, size=rows)
    cl = rng.integers(0, 25, size=cols)
    for policy in POLICIES:
        boo = _build(mat, rl, cl, policy, 'rowmajor', 3)
        _check_arrays(boo, O.boo_build(mat.indptr, mat.indices, mat.data, rows, cols, rl, cl, policy,
                                       3, 'rowmajor'))


@pytest.mark.parametrize('policy', POLICIES)
def test_nondefault_stream_producer_consumer(cuda, policy):
    mat, rl, cl = _example()
    boo = _build(mat, rl, cl, policy).to('cuda')
    stream = torch.cuda.Stream()
    outputs = []
    base = _x((13, 11))
    with torch.cuda.stream(stream):
        for i in range(8):
            x = (base.to('cuda') + i).T
            outputs.append(S.boo_matmul(boo, x, row_seg=bool(i % 2)) * 2 + 1)
    stream.synchronize()
    for i, got in enumerate(outputs):
        expected = torch.from_numpy(mat.toarray()).double() @ (base.double() + i).T
        torch.testing.assert_close(got.cpu().double(), expected * 2 + 1, rtol=3e-5, atol=3e-5)


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason='requires two GPUs')
def test_noncurrent_device_and_device_mismatch():
    mat, rl, cl = _example()
    with torch.cuda.device(0):
        boo = _build(mat, rl, cl).to('cuda:1')
        _check_product(mat, boo, _x((11, 17)).to('cuda:1'))
        assert torch.cuda.current_device() == 0
        with pytest.raises(ValueError, match='same CUDA device'):
            S.boo_matmul(boo, _x((11, 17)).to('cuda:0'))


def test_device_staging_is_idempotent_and_reversible(cuda):
    mat, rl, cl = _example()
    boo = _build(mat, rl, cl).to('cuda')
    meta = boo._gpu_meta
    assert boo.to('cuda') is boo and boo._gpu_meta is meta
    boo.to('cpu')
    _check_product(mat, boo, _x((11, 17)))
    with pytest.raises(RuntimeError, match='not'):
        S.boo_matmul(boo, _x((11, 17)).cuda())
    _check_product(mat, boo.to('cuda'), _x((11, 17)).cuda())


def test_invalid_x_contract(cuda):
    mat, rl, cl = _example()
    for device in ('cpu', 'cuda'):
        boo = _build(mat, rl, cl).to(device)
        for shape in [(11,), (1, 1, 11, 3)]:
            with pytest.raises(ValueError, match='2D or 3D'):
                S.boo_matmul(boo, torch.zeros(shape, device=device))
        with pytest.raises(ValueError, match='rows'):
            S.boo_matmul(boo, torch.zeros(10, 3, device=device))
        for dtype in (torch.float64, torch.float16, torch.int32, torch.complex64):
            with pytest.raises(TypeError, match='dtype'):
                S.boo_matmul(boo, torch.zeros(11, 3, dtype=dtype, device=device))
        with pytest.raises(ValueError, match='dense'):
            S.boo_matmul(boo, torch.zeros(11, 3, device=device).to_sparse())


@pytest.mark.parametrize('kwargs', [{'p': 0}, {'p': 4}, {'p': 12}, {'p': 256}, {'threads': 0},
                                    {'threads': 192}, {'threads': 1024}, {'csr_mode': 3}])
def test_invalid_launch_parameters(cuda, kwargs):
    mat, rl, cl = _example()
    boo = _build(mat, rl, cl).to('cuda')
    with pytest.raises(ValueError):
        S.boo_matmul(boo, _x((11, 17)).cuda(), **kwargs)


def test_rowseg_rejects_column_major(cuda):
    mat, rl, cl = _example()
    boo = _build(mat, rl, cl, order='colmajor').to('cuda')
    with pytest.raises(ValueError, match='rowmajor'):
        S.boo_matmul(boo, _x((11, 17)).cuda(), row_seg=True)


def test_torch_csr_input_and_default_clustering(cuda):
    mat, rl, cl = _example()
    t = torch.sparse_csr_tensor(torch.from_numpy(mat.indptr), torch.from_numpy(mat.indices),
                                torch.from_numpy(mat.data), size=mat.shape)
    boo = S.csr_to_boo(t, row_labels=rl, col_labels=cl)
    np.testing.assert_array_equal(S.boo_to_csr(boo).toarray(), mat.toarray())
    a = sp.random(300, 300, density=0.02, format='csr', random_state=1, dtype=np.float32)
    boo = S.csr_to_boo(a)   # default: cluster='hem', target 32
    rl2, cl2 = S.cluster_axes(a, method='hem', target_nr=32, target_nc=32, max_nr=32, max_nc=32,
                              feasible_first=True)
    ob = O.boo_build(a.indptr, a.indices, a.data, 300, 300, rl2, cl2, 'remainder', 4, 'rowmajor')
    _check_arrays(boo, ob)


def test_boo_info_fields(cuda):
    mat, rl, cl = _example()
    info = S.boo_info(_build(mat, rl, cl, 'remainder'))
    assert info.total_nnz == 11 and info.compressed_nnz == 8 and info.remainder_nnz == 3
    assert info.compressed_fraction == pytest.approx(8 / 11)
