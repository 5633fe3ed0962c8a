"""BOO product on the tensor cores (tcgen05 3xTF32) against the oracle.

The tensor-core engine must meet the float32 bar of the CUDA-core engine:
max|dY| <= 1e-5 * (|A||X|) elementwise, with the reference's semantics for
non-finite values (a NaN or Inf reaches exactly the rows whose nonzeros use
it).  Engines are forced through boo_matmul(..., engine=...)."""

import numpy as np
import pytest
import scipy.sparse as sp
import torch

import spmm_b200 as S
from oracle import oracle as O
from spmm_b200 import _lib, workloads
from tests.conftest import TOL, abs_bound, assert_spmm_close

pytestmark = pytest.mark.gpu

POLICIES = ['keep', 'remainder', 'tail_batch']


def _oracle_y(boo, xn):
    d = {f: getattr(boo, f) for f in O.BOO_FIELDS}
    d.update(rows=boo.rows, cols=boo.cols)
    return O.boo_matmul(d, xn)


def _product(boo_dev, x, engine):
    y = S.boo_matmul(boo_dev, x, engine=engine)
    torch.cuda.synchronize()
    assert _lib.lib().spmm_tc_status(1) == 0
    return y


def _check(mat, boo, x, engine='tensor_cores'):
    got = _product(boo.to('cuda'), x.cuda(), engine).cpu().numpy()
    xn = x.numpy()
    ref = _oracle_y(boo, xn)
    assert_spmm_close(got, ref, abs_bound(mat.indptr, mat.indices, mat.data, xn), TOL[np.dtype(np.float32)])
    return got


def _labels(n, g, rng, shuffle):
    lab = np.arange(n) // g
    return rng.permutation(lab) if shuffle else lab


@pytest.mark.parametrize('seed', range(32))
def test_tc_seeded_sweep(cuda, seed):
    rng = np.random.default_rng(7000 + seed)
    rows, cols = int(rng.integers(1, 3000)), int(rng.integers(1, 3000))
    mat = sp.random(rows, cols, density=float(rng.uniform(0.002, 0.08)), format='csr',
                    random_state=seed, dtype=np.float64)
    mat.data = rng.standard_normal(mat.nnz)
    mat = mat.astype(np.float32)
    gr, gc = (int(rng.choice([1, 5, 8, 16, 31, 32, 48, 64])) for _ in range(2))
    rl, cl = _labels(rows, gr, rng, seed % 2 == 1), _labels(cols, gc, rng, seed % 4 == 3)
    policy = POLICIES[seed % 3]
    order = ('rowmajor', 'colmajor')[(seed // 3) % 2]
    boo = S.csr_to_boo(mat, row_labels=rl, col_labels=cl, small_block_policy=policy,
                       small_block_threshold=int(rng.integers(0, 6)), nz_order=order)
    k = int(rng.choice([128, 256, 384]))
    batch = int(rng.integers(1, 3))
    x = torch.from_numpy(rng.standard_normal((batch, cols, k)).astype(np.float32))
    y_tc = _check(mat, boo, x, 'tensor_cores')
    y_cc = _check(mat, boo, x, 'cuda_cores')
    y_auto = _product(boo.to('cuda'), x.cuda(), 'auto').cpu().numpy()
    dense = boo.max_nr <= 64 and boo.max_nc <= 64 and boo.compressed_nnz() >= 96 * boo.num_blocks()
    np.testing.assert_array_equal(y_auto, y_tc if dense else y_cc)   # auto's measured crossover


@pytest.mark.parametrize('name,gen,kw,target,k', [
    ('fem3d', workloads.fem3d, dict(n=10), 32, 128),
    ('laplacian2d', workloads.laplacian2d, dict(n=70), 32, 256),
    ('blockdiag64', workloads.blockdiag, dict(n_blocks=24, b=64), 64, 512),
    ('powerlaw', workloads.powerlaw, dict(n=3000), 32, 128),
    ('uniform', workloads.uniform, dict(n=4000), 32, 128),
])
def test_tc_workload_shapes(cuda, name, gen, kw, target, k):
    mat = gen(**kw)
    rows, cols = mat.shape
    boo = S.csr_to_boo(mat, row_labels=np.arange(rows) // target, col_labels=np.arange(cols) // target)
    x = torch.from_numpy(np.random.default_rng(5).standard_normal((cols, k)).astype(np.float32))
    _check(mat, boo, x)


def test_tc_deterministic(cuda):
    mat = workloads.fem3d(n=8)
    boo = S.csr_to_boo(mat, cluster='identity', target_nr=32, target_nc=32).to('cuda')
    x = torch.randn(mat.shape[1], 256, generator=torch.Generator().manual_seed(3)).cuda()
    a = _product(boo, x, 'tensor_cores')
    b = _product(boo, x, 'tensor_cores')
    assert torch.equal(a, b)


def test_tc_wide_dynamic_range(cuda):
    rng = np.random.default_rng(11)
    mat = sp.random(900, 700, density=0.05, format='csr', random_state=4, dtype=np.float64)
    mat.data = rng.choice([-1, 1], mat.nnz) * np.exp(rng.uniform(-20, 20, mat.nnz))
    mat = mat.astype(np.float32)
    boo = S.csr_to_boo(mat, cluster='identity', target_nr=32, target_nc=32)
    x = rng.choice([-1, 1], (700, 128)) * np.exp(rng.uniform(-25, 25, (700, 128)))
    _check(mat, boo, torch.from_numpy(x.astype(np.float32)))


@pytest.mark.parametrize('policy,threshold', [('remainder', 6), ('tail_batch', 6), ('remainder', 1000)])
def test_tc_spills_and_empty_groups(cuda, policy, threshold):
    """Row groups whose blocks all spilled (or that hold no nonzeros at all)
    get only their remainder / tail entries."""
    rng = np.random.default_rng(3)
    dense = rng.standard_normal((640, 512)).astype(np.float32)
    dense[rng.random(dense.shape) > 0.02] = 0
    dense[100:164] = 0                      # two empty row groups
    dense[300:310, :] = 0
    mat = sp.csr_matrix(dense)
    boo = S.csr_to_boo(mat, row_labels=np.arange(640) // 32, col_labels=np.arange(512) // 32,
                       small_block_policy=policy, small_block_threshold=threshold)
    x = torch.from_numpy(rng.standard_normal((2, 512, 128)).astype(np.float32))
    if boo.num_blocks() == 0:
        with pytest.raises(_lib.SpmmError):
            _product(boo.to('cuda'), x.cuda(), 'tensor_cores')
        _check(mat, boo, x, 'auto')
    else:
        _check(mat, boo, x)


def _assert_same_nonfinite(got, ref, bound):
    assert np.array_equal(np.isnan(got), np.isnan(ref))
    assert np.array_equal(np.isposinf(got), np.isposinf(ref))
    assert np.array_equal(np.isneginf(got), np.isneginf(ref))
    fin = np.isfinite(ref)
    assert_spmm_close(np.where(fin, got, 0), np.where(fin, ref, 0), np.where(fin, bound, 0),
                      TOL[np.dtype(np.float32)])


def test_tc_nonfinite_values(cuda):
    """NaN / Inf in A or X propagate exactly as in the reference's CPU path:
    0 * Inf never reaches rows that do not use the value."""
    rng = np.random.default_rng(21)
    mat = sp.random(512, 384, density=0.06, format='csr', random_state=9, dtype=np.float32)
    mat.data[:] = rng.standard_normal(mat.nnz)
    mat.data[[3, 70, 500]] = [np.inf, -np.inf, np.nan]
    boo = S.csr_to_boo(mat, cluster='identity', target_nr=32, target_nc=32)
    x = rng.standard_normal((384, 128)).astype(np.float32)
    x[5, 7] = np.inf
    x[200, :] = -np.inf
    x[301, 64:96] = np.nan
    got = _product(boo.to('cuda'), torch.from_numpy(x).cuda(), 'tensor_cores').cpu().numpy()
    ref = _oracle_y(boo, x)
    with np.errstate(invalid='ignore'):
        bound = abs_bound(mat.indptr, mat.indices, np.nan_to_num(mat.data, posinf=0, neginf=0),
                          np.nan_to_num(x, posinf=0, neginf=0))
    assert np.isnan(ref).any() and np.isinf(ref).any() and np.isfinite(ref).any()
    _assert_same_nonfinite(got, ref, bound)


def test_tc_not_applicable(cuda):
    mat = workloads.laplacian2d(n=20)
    boo32 = S.csr_to_boo(mat, cluster='identity', target_nr=32, target_nc=32)
    x = torch.randn(mat.shape[1], 64).cuda()
    with pytest.raises(_lib.SpmmError):             # K not a multiple of 128
        S.boo_matmul(boo32.to('cuda'), x, engine='tensor_cores')
    y = S.boo_matmul(boo32.to('cuda'), x, engine='auto')     # falls back to CUDA cores
    assert y.shape == (mat.shape[0], 64)
    boo64 = S.csr_to_boo(mat.astype(np.float64), cluster='identity', target_nr=32, target_nc=32)
    with pytest.raises(_lib.SpmmError):             # float64 has no tensor-core path
        S.boo_matmul(boo64.to('cuda'), x.double().repeat(1, 2), engine='tensor_cores')
    big = S.csr_to_boo(mat, row_labels=np.arange(mat.shape[0]) // 100, col_labels=np.arange(mat.shape[1]) // 100)
    with pytest.raises(_lib.SpmmError):             # blocks larger than 64 x 64
        S.boo_matmul(big.to('cuda'), torch.randn(mat.shape[1], 128).cuda(), engine='tensor_cores')
    with pytest.raises(ValueError):
        S.boo_matmul(boo32.to('cuda'), x, engine='tensor')


def test_tc_abi_workspace_required(cuda):
    """Through the C ABI: the tensor-core product's scratch (X gathered by
    column group) comes from the caller -- none or too little gives
    SPMM_EWORKSPACE and launches nothing -- and two calls give the same bits."""
    import ctypes as C
    from spmm_b200._device import stream_handle
    mat = workloads.fem3d(n=8)
    boo = S.csr_to_boo(mat, cluster='identity', target_nr=32, target_nc=32).to('cuda')
    st = boo._dev_struct(boo._gpu_meta)
    x = torch.randn(mat.shape[1], 256, generator=torch.Generator().manual_seed(9)).cuda()
    L = _lib.lib()
    cfg = _lib.launch_cfg('tensor_cores')
    ws_bytes = L.spmm_boo_matmul_workspace_size(C.byref(st), 1, 256, C.byref(cfg))
    assert ws_bytes == boo.num_col_groups() * 32 * 256 * 4 + 256   # panels + range words
    y = torch.empty(mat.shape[0], 256, device='cuda')
    args = (C.byref(st), C.c_void_p(x.data_ptr()), C.c_void_p(y.data_ptr()), 1, 256, C.byref(cfg),
            stream_handle(x.device))
    n0 = L.spmm_product_launches()
    assert L.spmm_boo_matmul(*args) == _lib.SPMM_EWORKSPACE
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device='cuda')
    cfg.workspace, cfg.workspace_bytes = ws.data_ptr(), ws_bytes - 16
    assert L.spmm_boo_matmul(*args) == _lib.SPMM_EWORKSPACE
    assert L.spmm_product_launches() == n0
    cfg.workspace_bytes = ws_bytes
    out = []
    for _ in range(2):
        assert L.spmm_boo_matmul(*args) == 0
        torch.cuda.synchronize()
        out.append(y.clone())
    assert L.spmm_tc_status(1) == 0
    assert torch.equal(out[0], out[1])
    cc = _lib.launch_cfg('cuda_cores')
    assert L.spmm_boo_matmul_workspace_size(C.byref(st), 1, 256, C.byref(cc)) == 0


def test_tc_status_per_call(cuda):
    """Two products in flight on two streams report into their own status
    words.  One runs with SPMM_CFG_EXPIRE_FIRST_WAIT: each worker's first wait
    is on a barrier nothing arrives on, bounded to 50 us, so it expires and
    the launch stops early (SPMM_ETIMEOUT); the other completes (0, Y right).
    The timeout path drains the MMAs it issued and releases tensor memory:
    the context stays usable and later products are exact."""
    import ctypes as C
    mat = workloads.fem3d(n=12)
    boo = S.csr_to_boo(mat, cluster='identity', target_nr=32, target_nc=32)
    dev = boo.to('cuda')
    st = dev._dev_struct(dev._gpu_meta)
    x = torch.randn(mat.shape[1], 256, generator=torch.Generator().manual_seed(2))
    xd = x.cuda()
    L = _lib.lib()
    words = torch.full((2, 64), 7, dtype=torch.int32, device='cuda')   # stale values: the call clears its own
    ys = [torch.empty(mat.shape[0], 256, device='cuda') for _ in range(2)]
    cfgs, keep = [], []
    for k, flags in enumerate((_lib.SPMM_CFG_EXPIRE_FIRST_WAIT, 0)):
        cfg = _lib.launch_cfg('tensor_cores', status=words[k].data_ptr(), wait_us=50, flags=flags)
        n = L.spmm_boo_matmul_workspace_size(C.byref(st), 1, 256, C.byref(cfg))
        ws = torch.empty(n, dtype=torch.uint8, device='cuda')
        cfg.workspace, cfg.workspace_bytes = ws.data_ptr(), n
        cfgs.append(cfg)
        keep.append(ws)
    streams = [torch.cuda.Stream(), torch.cuda.Stream()]
    torch.cuda.synchronize()
    for cfg, y, stream in zip(cfgs, ys, streams):
        rc = L.spmm_boo_matmul(C.byref(st), C.c_void_p(xd.data_ptr()), C.c_void_p(y.data_ptr()), 1, 256,
                               C.byref(cfg), C.c_void_p(stream.cuda_stream))
        assert rc == 0
    torch.cuda.synchronize()
    assert int(words[0, 0]) == _lib.SPMM_ETIMEOUT
    assert int(words[1, 0]) == 0
    ref = _oracle_y(boo, x.numpy())
    bound = abs_bound(mat.indptr, mat.indices, mat.data, x.numpy())
    assert_spmm_close(ys[1].cpu().numpy(), ref, bound, TOL[np.dtype(np.float32)])
    assert L.spmm_tc_status(1) == 0      # calls with a status word leave the shared one alone
    bad = _lib.launch_cfg('tensor_cores', flags=_lib.SPMM_CFG_EXPIRE_FIRST_WAIT)   # needs wait_us > 0
    assert L.spmm_boo_matmul(C.byref(st), C.c_void_p(xd.data_ptr()), C.c_void_p(ys[0].data_ptr()), 1, 256,
                             C.byref(bad), None) == _lib.SPMM_EINVAL
    again = S.boo_matmul(dev, xd, engine='tensor_cores')
    assert S.product_status(again) == 0
    assert_spmm_close(S.check_product(again).cpu().numpy(), ref, bound, TOL[np.dtype(np.float32)])


@pytest.mark.parametrize('g,n_sparse,rem_rows', [
    (32, 31, 'none'), (32, 32, 'none'), (32, 33, 'none'), (32, 20, 'all'), (32, 40, 'even'),
    (64, 1, 'all'), (64, 97, 'even'), (64, 130, 'all'),
])
def test_tc_cuda_core_segment_lists(cuda, g, n_sparse, rem_rows):
    """Row groups whose CUDA-core part spans many segments -- sparse blocks and
    rows with remainder entries, empty rows in between -- so the segment list
    fills in the middle of a window of candidates and resumes there, and
    lists several times per row group."""
    rng = np.random.default_rng(g * 1000 + n_sparse)
    n_groups = 3
    rows, ncg = g * n_groups, 1 + n_sparse + g
    cols = g * ncg
    r, c = [], []
    for grp in range(n_groups):
        r0 = grp * g
        r += list(r0 + rng.integers(0, g, 3 * g))                 # one tensor-core block (col group 0)
        c += list(rng.integers(0, g, 3 * g))
        for s in range(1, 1 + n_sparse):                          # kept blocks of 6-12 nonzeros
            k = int(rng.integers(6, 13))
            r += list(r0 + rng.integers(0, g, k))
            c += list(s * g + rng.integers(0, g, k))
        for q in range(g):                                        # one entry in a block of its own:
            if rem_rows == 'all' or (rem_rows == 'even' and q % 2 == 0):   # spilled to the remainder
                r.append(r0 + q)
                c.append((1 + n_sparse + q) * g + int(rng.integers(0, g)))
    vals = rng.standard_normal(len(r)).astype(np.float32)
    mat = sp.csr_matrix((vals, (np.array(r), np.array(c))), shape=(rows, cols), dtype=np.float32)
    mat.sum_duplicates()
    mat.sort_indices()
    boo = S.csr_to_boo(mat, row_labels=np.arange(rows) // g, col_labels=np.arange(cols) // g)
    assert boo.num_blocks() == n_groups * (1 + n_sparse)
    assert boo.remainder_nnz() == n_groups * {'none': 0, 'all': g, 'even': g // 2}[rem_rows]
    x = torch.from_numpy(rng.standard_normal((cols, 128)).astype(np.float32))
    _check(mat, boo, x, 'tensor_cores')
    _check(mat, boo, x, 'cuda_cores')


@pytest.mark.parametrize('policy', ['remainder', 'tail_batch', 'keep'])
def test_tc_row_groups_larger_than_blocks(cuda, policy):
    """max_nr counts only the row groups of kept blocks, so a row group larger
    than the tensor-core tile (100 rows here, tile 32) passes the engine's
    check when its blocks all spilled (remainder / tail) or when it holds no
    nonzeros at all (keep): all of its rows must still be written."""
    rng = np.random.default_rng(41)
    sizes = [32, 32, 100, 32, 100, 32]                 # groups 2 and 4 have 100 rows
    rl = np.repeat(np.arange(len(sizes)), sizes)
    rows, cols = len(rl), 256
    dense = np.zeros((rows, cols), np.float32)
    starts = np.concatenate([[0], np.cumsum(sizes)])
    for g in (0, 1, 3, 5):                             # dense blocks in the 32-row groups
        sl = slice(starts[g], starts[g + 1])
        m = rng.random((sizes[g], cols)) < 0.3
        dense[sl][m] = rng.standard_normal(int(m.sum()))
    if policy != 'keep':                               # group 2: one entry per block, spilled,
        for k, q in enumerate((5, 33, 40, 64, 70, 90, 99)):   # rows past the tile's 32 included
            dense[starts[2] + q, 32 * k + (q % 32)] = rng.standard_normal()
    mat = sp.csr_matrix(dense)
    cl = np.arange(cols) // 32
    boo = S.csr_to_boo(mat, row_labels=rl, col_labels=cl, small_block_policy=policy,
                       small_block_threshold=4)
    assert boo.max_nr == 32
    x = torch.from_numpy(rng.standard_normal((cols, 128)).astype(np.float32))
    import ctypes as C
    from spmm_b200._device import stream_handle
    dev = boo.to('cuda')
    st = dev._dev_struct(dev._gpu_meta)
    xd = x.cuda()
    y = torch.full((rows, 128), float('nan'), device='cuda')   # stale contents must not survive
    L = _lib.lib()
    cfg = _lib.launch_cfg('tensor_cores')
    ws_bytes = L.spmm_boo_matmul_workspace_size(C.byref(st), 1, 128, C.byref(cfg))
    ws = torch.empty(max(ws_bytes, 16), dtype=torch.uint8, device='cuda')
    cfg.workspace, cfg.workspace_bytes = ws.data_ptr(), ws_bytes
    rc = L.spmm_boo_matmul(C.byref(st), C.c_void_p(xd.data_ptr()), C.c_void_p(y.data_ptr()), 1, 128,
                           C.byref(cfg), stream_handle(xd.device))
    assert rc == 0
    torch.cuda.synchronize()
    assert L.spmm_tc_status(1) == 0
    got = y.cpu().numpy()
    assert np.isfinite(got).all()
    ref = _oracle_y(boo, x.numpy())
    assert_spmm_close(got, ref, abs_bound(mat.indptr, mat.indices, mat.data, x.numpy()), TOL[np.dtype(np.float32)])


@pytest.mark.parametrize('name,gen,kw,target,k', [
    ('fem3d', workloads.fem3d, dict(n=10), 32, 128),
    ('blockdiag64', workloads.blockdiag, dict(n_blocks=24, b=64), 64, 512),
])
def test_tf32_engine_within_tf32_tolerance(cuda, name, gen, kw, target, k):
    """The opt-in one-term engine ('tensor_cores_tf32'): within 2e-3 (|A||X|)
    of the oracle -- tf32's accuracy, stated apart from the float32 bar --
    and deterministic; the three-term engine stays within 1e-5."""
    mat = gen(**kw)
    rows, cols = mat.shape
    boo = S.csr_to_boo(mat, row_labels=np.arange(rows) // target, col_labels=np.arange(cols) // target)
    x = torch.from_numpy(np.random.default_rng(8).standard_normal((cols, k)).astype(np.float32))
    dev, xd = boo.to('cuda'), x.cuda()
    y1 = _product(dev, xd, 'tensor_cores_tf32')
    assert torch.equal(y1, _product(dev, xd, 'tensor_cores_tf32'))
    ref = _oracle_y(boo, x.numpy())
    bound = abs_bound(mat.indptr, mat.indices, mat.data, x.numpy())
    assert_spmm_close(y1.cpu().numpy(), ref, bound, 2e-3)
    err = np.abs(y1.cpu().numpy().astype(np.float64) - ref).max()
    assert err > 0                        # a single tf32 term is not float32-exact
    _check(mat, boo, x, 'tensor_cores')
