"""spmm_boo_build_noalloc: the BOO build for callers that cannot allocate device
memory (a framework pool that owns all device memory, a loop where an
allocation may block or fail, a plugin host that forbids heap growth).

Its scratch is a fixed 32 MiB array inside the library.  Called through the C
ABI, its output must equal that of the two-phase entry points
(spmm_boo_build_analyze / _emit with a caller workspace) array for array, on
two calls in a row -- the second call finds the first call's leftovers in the
shared array.  This file is collected last so that a run stopping at the first
failure has already run every other test; it also passes alone in a fresh
process."""

import ctypes as C

import numpy as np
import pytest
import scipy.sparse as sp
import torch

import spmm_b200 as S
from spmm_b200 import _lib
from spmm_b200._device import ptr, stream_handle, to_device

pytestmark = pytest.mark.gpu

FIELDS = _lib.BOO_PTR_FIELDS


def _noalloc_build(mat, rl, cl, policy, threshold, order):
    """Calls spmm_boo_build_noalloc with worst-case caller-allocated outputs."""
    dev = torch.device('cuda', torch.cuda.current_device())
    rows, cols = mat.shape
    nnz = mat.nnz
    idt = np.int32 if mat.indptr.dtype == np.int32 and mat.indices.dtype == np.int32 else np.int64
    d_ip = to_device(mat.indptr, dev, idt)
    d_ix = to_device(mat.indices, dev, idt)
    d_v = to_device(mat.data, dev)
    d_rl = to_device(rl, dev, np.int32)
    d_cl = to_device(cl, dev, np.int32)
    A = _lib.CsrDev()
    A.rows, A.cols, A.nnz = rows, cols, nnz
    A.indptr, A.indices, A.values = ptr(d_ip), ptr(d_ix), ptr(d_v)
    A.index_type = _lib.I32 if idt == np.int32 else _lib.I64
    A.scalar_type = _lib.F32 if mat.dtype == np.float32 else _lib.F64
    vdt = torch.float32 if mat.dtype == np.float32 else torch.float64
    cap = {'row_grp_ptr': rows + 1, 'row_ids': rows, 'col_grp_ptr': cols + 1, 'col_ids': cols,
           'blk_nz_ptr': nnz + 1, 'rem_indptr': rows + 1}
    dt = {'blk_shift': torch.uint8, 'nz_idx': torch.int16, 'nz_val': vdt, 'rem_vals': vdt,
          'tail_val': vdt}
    bufs = {f: torch.full((max(cap.get(f, nnz), 1),), -7, dtype=dt.get(f, torch.int32), device=dev)
            for f in FIELDS}
    out = _lib.BooDev()
    for f in FIELDS:
        setattr(out, f, bufs[f].data_ptr())
    rc = _lib.lib().spmm_boo_build_noalloc(C.byref(A), ptr(d_rl), ptr(d_cl), policy, threshold,
                                            order, C.byref(out), stream_handle(dev))
    torch.cuda.synchronize(dev)
    return rc, out, bufs


def _sizes(out):
    n = {k: int(getattr(out, k)) for k in _lib.BOO_SIZE_FIELDS}
    return {'row_grp_ptr': n['n_rg'] + 1, 'row_ids': n['rows'], 'col_grp_ptr': n['n_cg'] + 1,
            'col_ids': n['cols'], 'blk_row_grp': n['nb'], 'blk_col_grp': n['nb'],
            'blk_nz_ptr': n['nb'] + 1, 'blk_shift': n['nb'], 'nz_idx': n['nnz_c'],
            'nz_val': n['nnz_c'], 'rem_indptr': n['rows'] + 1, 'rem_col_ind': n['rem_nnz'],
            'rem_vals': n['rem_nnz'], 'tail_row': n['tail_nnz'], 'tail_col': n['tail_nnz'],
            'tail_val': n['tail_nnz']}


def _problem(seed, rows, cols, density, dtype):
    rng = np.random.default_rng(seed)
    mat = sp.random(rows, cols, density=density, format='csr', random_state=seed, dtype=np.float64)
    mat.data = rng.standard_normal(mat.nnz)
    mat = mat.astype(dtype)
    rl = rng.integers(0, max(1, rows // 24), size=rows).astype(np.int32)
    cl = rng.integers(0, max(1, cols // 24), size=cols).astype(np.int32)
    return mat, rl, cl


CASES = [  # two calls in a row: different problems, policies and orders
    (11, 2000, 1500, 0.02, np.float32, 'remainder', 4, 'rowmajor'),
    (12, 900, 2100, 0.05, np.float64, 'tail_batch', 6, 'colmajor'),
]


def test_noalloc_build_matches_workspace_build():
    if not torch.cuda.is_available():
        pytest.fail('CUDA device required for gpu-marked tests')
    codes = {'keep': 0, 'remainder': 2, 'tail_batch': 3}
    orders = {'rowmajor': 0, 'colmajor': 1}
    for seed, rows, cols, dens, dtype, policy, thr, order in CASES:
        mat, rl, cl = _problem(seed, rows, cols, dens, dtype)
        # existing entry points (analyze + emit with a caller workspace)
        ref = S.csr_to_boo(mat, row_labels=rl, col_labels=cl, small_block_policy=policy,
                           small_block_threshold=thr, nz_order=order)
        rc, out, bufs = _noalloc_build(mat, rl, cl, codes[policy], thr, orders[order])
        assert rc == _lib.SPMM_OK, _lib.status_string(rc)
        assert int(out.nb) == ref.num_blocks() and int(out.nnz_c) == ref.compressed_nnz()
        assert int(out.rem_nnz) == ref.remainder_nnz() and int(out.tail_nnz) == ref.tail_nnz()
        assert (int(out.max_nr), int(out.max_nc), int(out.max_nnz_blk)) == \
            (ref.max_nr, ref.max_nc, ref.max_nnz_blk)
        sizes = _sizes(out)
        for f in FIELDS:
            got = bufs[f][:sizes[f]].cpu().numpy()
            want = ref._dev.__dict__[f].cpu().numpy()
            assert got.shape == want.shape and np.array_equal(got, want), f


def test_noalloc_rejects_oversized_problem_without_device_work():
    if not torch.cuda.is_available():
        pytest.fail('CUDA device required for gpu-marked tests')
    A = _lib.CsrDev()
    A.rows, A.cols, A.nnz = 1 << 20, 1 << 20, 1 << 22      # needs far more than 32 MiB
    A.indptr, A.indices, A.values = 1, 1, 1                # never dereferenced
    out = _lib.BooDev()
    rc = _lib.lib().spmm_boo_build_noalloc(C.byref(A), 1, 1, 2, 4, 0, C.byref(out), None)
    assert rc == _lib.SPMM_ESCRATCH
    assert 'scratch' in _lib.status_string(rc)


def _nnz_limit(rows, cols):
    """Largest nnz whose builder workspace fits the 32 MiB scratch."""
    L = _lib.lib()
    lo, hi = 0, rows * cols
    while lo < hi:
        mid = (lo + hi + 1) // 2
        if L.spmm_boo_build_workspace_size(rows, cols, mid) <= 32 << 20:
            lo = mid
        else:
            hi = mid - 1
    return lo


def _exact_nnz(seed, rows, cols, nnz):
    rng = np.random.default_rng(seed)
    keys = np.sort(rng.choice(rows * cols, nnz, replace=False))
    r, c = keys // cols, keys % cols
    indptr = np.zeros(rows + 1, dtype=np.int64)
    np.cumsum(np.bincount(r, minlength=rows), out=indptr[1:])
    mat = sp.csr_matrix((rng.standard_normal(nnz).astype(np.float32), c, indptr), shape=(rows, cols))
    return mat, rng.integers(0, rows // 32, rows).astype(np.int32), (np.arange(cols) // 32).astype(np.int32)


def _assert_same_as_workspace_build(mat, rl, cl, rc, out, bufs):
    assert rc == _lib.SPMM_OK, _lib.status_string(rc)
    ref = S.csr_to_boo(mat, row_labels=rl, col_labels=cl)
    assert int(out.nb) == ref.num_blocks() and int(out.rem_nnz) == ref.remainder_nnz()
    sizes = _sizes(out)
    for f in FIELDS:
        got = bufs[f][:sizes[f]].cpu().numpy()
        want = ref._dev.__dict__[f].cpu().numpy()
        assert got.shape == want.shape and np.array_equal(got, want), f


def test_noalloc_at_the_scratch_limit():
    """The largest problem whose workspace fits 32 MiB builds correctly; one
    more nonzero is rejected with SPMM_ESCRATCH before any device work."""
    if not torch.cuda.is_available():
        pytest.fail('CUDA device required for gpu-marked tests')
    L = _lib.lib()
    rows = cols = 40000
    nmax = _nnz_limit(rows, cols)
    assert L.spmm_boo_build_workspace_size(rows, cols, nmax) <= 32 << 20 < \
        L.spmm_boo_build_workspace_size(rows, cols, nmax + 1)
    mat, rl, cl = _exact_nnz(5, rows, cols, nmax)
    _assert_same_as_workspace_build(mat, rl, cl, *_noalloc_build(mat, rl, cl, 2, 4, 0))
    over, rl2, cl2 = _exact_nnz(6, rows, cols, nmax + 1)
    rc, _, _ = _noalloc_build(over, rl2, cl2, 2, 4, 0)
    assert rc == _lib.SPMM_ESCRATCH


def test_noalloc_after_a_failed_call():
    """A call that fails inside the build (a row label out of range) leaves
    the shared scratch in a state the next valid call does not depend on."""
    if not torch.cuda.is_available():
        pytest.fail('CUDA device required for gpu-marked tests')
    mat, rl, cl = _problem(21, 1200, 900, 0.03, np.float32)
    bad = rl.copy()
    bad[17] = mat.shape[0]                      # labels must lie in [0, rows)
    rc, _, _ = _noalloc_build(mat, bad, cl, 2, 4, 0)
    assert rc == _lib.SPMM_ELABEL
    _assert_same_as_workspace_build(mat, rl, cl, *_noalloc_build(mat, rl, cl, 2, 4, 0))
