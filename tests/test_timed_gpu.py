"""Paired timing harnesses (BOOTimedSpMM, PBRTimedSpMM, DirectSpMM) and the
on-disk formats on the GPU: the harnesses produce the public products' Y,
time with CUDA events, refuse foreign streams; a reloaded format multiplies
exactly like the original."""

import numpy as np
import pytest
import scipy.sparse as sp
import torch

import spmm_b200 as S
from spmm_b200 import workloads

pytestmark = pytest.mark.gpu


def _meta_args(boo):
    m = boo._gpu_meta
    return (boo.rows, boo.cols, boo.max_nr, boo.max_nc, boo.max_nnz_blk, m.row_grp_ptr, m.row_ids, m.col_grp_ptr,
            m.col_ids, m.blk_row_grp, m.blk_col_grp, m.blk_nz_ptr, m.blk_shift, m.nz_idx, m.nz_val, m.rem_indptr,
            m.rem_col_ind, m.rem_vals, m.tail_row, m.tail_col, m.tail_val)


@pytest.mark.parametrize('gen,kw,k', [(workloads.fem3d, dict(n=8), 128), (workloads.powerlaw, dict(n=3000), 64)])
def test_boo_timed_matches_boo_matmul(cuda, gen, kw, k):
    mat = gen(**kw)
    boo = S.csr_to_boo(mat, cluster='identity', target_nr=32, target_nc=32,
                       small_block_policy='tail_batch').to('cuda')
    x = torch.randn(mat.shape[1], k, generator=torch.Generator().manual_seed(1)).cuda()
    timed = S.BOOTimedSpMM(*_meta_args(boo), x)
    y = timed.run()
    assert torch.equal(y, S.boo_matmul(boo, x))
    ms = timed.timed_run()
    assert ms > 0 and torch.equal(timed.output, y)
    assert timed.info()['row_seg'] is True
    side = torch.cuda.Stream()
    with torch.cuda.stream(side):
        with pytest.raises(RuntimeError, match='construction stream'):
            timed.run()
    with pytest.raises(RuntimeError):
        S.BOOTimedSpMM(*_meta_args(boo), x, threads=100)
    diag = S.BOOTimedSpMM(*_meta_args(boo), x, diagnostic_raw_store=True)
    assert diag.timed_run() > 0
    with pytest.raises(RuntimeError, match='not meaningful'):
        diag.output


def test_pbr_timed_matches_pbr_matmul(cuda):
    mat = workloads.uniform(n=20000)
    pbr = S.csr_to_pbr(mat, 8, 8, 2).to('cuda')
    m = pbr._gpu_meta
    x = torch.randn(2, mat.shape[1], 64, generator=torch.Generator().manual_seed(2)).cuda()
    timed = S.PBRTimedSpMM(pbr.cols, pbr.rows, pbr.block_rows, pbr.block_cols, m.codes, m.coords, m.offsets,
                           m.data, m.rem_indptr, m.rem_col_ind, m.rem_vals, x)
    assert torch.equal(timed.run(), S.pbr_matmul(pbr, x))
    assert timed.timed_run() > 0
    with pytest.raises(RuntimeError):
        S.PBRTimedSpMM(pbr.cols, pbr.rows, 8, 8, m.codes, m.coords, m.offsets, m.data, m.rem_indptr,
                       m.rem_col_ind, m.rem_vals, x, kernel='nope')


@pytest.mark.parametrize('alg', ['DEFAULT', 'CSR_ALG1', 'CSR_ALG2', 'CSR_ALG3'])
def test_direct_spmm(cuda, alg):
    mat = sp.random(3000, 2000, density=0.01, format='csr', random_state=3, dtype=np.float32)
    x = torch.randn(2000, 96, generator=torch.Generator().manual_seed(4)).cuda()
    crow = torch.from_numpy(mat.indptr.astype(np.int32)).cuda()
    col = torch.from_numpy(mat.indices.astype(np.int32)).cuda()
    val = torch.from_numpy(mat.data).cuda()
    d = S.DirectSpMM(crow, col, val, x, alg)
    if not d.supported:
        pytest.skip(d.reason)
    y = d.run().cpu().numpy()
    ref = mat.astype(np.float64) @ x.cpu().numpy().astype(np.float64)
    np.testing.assert_allclose(y, ref, rtol=1e-4, atol=1e-4)
    assert d.timed_run() > 0
    with pytest.raises(RuntimeError):
        S.DirectSpMM(crow, col, val, x, 'ALG9')


def test_saved_formats_multiply_like_the_originals(cuda, tmp_path):
    mat = workloads.fem3d(n=6)
    boo = S.csr_to_boo(mat, cluster='hem', target_nr=32, target_nc=32)
    pbr = S.csr_to_pbr(mat, 8, 8, 4)
    S.save_boo(tmp_path / 'a.npz', boo)
    S.save_pbr(tmp_path / 'b.npz', pbr)
    boo2, pbr2 = S.load_boo(tmp_path / 'a.npz'), S.load_pbr(tmp_path / 'b.npz')
    x = torch.randn(mat.shape[1], 128, generator=torch.Generator().manual_seed(5)).cuda()
    assert torch.equal(S.boo_matmul(boo2.to('cuda'), x), S.boo_matmul(boo.to('cuda'), x))
    assert torch.equal(S.pbr_matmul(pbr2.to('cuda'), x), S.pbr_matmul(pbr.to('cuda'), x))
    assert (S.boo_to_csr(boo2) != S.boo_to_csr(boo)).nnz == 0
