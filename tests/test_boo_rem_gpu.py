"""Remainder-major BOO products (the load-balanced remainder kernels) against
the oracle: skewed rows (including rows longer than the 1,024-entry long-row
threshold), fp32 and fp64, vector and scalar K, batched X, tail entries."""

import numpy as np
import pytest
import scipy.sparse as sp
import torch

import spmm_b200 as S
from oracle import oracle as O
from tests.conftest import TOL, abs_bound, assert_spmm_close

pytestmark = pytest.mark.gpu


def _skewed(rows, cols, seed, dtype, long_rows=(0, 7, 300), long_len=3000):
    rng = np.random.default_rng(seed)
    lens = np.minimum(rng.zipf(2.0, rows), 200)
    for r in long_rows:
        if r < rows:
            lens[r] = min(long_len, cols)
    indptr = np.concatenate([[0], np.cumsum(lens)]).astype(np.int64)
    indices = np.concatenate([np.sort(rng.choice(cols, n, replace=False)) for n in lens]).astype(np.int64)
    data = rng.standard_normal(indptr[-1]).astype(dtype)
    return sp.csr_matrix((data, indices, indptr), shape=(rows, cols))


def _check(mat, boo, x, slabs=(0,)):
    d = {f: getattr(boo, f) for f in O.BOO_FIELDS}
    d.update(rows=boo.rows, cols=boo.cols)
    xn = x.numpy()
    ref = O.boo_matmul(d, xn)
    bound = abs_bound(mat.indptr, mat.indices, mat.data, xn)
    dev, xd = boo.to('cuda'), x.cuda()
    for slab in slabs:
        got = S.boo_matmul(dev, xd, slab_features=slab)
        assert_spmm_close(got.cpu().numpy(), ref, bound, TOL[np.dtype(mat.dtype)])
        assert torch.equal(got, S.boo_matmul(dev, xd, slab_features=slab))   # deterministic


# slab_features: automatic (0: the nnz-flat chunks, or half a warp per row
# for a short remainder at K <= 16 vectors), the nnz-flat chunks (> 0) and
# the register path (< 0)
SLABS = {np.float32: (0, -1, 16), np.float64: (0, -1, 8)}


@pytest.mark.parametrize('dtype', [np.float32, np.float64])
@pytest.mark.parametrize('k', [1, 7, 32, 64, 128, 256, 300])
def test_remainder_major_skewed_rows(cuda, dtype, k):
    mat = _skewed(1200, 5000, 11 + k, dtype)
    boo = S.csr_to_boo(mat, cluster="identity", target_nr=32, target_nc=32, small_block_threshold=64)
    assert 2 * boo.remainder_nnz() >= boo.total_nnz       # the remainder-major path
    assert np.diff(boo.rem_indptr).max() > 1024           # long rows present
    tdt = torch.float32 if dtype == np.float32 else torch.float64
    x = torch.from_numpy(np.random.default_rng(k).standard_normal((2, 5000, k))).to(tdt)
    _check(mat, boo, x, SLABS[dtype])


@pytest.mark.parametrize('policy', ['remainder', 'tail_batch'])
def test_remainder_major_with_blocks_and_tail(cuda, policy):
    rng = np.random.default_rng(5)
    skew = _skewed(640, 2048, 3, np.float32, long_rows=(1, 600), long_len=1500)
    dense = sp.random(640, 2048, density=0.002, format='csr', random_state=1, dtype=np.float32)
    dense[:64, :64] = rng.standard_normal((64, 64)).astype(np.float32)   # a few kept blocks
    mat = (skew + dense).tocsr()
    mat.sort_indices()
    boo = S.csr_to_boo(mat, cluster='identity', target_nr=32, target_nc=32,
                       small_block_policy=policy, small_block_threshold=8)
    assert boo.num_blocks() > 0
    x = torch.from_numpy(rng.standard_normal((2048, 96)).astype(np.float32))
    _check(mat, boo, x, SLABS[np.float32])


def test_remainder_major_deterministic(cuda):
    mat = _skewed(900, 3000, 8, np.float32)
    boo = S.csr_to_boo(mat, cluster='identity', target_nr=32, target_nc=32).to('cuda')
    x = torch.randn(3000, 256, generator=torch.Generator().manual_seed(0)).cuda()
    assert torch.equal(S.boo_matmul(boo, x), S.boo_matmul(boo, x))


def test_product_launch_counter(cuda):
    """spmm_product_launches counts the kernels each product launches: four
    for a remainder-major BOO matrix (nnz-flat plan, chunks, fix-up, block
    kernel; three on the register path: tiles, long rows, block kernel; three
    for its short remainder at K = 64 by default: half a warp per row, long
    rows, block kernel), two for the tensor-core product (gather pass +
    worker kernel), one for the CUDA-core block kernel."""
    from spmm_b200 import _lib, workloads
    L = _lib.lib()
    mat = _skewed(1200, 5000, 2, np.float32)
    rem = S.csr_to_boo(mat, cluster='identity', target_nr=32, target_nc=32, small_block_threshold=64).to('cuda')
    fem = workloads.fem3d(n=6)
    blk = S.csr_to_boo(fem, cluster='identity', target_nr=32, target_nc=32).to('cuda')
    xr = torch.randn(5000, 128, device='cuda')
    xn = torch.randn(5000, 64, device='cuda')
    xb = torch.randn(fem.shape[1], 128, device='cuda')
    cases = [(rem, xr, dict(), 4), (rem, xr, dict(slab_features=-1), 3),
             (rem, xn, dict(), 3), (rem, xn, dict(slab_features=1), 4),
             (blk, xb, dict(engine='tensor_cores'), 2), (blk, xb, dict(engine='cuda_cores'), 1)]
    for boo, x, kw, want in cases:
        n0 = L.spmm_product_launches()
        S.boo_matmul(boo, x, **kw)
        assert L.spmm_product_launches() - n0 == want, kw
    torch.cuda.synchronize()


def test_remainder_flat_chunk_boundaries(cuda):
    """nnz-flat chunks cut rows anywhere: rows spanning many chunks, rows
    ending exactly on a chunk boundary, runs of empty rows inside a chunk and
    a window of more than 32 rows inside one chunk."""
    rng = np.random.default_rng(17)
    lens = rng.integers(0, 4, 3000)
    lens[100] = 9000                  # spans many chunks
    lens[200:260] = 0                 # empty rows
    lens[500] = 256 - int(lens[:500].sum()) % 256 + 256   # ends on a multiple of 256
    indptr = np.concatenate([[0], np.cumsum(lens)]).astype(np.int64)
    cols = 12000
    indices = np.concatenate([np.sort(rng.choice(cols, n, replace=False)) for n in lens]).astype(np.int64)
    data = rng.standard_normal(indptr[-1]).astype(np.float32)
    mat = sp.csr_matrix((data, indices, indptr), shape=(3000, cols))
    boo = S.csr_to_boo(mat, cluster='identity', target_nr=32, target_nc=32, small_block_threshold=64)
    assert 2 * boo.remainder_nnz() >= boo.total_nnz
    for k in (4, 96, 260):
        x = torch.from_numpy(rng.standard_normal((2, cols, k)).astype(np.float32))
        _check(mat, boo, x, (0, -1))


def test_remainder_flat_abi_workspace_required(cuda):
    """Through the C ABI: the nnz-flat remainder runs on the caller's scratch
    and the library allocates none -- without it the call returns
    SPMM_EWORKSPACE; the register path (slab_features < 0) needs none and gives
    results within tolerance of the nnz-flat path."""
    import ctypes as C
    from spmm_b200 import _lib
    from spmm_b200._device import stream_handle
    mat = _skewed(1500, 4000, 5, np.float32)
    boo = S.csr_to_boo(mat, cluster='identity', target_nr=32, target_nc=32, small_block_threshold=64).to('cuda')
    st = boo._dev_struct(boo._gpu_meta)
    x = torch.randn(2, 4000, 192, generator=torch.Generator().manual_seed(4)).cuda()
    L = _lib.lib()
    out = []
    for slab in (0, -1):
        cfg = _lib.launch_cfg('auto', slab_features=slab)
        ws_bytes = L.spmm_boo_matmul_workspace_size(C.byref(st), 2, 192, C.byref(cfg))
        assert (ws_bytes > 0) == (slab == 0)
        y = torch.empty(2, 1500, 192, device='cuda')
        args = (C.byref(st), C.c_void_p(x.data_ptr()), C.c_void_p(y.data_ptr()), 2, 192, C.byref(cfg),
                stream_handle(x.device))
        if ws_bytes:
            assert L.spmm_boo_matmul(*args) == _lib.SPMM_EWORKSPACE
            ws = torch.empty(ws_bytes, dtype=torch.uint8, device='cuda')
            cfg.workspace, cfg.workspace_bytes = ws.data_ptr(), ws_bytes - 1   # too short
            assert L.spmm_boo_matmul(*args) == _lib.SPMM_EWORKSPACE
            cfg.workspace_bytes = ws_bytes
        assert L.spmm_boo_matmul(*args) == 0
        torch.cuda.synchronize()
        out.append(y)
    xn = x.cpu().numpy()
    bound = abs_bound(mat.indptr, mat.indices, mat.data, xn)
    assert_spmm_close(out[0].cpu().numpy(), out[1].cpu().numpy(), bound, 2 * TOL[np.dtype(np.float32)])
