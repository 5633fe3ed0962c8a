"""BOO product plans (spmm_boo_plan_build): per-matrix tables the product
reads instead of recomputing them -- each row group's first block, and for
remainder-major matrices with scattered blocks a row-ordered copy of every
entry.  Products with and without a plan agree (bit for bit where the plan
only replaces a search; within the float tolerance where the row-ordered
pass sums a row's entries in column order) and match the oracle."""

import ctypes as C

import numpy as np
import pytest
import scipy.sparse as sp
import torch

import spmm_b200 as S
from oracle import oracle as O
from spmm_b200 import _lib, workloads
from spmm_b200._device import stream_handle
from tests.conftest import TOL, abs_bound, assert_spmm_close

pytestmark = pytest.mark.gpu


def _product(dev, x, engine='auto', with_plan=True):
    L = _lib.lib()
    st = dev._dev_struct(dev._gpu_meta)
    plan = S.boo.product_plan(dev, dev._gpu_meta) if with_plan else None
    cfg = _lib.launch_cfg(engine, plan=plan.data_ptr() if plan is not None else 0)
    n = L.spmm_boo_matmul_workspace_size(C.byref(st), x.shape[0] if x.dim() == 3 else 1, x.shape[-1],
                                         C.byref(cfg))
    ws = torch.empty(max(n, 16), dtype=torch.uint8, device='cuda')
    if n:
        cfg.workspace, cfg.workspace_bytes = ws.data_ptr(), n
    batch = x.shape[0] if x.dim() == 3 else 1
    y = torch.empty((batch, dev.rows, x.shape[-1]), device='cuda', dtype=x.dtype)
    rc = L.spmm_boo_matmul(C.byref(st), C.c_void_p(x.data_ptr()), C.c_void_p(y.data_ptr()), batch, x.shape[-1],
                           C.byref(cfg), stream_handle(x.device))
    assert rc == 0, _lib.status_string(rc)
    torch.cuda.synchronize()
    return y.squeeze(0) if x.dim() == 2 else y


def _plan_size(s, f32=True):
    """The plan layout (plan.cuh): group table; packing arrays for float32
    matrices with groups up to 64 x 64; the row-ordered copy when chosen."""
    al = lambda v: (v + 255) // 256 * 256          # noqa: E731
    n = al(4 * (s['n_rg'] + 1))
    if f32 and s['nb'] > 0 and s['max_nr'] <= 64 and s['max_nc'] <= 64:
        n += al(s['nb']) + al(4 * (s['n_rg'] + 1)) + al(8 * s['nb']) + al(4)   # + identity-column flag
    entries = s['nnz_c'] + s['rem_nnz'] + s['tail_nnz']
    rem_major = s['rem_nnz'] > 0 and 2 * s['rem_nnz'] >= s['total_nnz']
    short_rows = not rem_major and 0 < entries <= 16 * s['rows']
    if (rem_major and 64 * (s['nnz_c'] + s['tail_nnz']) >= entries) or short_rows:
        n += al(4 * (s['rows'] + 1)) + al(4 * entries) + al((4 if f32 else 8) * entries)
    if short_rows:
        n += al(4)                                  # the identity-order flag
    return n


def _oracle(boo, xn):
    d = {f: getattr(boo, f) for f in O.BOO_FIELDS}
    d.update(rows=boo.rows, cols=boo.cols)
    return O.boo_matmul(d, xn)


def test_group_table_gives_the_same_bits(cuda):
    """On CUDA cores the plan only replaces the search for each group's
    blocks: the same bits.  (On the tensor cores a plan also packs sparse
    blocks into tensor-core tiles: test_packed_tiles_product.)"""
    mat = workloads.fem3d(n=9)
    dev = S.csr_to_boo(mat, cluster='identity', target_nr=32, target_nc=32).to('cuda')
    x = torch.randn(mat.shape[1], 128, generator=torch.Generator().manual_seed(1)).cuda()
    assert torch.equal(_product(dev, x, 'cuda_cores', True), _product(dev, x, 'cuda_cores', False))


def _scattered(n, seed, dtype):
    """Remainder-major with scattered small blocks, as HEM leaves a power-law
    graph: 8 random columns per row (the remainder) plus blocks of 6 entries
    inside 32 x 32 boxes, many of them in one hub row group."""
    rng = np.random.default_rng(seed)
    r = np.repeat(np.arange(n), 8)
    c = rng.integers(0, n, r.size)
    boxes = [(int(rng.integers(0, n // 32)), int(rng.integers(0, n // 32))) for _ in range(200)]
    boxes += [(3, int(g)) for g in rng.choice(n // 32, 120, replace=False)]     # the hub group 3
    br, bc = [], []
    for gr, gc in boxes:
        br += list(32 * gr + rng.integers(0, 32, 6))
        bc += list(32 * gc + rng.integers(0, 32, 6))
    rr = np.concatenate([r, br])
    cc = np.concatenate([c, bc])
    mat = sp.csr_matrix((rng.standard_normal(rr.size), (rr, cc)), shape=(n, n))
    mat.sum_duplicates()
    mat.sort_indices()
    return mat.astype(dtype)


@pytest.mark.parametrize('dtype', [np.float32, np.float64])
@pytest.mark.parametrize('k', [64, 96])
def test_row_view_of_scattered_blocks(cuda, dtype, k):
    """A remainder-major matrix with a share of its entries in scattered
    blocks (a hub group among them): the plan's row-ordered pass."""
    mat = _scattered(6400, 5, dtype)
    boo = S.csr_to_boo(mat, cluster='identity', target_nr=32, target_nc=32, small_block_threshold=4)
    s = boo._sizes
    assert 2 * s['rem_nnz'] >= s['total_nnz'] and 64 * s['nnz_c'] >= s['total_nnz']
    dev = boo.to('cuda')
    L = _lib.lib()
    st = dev._dev_struct(dev._gpu_meta)
    assert L.spmm_boo_plan_size(C.byref(st)) == _plan_size(s, dtype == np.float32)
    tdt = torch.float32 if dtype == np.float32 else torch.float64
    x = torch.from_numpy(np.random.default_rng(k).standard_normal((2, mat.shape[1], k))).to(tdt)
    ref = _oracle(boo, x.numpy())
    bound = abs_bound(mat.indptr, mat.indices, mat.data, x.numpy())
    with_plan = _product(dev, x.cuda(), 'auto', True).cpu().numpy()
    without = _product(dev, x.cuda(), 'auto', False).cpu().numpy()
    assert_spmm_close(with_plan, ref, bound, TOL[np.dtype(dtype)])
    assert_spmm_close(without, ref, bound, TOL[np.dtype(dtype)])
    got = S.boo_matmul(dev, x.cuda()).cpu().numpy()          # the public API uses the plan
    np.testing.assert_array_equal(got, with_plan)


def test_plan_without_row_view(cuda):
    """A remainder-major matrix whose blocks hold under 1/64 of its entries
    (1,974 of 131,072 here) keeps the two-step path; its plan is the group
    table and the packing arrays, and the product is the plan-less one."""
    mat = workloads.uniform(n=16384)
    boo = S.csr_to_boo(mat, cluster='identity', target_nr=32, target_nc=32)
    dev = boo.to('cuda')
    st = dev._dev_struct(dev._gpu_meta)
    L = _lib.lib()
    assert L.spmm_boo_plan_size(C.byref(st)) == _plan_size(boo._sizes)
    assert 0 < L.spmm_boo_plan_workspace_size(C.byref(st))          # the packing pass only
    x = torch.randn(mat.shape[1], 64, generator=torch.Generator().manual_seed(3)).cuda()
    assert torch.equal(_product(dev, x, 'auto', True), _product(dev, x, 'auto', False))


@pytest.mark.parametrize('dtype', [np.float32, np.float64])
@pytest.mark.parametrize('k', [128, 7, 300])
@pytest.mark.parametrize('cluster', ['identity', 'random'])
def test_short_rows_through_the_row_view(cuda, dtype, k, cluster):
    """A few entries per row (2-D Laplacian, tail entries from a small-block
    threshold): the plan holds the row-ordered copy and a warp per row
    computes Y, rows in any group order, any K, two batches."""
    mat = workloads.laplacian2d(n=70).astype(dtype)
    boo = S.csr_to_boo(mat, cluster=cluster, target_nr=32, target_nc=32, small_block_threshold=40,
                       small_block_policy='tail_batch')
    s = boo._sizes
    assert s['nnz_c'] + s['rem_nnz'] + s['tail_nnz'] <= 16 * s['rows']
    dev = boo.to('cuda')
    st = dev._dev_struct(dev._gpu_meta)
    assert _lib.lib().spmm_boo_plan_size(C.byref(st)) == _plan_size(s, dtype == np.float32)
    tdt = torch.float32 if dtype == np.float32 else torch.float64
    x = torch.from_numpy(np.random.default_rng(k).standard_normal((2, mat.shape[1], k))).to(tdt)
    ref = _oracle(boo, x.numpy())
    bound = abs_bound(mat.indptr, mat.indices, mat.data, x.numpy())
    with_plan = _product(dev, x.cuda(), 'cuda_cores', True).cpu().numpy()
    assert_spmm_close(with_plan, ref, bound, TOL[np.dtype(dtype)])
    np.testing.assert_array_equal(S.boo_matmul(dev, x.cuda()).cpu().numpy(), with_plan)


def test_plan_arguments(cuda):
    mat = workloads.fem3d(n=4)
    dev = S.csr_to_boo(mat, cluster='identity', target_nr=32, target_nc=32).to('cuda')
    st = dev._dev_struct(dev._gpu_meta)
    L = _lib.lib()
    n = L.spmm_boo_plan_size(C.byref(st))
    w = L.spmm_boo_plan_workspace_size(C.byref(st))
    buf = torch.empty(n + 512, dtype=torch.uint8, device='cuda')
    ws = torch.empty(w, dtype=torch.uint8, device='cuda')
    assert L.spmm_boo_plan_build(C.byref(st), buf.data_ptr(), n - 1, ws.data_ptr(), w, None) == _lib.SPMM_EWORKSPACE
    assert L.spmm_boo_plan_build(C.byref(st), buf.data_ptr() + 16, n, ws.data_ptr(), w, None) == _lib.SPMM_EALIGN
    assert L.spmm_boo_plan_build(C.byref(st), None, n, ws.data_ptr(), w, None) == _lib.SPMM_EINVAL
    assert L.spmm_boo_plan_build(C.byref(st), buf.data_ptr(), n, None, 0, None) == _lib.SPMM_EWORKSPACE
    assert L.spmm_boo_plan_build(C.byref(st), buf.data_ptr(), n, ws.data_ptr(), w, None) == 0
    torch.cuda.synchronize()
    rg_blk = buf[:4 * (dev.num_row_groups() + 1)].view(torch.int32).cpu().numpy()
    want = np.searchsorted(dev.blk_row_grp, np.arange(dev.num_row_groups() + 1), side='left')
    np.testing.assert_array_equal(rg_blk, want)


def _packing_rule(boo):
    """The plan's packing, restated: sparse blocks (< 48 entries) whose
    entries lie in one or two 4-column quads with >= 3 entries per quad;
    slots = (block, quad) in block order, quads ascending."""
    ptr = np.asarray(boo.blk_nz_ptr, dtype=np.int64)
    idx = np.asarray(boo.nz_idx).astype(np.int64)
    shift = np.asarray(boo.blk_shift).astype(np.int64)
    packed = np.zeros(boo.num_blocks(), dtype=np.uint8)
    slots = []
    for b in range(boo.num_blocks()):
        k0, k1 = ptr[b], ptr[b + 1]
        if k1 - k0 >= 48:
            continue
        quads = np.unique((idx[k0:k1] & ((1 << shift[b]) - 1)) >> 2)
        if 1 <= quads.size <= 2 and k1 - k0 >= 3 * quads.size:
            packed[b] = 1
            slots += [b * 16 + int(q) for q in quads]
    return packed, np.array(slots, dtype=np.int64)


@pytest.mark.parametrize('name,gen,kw,target', [
    ('fem3d', workloads.fem3d, dict(n=11), 32),
    ('blockdiag', workloads.blockdiag, dict(n_blocks=12, b=64), 64),
])
def test_packed_slots_follow_the_rule(cuda, name, gen, kw, target):
    mat = gen(**kw)
    boo = S.csr_to_boo(mat, cluster='identity', target_nr=target, target_nc=target)
    dev = boo.to('cuda')
    plan = S.boo.product_plan(dev, dev._gpu_meta).cpu().numpy()
    s = boo._sizes
    al = lambda v: (v + 255) // 256 * 256          # noqa: E731
    off_packed = al(4 * (s['n_rg'] + 1))
    off_rgslot = off_packed + al(s['nb'])
    off_slots = off_rgslot + al(4 * (s['n_rg'] + 1))
    packed = plan[off_packed:off_packed + s['nb']]
    rg_slot = plan[off_rgslot:off_rgslot + 4 * (s['n_rg'] + 1)].view(np.int32)
    want_packed, want_slots = _packing_rule(boo)
    np.testing.assert_array_equal(packed, want_packed)
    assert rg_slot[-1] == want_slots.size
    slots = plan[off_slots:off_slots + 4 * want_slots.size].view(np.int32)
    np.testing.assert_array_equal(slots, want_slots)
    if name == 'fem3d':
        assert want_slots.size > 0                  # the mesh's corner blocks are packed (241 blocks at n = 11)


@pytest.mark.parametrize('n,k', [(8, 128), (11, 256)])
def test_packed_tiles_product(cuda, n, k):
    """Tensor-core product with the plan (corner blocks in packed tiles) and
    without it (corner blocks on CUDA cores): both within 1e-5 of the oracle."""
    mat = workloads.fem3d(n=n)
    boo = S.csr_to_boo(mat, cluster='identity', target_nr=32, target_nc=32)
    dev = boo.to('cuda')
    x = torch.from_numpy(np.random.default_rng(n).standard_normal((mat.shape[1], k)).astype(np.float32))
    ref = _oracle(boo, x.numpy())
    bound = abs_bound(mat.indptr, mat.indices, mat.data, x.numpy())
    for with_plan in (True, False):
        got = _product(dev, x.cuda(), 'tensor_cores', with_plan).cpu().numpy()
        assert_spmm_close(got, ref, bound, TOL[np.dtype(np.float32)])
    assert _lib.lib().spmm_tc_status(1) == 0
