"""Row-group-range products (spmm_boo_matmul_groups) and the host-operand
path that overlaps the PCIe copies with them (spmm_b200.pipeline).

A partition of the row groups multiplied range by range gives the whole
product bit for bit, on both engines, and touches no Y row outside its
range; the pipelined host call gives the device call's bits."""

import ctypes as C

import numpy as np
import pytest
import scipy.sparse as sp
import torch

import spmm_b200 as S
from spmm_b200 import _lib, pipeline, workloads
from spmm_b200._device import stream_handle

pytestmark = pytest.mark.gpu


def _groups_call(dev, x, y, rg0, rg1, engine):
    L = _lib.lib()
    st = dev._dev_struct(dev._gpu_meta)
    K = x.shape[-1]
    plan = S.boo.product_plan(dev, dev._gpu_meta)      # as the whole-matrix call through the API
    cfg = _lib.launch_cfg(engine, plan=plan.data_ptr())
    n = L.spmm_boo_matmul_workspace_size(C.byref(st), 1, K, C.byref(cfg))
    ws = torch.empty(max(n, 16), dtype=torch.uint8, device='cuda')
    if n:
        cfg.workspace, cfg.workspace_bytes = ws.data_ptr(), n
    rc = L.spmm_boo_matmul_groups(C.byref(st), C.c_void_p(x.data_ptr()), C.c_void_p(y.data_ptr()), 1, K, rg0, rg1,
                                  C.byref(cfg), stream_handle(x.device))
    torch.cuda.synchronize()
    return rc


@pytest.mark.parametrize('engine', ['tensor_cores', 'cuda_cores'])
@pytest.mark.parametrize('name,gen,kw,target', [
    ('fem3d', workloads.fem3d, dict(n=10), 32),
    ('blockdiag', workloads.blockdiag, dict(n_blocks=20, b=64), 64),
    ('laplacian2d', workloads.laplacian2d, dict(n=64), 32),     # short rows: a warp per row
])
def test_ranges_reassemble_the_product(cuda, engine, name, gen, kw, target):
    mat = gen(**kw)
    rows, cols = mat.shape
    boo = S.csr_to_boo(mat, cluster='identity', target_nr=target, target_nc=target)
    dev = boo.to('cuda')
    x = torch.randn(cols, 128, generator=torch.Generator().manual_seed(1)).cuda()
    full = S.boo_matmul(dev, x, engine=engine)
    n_rg = boo.num_row_groups()
    cuts = [0, 1, n_rg // 3, n_rg // 3, n_rg - 2, n_rg]          # includes an empty range
    y = torch.full((rows, 128), float('nan'), device='cuda')
    rgp = boo.row_grp_ptr
    for a, b in zip(cuts[:-1], cuts[1:]):
        before = y.clone()
        assert _groups_call(dev, x, y, a, b, engine) == 0
        r0, r1 = int(rgp[a]), int(rgp[b])
        assert torch.equal(y[r0:r1], full[r0:r1])
        outside = torch.ones(rows, dtype=torch.bool, device='cuda')
        outside[r0:r1] = False
        assert torch.equal(y[outside].isnan(), before[outside].isnan())   # untouched
    assert torch.equal(y, full)


def test_range_arguments(cuda):
    mat = workloads.fem3d(n=6)
    dev = S.csr_to_boo(mat, cluster='identity', target_nr=32, target_nc=32).to('cuda')
    x = torch.randn(mat.shape[1], 128, device='cuda')
    y = torch.empty(mat.shape[0], 128, device='cuda')
    n_rg = dev.num_row_groups()
    for a, b in ((-1, 2), (3, 2), (0, n_rg + 1)):
        assert _groups_call(dev, x, y, a, b, 'auto') == _lib.SPMM_EINVAL
    um = workloads.uniform(n=4096)                                    # remainder-major
    ub = S.csr_to_boo(um, cluster='identity', target_nr=32, target_nc=32).to('cuda')
    xu = torch.randn(um.shape[1], 128, device='cuda')
    yu = torch.empty(um.shape[0], 128, device='cuda')
    assert _groups_call(ub, xu, yu, 0, 3, 'auto') == _lib.SPMM_EUNSUPPORTED
    assert _groups_call(ub, xu, yu, 0, ub.num_row_groups(), 'auto') == 0


@pytest.mark.parametrize('engine', ['auto', 'cuda_cores'])
def test_pipelined_host_call_matches_device_call(cuda, engine):
    mat = workloads.fem3d(n=24)                                       # X 42 MB at K = 256
    boo = S.csr_to_boo(mat, cluster='identity', target_nr=32, target_nc=32)
    dev = boo.to('cuda')
    x = torch.randn(mat.shape[1], 256, generator=torch.Generator().manual_seed(5)).pin_memory()
    assert pipeline.applies(boo, x)
    for _ in range(2):
        y = S.boo_matmul(dev, x, engine=engine)
        assert y.device.type == 'cpu' and y.is_pinned()
        assert torch.equal(y, S.boo_matmul(dev, x.cuda(), engine=engine).cpu())
    y3 = S.boo_matmul(dev, x.unsqueeze(0), engine=engine)             # batch of one
    assert y3.shape == (1, mat.shape[0], 256) and torch.equal(y3[0], y)


def test_pipeline_plan_windows(cuda):
    """Every chunk's X rows lie below the X rows waited for."""
    rng = np.random.default_rng(3)
    mat = workloads.fem3d(n=16)
    boo = S.csr_to_boo(mat, cluster='identity', target_nr=32, target_nc=32)
    pl = pipeline.plan(boo)
    assert pl is not None and pl.rg_bounds[0] == 0 and pl.rg_bounds[-1] == boo.num_row_groups()
    for i in range(len(pl.rg_bounds) - 1):
        r0, r1 = pl.row_bounds[i], pl.row_bounds[i + 1]
        sub = mat[r0:r1]
        if sub.nnz:
            assert sub.indices.max() < pl.x_need[i]
    shuffled = S.csr_to_boo(mat, row_labels=rng.permutation(mat.shape[0]) // 32,
                            col_labels=np.arange(mat.shape[1]) // 32)
    assert pipeline.plan(shuffled) is None                            # rows not in identity order
