"""BOO execution plans (boo_plan.py API): preparation errors, plan validation
in boo_matmul, and that a planned product equals the plain one."""

import numpy as np
import pytest
import scipy.sparse as sp
import torch

import spmm_b200 as S

pytestmark = pytest.mark.gpu


def _mat():
    return sp.random(300, 280, density=0.05, format='csr', random_state=3, dtype=np.float32)


def test_prepare_errors(cuda):
    boo = S.csr_to_boo(_mat(), cluster='identity', target_nr=32, target_nc=32)
    with pytest.raises(ValueError, match='to\\(.cuda.\\)'):
        S.prepare_boo_cuda(boo)
    with pytest.raises(ValueError, match='p must be'):
        S.prepare_boo_cuda(boo.to('cuda'), p=12)
    col = S.csr_to_boo(_mat(), cluster='identity', target_nr=32, target_nc=32, nz_order='colmajor')
    with pytest.raises(ValueError, match='rowmajor'):
        S.prepare_boo_cuda(col.to('cuda'))


@pytest.mark.parametrize('bucketed', [False, True])
@pytest.mark.parametrize('k', [64, 128])
def test_planned_product_equals_plain(cuda, bucketed, k):
    boo = S.csr_to_boo(_mat(), cluster='identity', target_nr=32, target_nc=32).to('cuda')
    plan = S.prepare_boo_cuda(boo, bucketed=bucketed, precomputed_rows=True, p=32)
    assert isinstance(plan, S.BOOExecutionPlan) and plan.extra_device_bytes == 0
    assert plan.buckets[0] == 0 and sum(plan.buckets[1::5]) == boo.num_blocks()
    x = torch.randn(280, k, generator=torch.Generator().manual_seed(k)).cuda()
    y = S.boo_matmul(boo, x, launch_mode='auto', row_seg=True, p=32, execution_plan=plan)
    assert torch.equal(y, S.boo_matmul(boo, x))


def test_plan_validation(cuda):
    boo = S.csr_to_boo(_mat(), cluster='identity', target_nr=32, target_nc=32).to('cuda')
    other = S.csr_to_boo(_mat(), cluster='identity', target_nr=32, target_nc=32).to('cuda')
    plan = S.prepare_boo_cuda(boo, p=64)
    x = torch.randn(280, 16).cuda()
    with pytest.raises(ValueError, match='does not match'):
        S.boo_matmul(other, x, launch_mode='auto', execution_plan=plan)
    with pytest.raises(ValueError, match='launch_mode'):
        S.boo_matmul(boo, x, execution_plan=plan)                         # legacy launch mode
    with pytest.raises(ValueError, match='launch_mode'):
        S.boo_matmul(boo, x, launch_mode='auto', p=32, execution_plan=plan)
    with pytest.raises(ValueError, match='CUDA inputs'):
        S.boo_matmul(boo, x.cpu(), launch_mode='auto', execution_plan=plan)
    boo.to('cpu').to('cuda')                                              # re-staged: plan is stale
    with pytest.raises(ValueError, match='does not match'):
        S.boo_matmul(boo, x, launch_mode='auto', execution_plan=plan)
