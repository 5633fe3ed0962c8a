"""HEM labels on the GPU (spmm_hem_labels) against the host restatement of
the reference's multilevel heavy-edge matching (clustering.py:128-351):
identical labels level for level's end result, across hub pruning, top-k,
size / nnz caps, feasible-first filtering, ties and empty rows."""

import numpy as np
import pytest
import scipy.sparse as sp

from spmm_b200 import workloads
from spmm_b200._hem import hem_labels
from spmm_b200.clustering import _pattern, cluster_axes, hem_labels_gpu

pytestmark = pytest.mark.gpu


def _cases():
    rng = np.random.default_rng(4)
    rect = sp.random(500, 800, density=0.02, format='csr', random_state=1)
    ties = sp.csr_matrix(np.kron(np.eye(40), np.ones((3, 5))))      # identical rows: ties everywhere
    empty_rows = sp.random(300, 300, density=0.03, format='csr', random_state=2).tolil()
    empty_rows[50:80] = 0
    return {
        'fem3d': workloads.fem3d(n=5),
        'laplacian2d': workloads.laplacian2d(n=30),
        'powerlaw': workloads.powerlaw(n=3000),
        'rect_rows': rect,
        'rect_cols': rect.T.tocsr(),
        'ties': ties,
        'empty_rows': empty_rows.tocsr(),
        'tiny': sp.csr_matrix(rng.random((3, 3)) > 0.5),
    }


CASES = _cases()


@pytest.mark.parametrize('name', sorted(CASES))
@pytest.mark.parametrize('params', [
    dict(target=32, max_size=32, max_nnz=None, hub_degree=1024, topk=32, feasible_first=True),
    dict(target=32, max_size=None, max_nnz=None, hub_degree=1024, topk=32, feasible_first=False),
    dict(target=8, max_size=8, max_nnz=200, hub_degree=40, topk=4, feasible_first=True),
    dict(target=16, max_size=16, max_nnz=None, hub_degree=1024, topk=None, feasible_first=False),
], ids=['default', 'uncapped', 'caps_hub_topk4', 'topk_all'])
def test_gpu_labels_equal_host(cuda, name, params):
    pat = _pattern(CASES[name])
    host = hem_labels(pat, params['target'], params['max_size'], params['max_nnz'], params['hub_degree'],
                      params['topk'], True, feasible_first=params['feasible_first'])
    gpu = hem_labels_gpu(pat, params['target'], params['max_size'], params['max_nnz'], params['hub_degree'],
                         params['topk'], params['feasible_first'])
    np.testing.assert_array_equal(gpu, host)


def test_cluster_axes_uses_gpu_labels(cuda):
    """csr_to_boo's clustering (cluster='hem') gives the host restatement's labels."""
    mat = workloads.powerlaw(n=2000)
    rl, cl = cluster_axes(mat, method='hem', target_nr=32, target_nc=32, max_nr=32, max_nc=32, feasible_first=True)
    from spmm_b200.clustering import _enforce_caps, _relabel_consecutive
    pat = _pattern(mat)
    host = hem_labels(pat, 32, 32, None, 1024, 32, True, feasible_first=True)
    want = _relabel_consecutive(_enforce_caps(host, np.diff(pat.indptr), 32, None)).astype(np.int32)
    np.testing.assert_array_equal(rl, want)
    np.testing.assert_array_equal(cl, want)        # symmetric pattern: one clustering for both axes
