"""HEM labels on the GPU (spmm_hem_labels / spmm_hem_hierarchy) against the C
oracle's restatement of the reference's multilevel heavy-edge matching
(clustering.py:128-351; oracle/hem_oracle.c, itself pinned to the
reference's labels by tests/test_clustering.py): identical labels and
per-level hierarchy across hub pruning, top-k, size / nnz caps,
feasible-first filtering, ties and empty rows."""

import numpy as np
import pytest
import scipy.sparse as sp

from spmm_b200 import workloads
from oracle import oracle as O
from spmm_b200.clustering import _pattern, cluster_axes, cluster_axis, hem_labels_gpu

pytestmark = pytest.mark.gpu


def _cases():
    rng = np.random.default_rng(4)
    rect = sp.random(500, 800, density=0.02, format='csr', random_state=1)
    ties = sp.csr_matrix(np.kron(np.eye(40), np.ones((3, 5))))      # identical rows: ties everywhere
    empty_rows = sp.random(300, 300, density=0.03, format='csr', random_state=2).tolil()
    empty_rows[50:80] = 0
    # rows sharing column pools: 600 rows of ~10,800 incidences (counted by
    # sorting), 600 of ~6,000 (the 512-thread hash tables), sparse rows after
    pr, pc = [], []
    for r in range(1600):
        if r < 600:
            c = rng.choice(200, 60, replace=False)
        elif r < 1200:
            c = 200 + rng.choice(250, 50, replace=False)
        else:
            c = rng.choice(1600, 5, replace=False)
        pr += [r] * c.size
        pc += list(c)
    pools = sp.csr_matrix((np.ones(len(pr)), (pr, pc)), shape=(1600, 1600))
    # one row over every column: each other row's heaviest neighbour, so the
    # level graph gives it ~5,000 edges (picked by a CTA of its own)
    sr = [0] * 5000 + list(np.repeat(np.arange(1, 5000), 3))
    sc = list(range(5000)) + [int(c) for i in range(1, 5000) for c in (i, (7 * i + 1) % 5000, (13 * i + 2) % 5000)]
    star = sp.csr_matrix((np.ones(len(sr)), (sr, sc)), shape=(5000, 5000))
    return {
        'star': star,
        'pools': pools,
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
    host = O.hem_labels(pat, params['target'], params['max_size'], params['max_nnz'], params['hub_degree'],
                        params['topk'], feasible_first=params['feasible_first'])
    gpu = hem_labels_gpu(pat, params['target'], params['max_size'], params['max_nnz'], params['hub_degree'],
                         params['topk'], params['feasible_first'])
    np.testing.assert_array_equal(gpu, host)


def test_cluster_axes_uses_gpu_labels(cuda):
    """csr_to_boo's clustering (cluster='hem') gives the oracle's labels after
    the same cap enforcement."""
    mat = workloads.powerlaw(n=2000)
    rl, cl = cluster_axes(mat, method='hem', target_nr=32, target_nc=32, max_nr=32, max_nc=32, feasible_first=True)
    want = O.hem_cluster(mat, 32, 32, None, feasible_first=True)
    np.testing.assert_array_equal(rl, want)
    np.testing.assert_array_equal(cl, want)        # symmetric pattern: one clustering for both axes


@pytest.mark.parametrize('name', ['fem3d', 'powerlaw', 'rect_cols', 'ties', 'tiny'])
def test_hierarchy_equals_oracle(cuda, name):
    """hem_hierarchy=[]: identity, then the labels after every level that
    matched, finest to coarsest, as the reference records them."""
    pat = _pattern(CASES[name])
    got = []
    lab = cluster_axis(CASES[name], method='hem', target=16, max_size=16, hem_hierarchy=got)
    _, want = O.hem_labels(pat, 16, 16, None, 1024, 32, hierarchy=True)
    assert len(got) == len(want) >= 1
    for g, w in zip(got, want):
        np.testing.assert_array_equal(g, w)
    np.testing.assert_array_equal(lab, O.hem_cluster(CASES[name], 16, 16, None))
