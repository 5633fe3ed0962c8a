"""Host clustering labels against the reference's clustering module (golden
fixtures from tests/golden/gen_golden.py), plus cap invariants."""

import json
import os

import numpy as np
import pytest
import scipy.sparse as sp

from spmm_b200.clustering import cluster_axes, cluster_axis

GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), 'golden')
MANIFEST = json.load(open(os.path.join(GOLD, 'manifest.json')))
CL = np.load(os.path.join(GOLD, 'clustering_golden.npz'))


@pytest.mark.parametrize('case', MANIFEST['clustering'], ids=lambda c: f"{c['method']}{c['case']}")
def test_labels_match_reference(case):
    p = f"c{case['case']}/"
    n = case['n']
    a = sp.csr_matrix((CL[p + 'data'], CL[p + 'indices'], CL[p + 'indptr']), shape=(n, n))
    kw = {k: case[k] for k in ('method', 'target_nr', 'target_nc', 'max_nr', 'max_nc',
                               'max_block_nnz', 'seed', 'feasible_first')}
    rl, cl = cluster_axes(a, **kw)
    assert np.array_equal(rl, CL[p + 'row_labels'])
    assert np.array_equal(cl, CL[p + 'col_labels'])


@pytest.mark.parametrize('method', ['identity', 'random', 'degree', 'rcm', 'hem'])
def test_caps_respected(method):
    a = sp.random(300, 300, density=0.03, format='csr', random_state=3)
    a = (a + a.T).tocsr()
    lab = cluster_axis(a, method=method, target=16, max_size=16, max_nnz=200)
    assert lab.dtype == np.int32
    counts = np.bincount(lab)
    assert counts.max() <= 16 and counts.min() >= 1
    nnz = np.bincount(lab, weights=np.diff(a.indptr))
    assert np.all((nnz <= 200) | (counts == 1))


def test_missing_backends_do_not_fall_back():
    a = sp.eye(10, format='csr')
    for m in ('graclus', 'metis'):
        with pytest.raises(ImportError):
            cluster_axis(a, method=m)
    with pytest.raises(ValueError):
        cluster_axis(a, method='nope')
