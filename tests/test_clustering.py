"""Clustering labels against the reference's clustering module (golden
fixtures from tests/golden/gen_golden.py), plus cap invariants.

CPU: the product's host methods (identity, random, degree, rcm) and the C
oracle's HEM (oracle/hem_oracle.c) against the fixtures; the product's cap
enforcement against the oracle's.  GPU: the product's HEM (spmm_hem_labels)
against the same fixtures."""

import json
import os

import numpy as np
import pytest
import scipy.sparse as sp

from oracle import oracle as O
from spmm_b200.clustering import _enforce_caps, _pattern, cluster_axes, cluster_axis, is_pattern_symmetric

GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), 'golden')
MANIFEST = json.load(open(os.path.join(GOLD, 'manifest.json')))
CL = np.load(os.path.join(GOLD, 'clustering_golden.npz'))
HEM_CASES = [c for c in MANIFEST['clustering'] if c['method'] == 'hem']
HOST_CASES = [c for c in MANIFEST['clustering'] if c['method'] != 'hem']
KW = ('method', 'target_nr', 'target_nc', 'max_nr', 'max_nc', 'max_block_nnz', 'seed', 'feasible_first')


def _case(case):
    p = f"c{case['case']}/"
    n = case['n']
    a = sp.csr_matrix((CL[p + 'data'], CL[p + 'indices'], CL[p + 'indptr']), shape=(n, n))
    return a, CL[p + 'row_labels'], CL[p + 'col_labels']


@pytest.mark.parametrize('case', HOST_CASES, ids=lambda c: f"{c['method']}{c['case']}")
def test_host_labels_match_reference(case):
    a, want_r, want_c = _case(case)
    rl, cl = cluster_axes(a, **{k: case[k] for k in KW})
    assert np.array_equal(rl, want_r)
    assert np.array_equal(cl, want_c)


@pytest.mark.parametrize('case', HEM_CASES, ids=lambda c: f"hem{c['case']}")
def test_oracle_hem_matches_reference(case):
    """The checker of the GPU labeller is pinned to the reference's labels."""
    a, want_r, want_c = _case(case)
    kw = dict(max_nnz=case['max_block_nnz'], feasible_first=case['feasible_first'])
    rl = O.hem_cluster(a, case['target_nr'], case['max_nr'], **kw)
    sym = case['target_nr'] == case['target_nc'] and is_pattern_symmetric(a)
    cl = rl if sym else O.hem_cluster(a.T.tocsr(), case['target_nc'], case['max_nc'], **kw)
    assert np.array_equal(rl, want_r)
    assert np.array_equal(cl, want_c)


@pytest.mark.gpu
@pytest.mark.parametrize('case', HEM_CASES, ids=lambda c: f"hem{c['case']}")
def test_gpu_hem_matches_reference(cuda, case):
    """cluster='hem' through the product (GPU labels) gives the reference's labels."""
    a, want_r, want_c = _case(case)
    rl, cl = cluster_axes(a, **{k: case[k] for k in KW})
    assert np.array_equal(rl, want_r)
    assert np.array_equal(cl, want_c)


@pytest.mark.parametrize('seed', range(12))
def test_enforce_caps_matches_oracle(seed):
    rng = np.random.default_rng(seed)
    n = int(rng.integers(1, 400))
    labels = rng.integers(0, max(1, n // int(rng.integers(1, 40))), n) * int(rng.integers(1, 4))
    row_nnz = rng.integers(0, 60, n)
    max_size = [None, int(rng.integers(1, 20))][seed % 2]
    max_nnz = [None, int(rng.integers(1, 300))][(seed // 2) % 2]
    got = _enforce_caps(labels.astype(np.int64), row_nnz, max_size, max_nnz)
    _, got = np.unique(got, return_inverse=True)
    np.testing.assert_array_equal(got, O.enforce_caps(labels, row_nnz, max_size, max_nnz))


def test_pattern_and_symmetry():
    rng = np.random.default_rng(2)
    r = rng.integers(0, 50, 400)
    c = rng.integers(0, 60, 400)
    a = sp.coo_matrix((rng.standard_normal(400), (r, c)), shape=(50, 60))   # duplicates
    p = _pattern(a)
    q = O.binary_pattern(a)
    assert np.array_equal(p.indptr, q.indptr) and np.array_equal(p.indices, q.indices)
    assert (p.data == 1).all()
    s = sp.random(40, 40, density=0.1, random_state=1)
    assert is_pattern_symmetric(s + s.T) and not is_pattern_symmetric(sp.triu(s, 1) + sp.eye(40))
    assert not is_pattern_symmetric(a)


@pytest.mark.parametrize('method', ['identity', 'random', 'degree', 'rcm',
                                    pytest.param('hem', marks=pytest.mark.gpu)])
def test_caps_respected(method):
    a = sp.random(300, 300, density=0.03, format='csr', random_state=3)
    a = (a + a.T).tocsr()
    lab = cluster_axis(a, method=method, target=16, max_size=16, max_nnz=200)
    assert lab.dtype == np.int32
    counts = np.bincount(lab)
    assert counts.max() <= 16 and counts.min() >= 1
    nnz = np.bincount(lab, weights=np.diff(a.indptr))
    assert np.all((nnz <= 200) | (counts == 1))


@pytest.mark.parametrize('method', ['identity', 'random', 'degree'])
@pytest.mark.parametrize('max_nnz', [None, 40])
def test_count_methods_need_no_symmetry_test(method, max_nnz):
    """identity / random / degree label each axis from its own counts; on a
    symmetric pattern that equals reusing the row labels (the reference's
    symmetric branch), also for an input with repeated entries."""
    rng = np.random.default_rng(5)
    r, c = rng.integers(0, 200, 1500), rng.integers(0, 200, 1500)
    rows, cols = np.r_[r, c, r[:100]], np.r_[c, r, c[:100]]       # 100 entries repeated
    order = np.argsort(rows, kind='stable')
    a = sp.csr_matrix((np.ones(rows.size), cols[order], np.r_[0, np.cumsum(np.bincount(rows, minlength=200))]),
                      shape=(200, 200))
    assert not a.has_canonical_format
    kw = dict(method=method, target_nr=16, target_nc=16, max_nr=16, max_nc=16, max_block_nnz=max_nnz)
    rl, cl = cluster_axes(a, **kw)
    sr, sc = cluster_axes(a, symmetric=True, **kw)
    assert np.array_equal(rl, sr) and np.array_equal(cl, sc)
    pat = O.binary_pattern(a)
    want = cluster_axis(pat, method=method, target=16, max_size=16, max_nnz=max_nnz)
    assert np.array_equal(rl, want)
    t = sp.random(90, 150, density=0.05, format='csr', random_state=2)
    tr, tc = cluster_axes(t, **kw)
    assert np.array_equal(tc, cluster_axis(t.T.tocsr(), method=method, target=16, max_size=16, max_nnz=max_nnz))
    assert tr.size == 90 and tc.size == 150


def test_missing_backends_do_not_fall_back():
    a = sp.eye(10, format='csr')
    for m in ('graclus', 'metis'):
        with pytest.raises(ImportError):
            cluster_axis(a, method=m)
    with pytest.raises(ValueError):
        cluster_axis(a, method='nope')
    with pytest.raises(ValueError):
        cluster_axis(a, method='identity', hem_hierarchy=[])
