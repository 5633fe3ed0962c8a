"""The CPU oracle against golden fixtures produced by the reference itself
(tests/golden/gen_golden.py).  Bit-exact: format arrays, CPU SpMM results and
the inverse conversions."""

import json
import os

import numpy as np
import pytest

from oracle import oracle as O

GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), 'golden')
MANIFEST = json.load(open(os.path.join(GOLD, 'manifest.json')))
BOO = np.load(os.path.join(GOLD, 'boo_golden.npz'))
PBR = np.load(os.path.join(GOLD, 'pbr_golden.npz'))


def _eq(a, b):
    a, b = np.asarray(a), np.asarray(b)
    return a.shape == b.shape and np.array_equal(a.astype(b.dtype) if a.dtype != b.dtype else a, b)


@pytest.mark.parametrize('case', MANIFEST['boo'], ids=lambda c: f"boo{c['case']}")
def test_boo_oracle_matches_reference_fixture(case):
    p = f"b{case['case']}/"
    g = {k[len(p):]: BOO[k] for k in BOO.files if k.startswith(p)}
    ob = O.boo_build(g['indptr'], g['indices'], g['data'], case['rows'], case['cols'],
                     g['row_labels'], g['col_labels'], case['policy'], case['threshold'],
                     case['order'])
    for f in O.BOO_FIELDS:
        assert _eq(g[f], ob[f]), f
    for f in ('max_nr', 'max_nc', 'max_nnz_blk', 'total_nnz'):
        assert ob[f] == case[f], f
    # CPU SpMM on the reference's own arrays, bit for bit
    ref = dict(g, rows=case['rows'], cols=case['cols'])
    assert np.array_equal(O.boo_matmul(ref, g['x']), g['y'])
    assert np.array_equal(O.boo_matmul(ob, g['x']), g['y'])
    ip, ix, dv = O.boo_to_csr(ob)
    assert _eq(g['csr_indptr'], ip) and _eq(g['csr_indices'], ix) and _eq(g['csr_data'], dv)


@pytest.mark.parametrize('case', MANIFEST['pbr'], ids=lambda c: f"pbr{c['case']}")
def test_pbr_oracle_matches_reference_fixture(case):
    p = f"p{case['case']}/"
    g = {k[len(p):]: PBR[k] for k in PBR.files if k.startswith(p)}
    meta = dict(rows=case['rows'], cols=case['cols'], block_rows=case['block_rows'],
                block_cols=case['block_cols'], total_nnz=case['total_nnz'])
    ref = dict(meta, **{f: g[f] for f in O.PBR_FIELDS})
    op = O.pbr_build(g['indptr'], g['indices'], g['data'], case['rows'], case['cols'],
                     case['block_rows'], case['block_cols'], case['min_nnz'])
    canon = O.pbr_canonical(ref)
    for f in O.PBR_FIELDS:
        assert _eq(canon[f], op[f]), f
    # CPU SpMM in the reference's own block order reproduces its result exactly
    assert np.array_equal(O.pbr_matmul(ref, g['x']), g['y'])
    ip, ix, dv = O.pbr_to_csr(op)
    assert _eq(g['csr_indptr'], ip) and _eq(g['csr_indices'], ix) and _eq(g['csr_data'], dv)


def test_uint16_overflow_rejected_by_oracle():
    c = MANIFEST['boo_overflow']
    indptr = np.zeros(c['rows'] + 1, np.int64)
    indptr[c['entry'][0] + 1:] = 1
    with pytest.raises(O.OracleError) as e:
        O.boo_build(indptr, np.array([c['entry'][1]]), np.array([1.0], np.float32), c['rows'],
                    c['cols'], np.zeros(c['rows'], np.int32), np.zeros(c['cols'], np.int32), 'keep', 0,
                    'rowmajor')
    assert e.value.code == 2


def test_merge_policy_rejected_by_oracle():
    with pytest.raises(O.OracleError) as e:
        O.boo_build(np.array([0, 1]), np.array([0]), np.array([1.0]), 1, 1, [0], [0], 'merge', 0,
                    'rowmajor')
    assert e.value.code == 3
