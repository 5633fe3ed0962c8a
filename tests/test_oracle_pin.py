"""Pins the oracle to the reference's own compiled core (oracle/_ref), on a
seeded sweep wider than the committed fixtures.  Skipped where the reference
core has not been built (``python oracle/build_ref.py``)."""

import numpy as np
import pytest
import scipy.sparse as sp

from oracle import oracle as O
from oracle.build_ref import load_reference

core = load_reference()
pytestmark = pytest.mark.skipif(core is None, reason='reference core not built (oracle/build_ref.py)')


def _cases(n):
    rng = np.random.default_rng(7)
    for t in range(n):
        rows, cols = int(rng.integers(1, 150)), int(rng.integers(1, 150))
        m = sp.random(rows, cols, density=float(rng.uniform(0.01, 0.5)), format='csr',
                      random_state=int(rng.integers(1 << 30)))
        dt = np.float32 if t % 2 else np.float64
        idt = np.int32 if t % 3 else np.int64
        m = m.astype(dt)
        m.indptr, m.indices = m.indptr.astype(idt), m.indices.astype(idt)
        yield t, rng, rows, cols, m, dt


@pytest.mark.parametrize('policy', [0, 2, 3])
@pytest.mark.parametrize('order', [0, 1])
def test_boo_sweep(policy, order):
    import torch
    for t, rng, rows, cols, m, dt in _cases(25):
        rl = rng.integers(0, max(1, rows // int(rng.integers(1, 12))), size=rows).astype(np.int32)
        cl = rng.integers(0, max(1, cols // int(rng.integers(1, 12))), size=cols).astype(np.int32)
        thr = int(rng.integers(0, 9))
        ref = core.csr_to_boo(m.indptr, m.indices, m.data, rows, cols, rl, cl, policy, thr, order)
        mine = O.boo_build(m.indptr, m.indices, m.data, rows, cols, rl, cl, policy, thr, order)
        R = O.reference_boo_arrays(ref)
        for f in O.BOO_FIELDS + ('nb', 'nnz_c', 'rem_nnz', 'tail_nnz', 'max_nr', 'max_nc',
                                 'max_nnz_blk', 'n_rg', 'n_cg'):
            assert np.array_equal(np.asarray(R[f]), np.asarray(mine[f])), (t, f)
        x = rng.standard_normal((2, cols, 5)).astype(dt)
        assert np.array_equal(core.boo_batched_matmul_cpu(ref, torch.from_numpy(x)).numpy(),
                              O.boo_matmul(mine, x))


@pytest.mark.parametrize('shape', [(2, 2), (4, 4), (8, 8), (2, 32), (5, 3)])
def test_pbr_sweep(shape):
    import torch
    for t, rng, rows, cols, m, dt in _cases(20):
        mn = int(rng.integers(1, 12))
        ref = core.csr_to_pbr(m.indptr, m.indices, m.data, rows, cols, shape[0], shape[1], mn)
        mine = O.pbr_build(m.indptr, m.indices, m.data, rows, cols, shape[0], shape[1], mn)
        R = O.reference_pbr_arrays(ref)
        C = O.pbr_canonical(R)
        for f in O.PBR_FIELDS:
            assert np.array_equal(np.asarray(C[f]).astype(np.asarray(mine[f]).dtype), mine[f]), (t, f)
        x = rng.standard_normal((1, cols, 4)).astype(dt)
        assert np.array_equal(core.pbr_batched_matmul_cpu(ref, torch.from_numpy(x)).numpy(),
                              O.pbr_matmul(R, x))
