"""Shared test configuration.

Tests marked ``gpu`` need a CUDA device (B200); everything else runs on CPU.
The CPU oracle (``oracle/``) is the checker; the reference's own core, when
built into ``oracle/_ref`` (``python oracle/build_ref.py``), pins the oracle.
"""

import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line('markers', 'gpu: needs a CUDA device (sm_100a)')


def abs_bound(indptr, indices, data, x):
    """(|A| |X|) in float64, the scale of the tolerance max|dY| <= tol * (|A||X|)."""
    import scipy.sparse as sp
    n_rows = len(indptr) - 1
    x = np.asarray(x, dtype=np.float64)
    x3 = x[None] if x.ndim == 2 else x
    a = sp.csr_matrix((np.abs(np.asarray(data, dtype=np.float64)), np.asarray(indices),
                       np.asarray(indptr)), shape=(n_rows, x3.shape[1]))
    out = np.stack([a @ np.abs(xb) for xb in x3])
    return out[0] if x.ndim == 2 else out


def assert_spmm_close(y, y_ref, bound, tol):
    """Elementwise |y - y_ref| <= tol * bound (+ a denormal-sized floor)."""
    y = np.asarray(y, dtype=np.float64)
    y_ref = np.asarray(y_ref, dtype=np.float64)
    assert y.shape == y_ref.shape, (y.shape, y_ref.shape)
    err = np.abs(y - y_ref)
    lim = tol * np.asarray(bound) + 1e-30
    bad = err > lim
    if bad.any():
        i = np.argmax(err - lim)
        raise AssertionError(f'{int(bad.sum())} elements out of tolerance; worst at flat index {i}: '
                             f'|dy|={err.flat[i]:.3e} > {lim.flat[i]:.3e} (tol {tol})')


TOL = {np.dtype(np.float32): 1e-5, np.dtype(np.float64): 1e-12}


@pytest.fixture(scope='session')
def cuda():
    import torch
    if not torch.cuda.is_available():
        pytest.fail('CUDA device required for gpu-marked tests')
    return torch.device('cuda', 0)
