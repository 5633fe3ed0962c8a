"""Argument checks of the drop-in API that fire before any GPU work, with the
reference's exception types and messages (boo.py:149-200;
tests/torch_fast_spdmm/test_boo_edges.py:308-383)."""

import numpy as np
import pytest
import scipy.sparse as sp
import torch

from spmm_b200 import csr_to_boo, csr_to_pbr


def _example(dtype=np.float32, index_dtype=np.int32):
    entries = [(0, 0, 2), (0, 2, -1), (2, 6, 3), (2, 0, 1), (0, 1, 4), (1, 1, 2), (1, 4, -3),
               (4, 7, 1), (4, 9, 2), (4, 3, -2), (3, 5, 1)]
    r, c, v = zip(*entries)
    mat = sp.csr_matrix((np.array(v, dtype=dtype), (r, c)), shape=(7, 11))
    mat.indptr = mat.indptr.astype(index_dtype)
    mat.indices = mat.indices.astype(index_dtype)
    return mat, np.array([0, 1, 0, 2, 1, 0, 2]), np.array([0, 1, 0, 2, 1, 2, 0, 1, 2, 1, 2])


@pytest.mark.parametrize('kwargs', [{'target_nr': 0}, {'max_nc': -1}, {'max_block_nnz': 0},
                                    {'small_block_threshold': -1}, {'nz_order': 'unknown'},
                                    {'small_block_policy': 'unknown'}])
def test_invalid_builder_parameters(kwargs):
    with pytest.raises(ValueError):
        csr_to_boo(_example()[0], **kwargs)


@pytest.mark.parametrize('case', ['missing', 'length', 'rank', 'negative', 'too_large', 'float'])
def test_invalid_labels(case):
    mat, rl, cl = _example()
    if case == 'missing':
        cl = None
    elif case == 'length':
        rl = rl[:-1]
    elif case == 'rank':
        rl = rl.reshape(1, -1)
    elif case == 'negative':
        rl[0] = -1
    elif case == 'too_large':
        rl[0] = 2 ** 40
    else:
        rl = rl.astype(float) + 0.5
    with pytest.raises((ValueError, TypeError), match='labels'):
        csr_to_boo(mat, row_labels=rl, col_labels=cl)


def test_builder_input_contract():
    mat, rl, cl = _example()
    with pytest.raises(TypeError, match='float32/float64'):
        csr_to_boo(mat.astype(np.int32))
    with pytest.raises(ValueError, match='sparse CSR'):
        csr_to_boo(torch.zeros(7, 11))
    broken = mat.copy()
    broken.indices[0] = 11
    with pytest.raises(ValueError):
        csr_to_boo(broken)
    with pytest.raises(TypeError):
        csr_to_boo([[1.0]])


def test_merge_policy_is_rejected_clearly():
    mat, rl, cl = _example()
    with pytest.raises(Exception, match='merge'):
        csr_to_boo(mat, row_labels=rl, col_labels=cl, small_block_policy='merge')


def test_pbr_argument_checks():
    mat = _example()[0]
    with pytest.raises(TypeError):
        csr_to_pbr([[1.0]])
    with pytest.raises(TypeError):
        csr_to_pbr(mat, min_nnz_per_block=256)
    with pytest.raises(ValueError):
        csr_to_pbr(mat, block_rows=9, block_cols=8)


def test_no_cpu_fallback_without_cuda(monkeypatch):
    """Without a CUDA device the product raises instead of computing on the CPU."""
    monkeypatch.setattr(torch.cuda, 'is_available', lambda: False)
    mat, rl, cl = _example()
    with pytest.raises(RuntimeError, match='CUDA'):
        csr_to_boo(mat, row_labels=rl, col_labels=cl)
    with pytest.raises(RuntimeError, match='CUDA'):
        csr_to_pbr(mat)
