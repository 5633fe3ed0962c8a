"""Row / column grouping labels for the BOO format (host side).

The BOO builder takes one int32 label per row and per column; this module
produces them with the methods of the reference's
``torch_fast_spdmm/torch_fast_spdmm/clustering.py`` (``cluster_axis``
:454-509, ``cluster_axes`` :512-545): ``identity`` (consecutive runs,
:483-484), ``random`` and ``degree`` (runs of a permutation, :485-490),
``rcm`` (runs of the reverse Cuthill-McKee order, :491-497) and ``hem``
(multilevel heavy-edge matching, see ``_hem``).  Every method's result goes
through the same cap enforcement (:83-121) and consecutive relabelling.
"""

from __future__ import annotations

from typing import Optional, Tuple

import numpy as np
import scipy.sparse as sp
import torch

__all__ = ['cluster_axes', 'cluster_axis', 'hem_labels_gpu', 'CLUSTER_METHODS']

CLUSTER_METHODS = ('identity', 'random', 'degree', 'rcm', 'hem', 'graclus', 'metis')
DEFAULT_HUB_DEGREE = 1024
DEFAULT_TOPK = 32
DEFAULT_CHUNK_ROWS = 4096


def _pattern(mat) -> sp.csr_matrix:
    """Binary CSR of the sparsity pattern (duplicates merged)."""
    out = sp.csr_matrix(mat, copy=True)
    out.data = np.ones_like(out.data, dtype=np.int32)
    out.sum_duplicates()
    out.data[:] = 1
    return out


def is_pattern_symmetric(mat) -> bool:
    if mat.shape[0] != mat.shape[1]:
        return False
    pat = _pattern(mat)
    return (pat != pat.T).nnz == 0


def _runs_of(perm: np.ndarray, n: int, target: int) -> np.ndarray:
    """Label the i-th vertex of `perm` with i // target."""
    labels = np.empty(n, dtype=np.int64)
    labels[perm] = np.arange(n, dtype=np.int64) // max(target, 1)
    return labels


def _relabel_consecutive(labels: np.ndarray) -> np.ndarray:
    _, inverse = np.unique(labels, return_inverse=True)
    return inverse.astype(np.int64, copy=False)


def _enforce_caps(labels, row_nnz, max_size, max_nnz):
    """Split groups over the size / nnz caps into consecutive chunks, members in
    ascending vertex order within each group (clustering.py:83-121)."""
    if max_size is None and max_nnz is None:
        return labels
    labels = _relabel_consecutive(labels)
    order = np.argsort(labels, kind='stable')
    sorted_labels = labels[order]
    heads = np.flatnonzero(np.r_[True, sorted_labels[1:] != sorted_labels[:-1]])
    ends = np.r_[heads[1:], sorted_labels.size]
    out = np.empty_like(labels)
    nxt = 0
    for h, e in zip(heads, ends):
        size = 0
        load = 0
        for m in order[h:e]:
            mn = int(row_nnz[m])
            if size > 0 and ((max_size is not None and size + 1 > max_size) or
                             (max_nnz is not None and load + mn > max_nnz)):
                nxt += 1
                size = 0
                load = 0
            out[m] = nxt
            size += 1
            load += mn
        nxt += 1
    return out


def hem_labels_gpu(pat: sp.csr_matrix, target: int, max_size: Optional[int], max_nnz: Optional[int],
                   hub_degree: int = DEFAULT_HUB_DEGREE, topk: Optional[int] = DEFAULT_TOPK,
                   feasible_first: bool = False, residual_rounds: int = 3) -> np.ndarray:
    """HEM labels of the rows of a canonical binary pattern on the current
    CUDA device (spmm_hem_labels); the same labels as the host restatement
    ``_hem.hem_labels`` (before cap enforcement)."""
    from . import _lib
    from ._device import default_device, ptr, stream_handle
    n, m = pat.shape
    if n == 0:
        return np.zeros(0, dtype=np.int64)
    dev = default_device()
    with torch.cuda.device(dev):
        indptr = torch.from_numpy(np.ascontiguousarray(pat.indptr, dtype=np.int64)).to(dev)
        indices = torch.from_numpy(np.ascontiguousarray(pat.indices, dtype=np.int32)).to(dev)
        labels = torch.empty(n, dtype=torch.int64, device=dev)
        rc = _lib.lib().spmm_hem_labels(
            n, m, ptr(indptr), ptr(indices), int(target), -1 if max_size is None else int(max_size),
            -1 if max_nnz is None else int(max_nnz), int(hub_degree), -1 if topk is None else int(topk),
            int(residual_rounds), 1 if feasible_first else 0, ptr(labels), stream_handle(dev))
        _lib.check(rc, 'hem_labels')
        return labels.cpu().numpy()


def cluster_axis(mat, method: str = 'hem', target: int = 32, max_size: Optional[int] = None,
                 max_nnz: Optional[int] = None, seed: int = 0,
                 hub_degree: int = DEFAULT_HUB_DEGREE, topk: Optional[int] = DEFAULT_TOPK,
                 exact_recompute: bool = True, feasible_first: bool = False,
                 hem_hierarchy: Optional[list] = None) -> np.ndarray:
    """int32 group label per ROW of `mat` (pass ``mat.T`` for columns)."""
    if hem_hierarchy is not None and (method != 'hem' or len(hem_hierarchy)):
        raise ValueError('hem_hierarchy must be an empty list with method=hem')
    if method not in CLUSTER_METHODS:
        raise ValueError(f'unknown clustering method {method!r}; expected one of {CLUSTER_METHODS}')
    pat = _pattern(mat)
    n = pat.shape[0]
    row_nnz = np.diff(pat.indptr).astype(np.int64)
    if n == 0:
        if hem_hierarchy is not None:
            hem_hierarchy.append(np.zeros(0, dtype=np.int64))
        return np.zeros(0, dtype=np.int32)
    if method == 'identity':
        labels = np.arange(n, dtype=np.int64) // max(target, 1)
    elif method == 'random':
        labels = _runs_of(np.random.default_rng(seed).permutation(n), n, target)
    elif method == 'degree':
        labels = _runs_of(np.argsort(row_nnz, kind='stable'), n, target)
    elif method == 'rcm':
        if pat.shape[0] != pat.shape[1]:
            raise ValueError("cluster method 'rcm' requires a square matrix")
        from scipy.sparse.csgraph import reverse_cuthill_mckee
        sym = (pat + pat.T).tocsr()
        sym.data[:] = 1
        labels = _runs_of(reverse_cuthill_mckee(sym, symmetric_mode=True).astype(np.int64), n, target)
    elif method == 'graclus':
        raise ImportError("cluster='graclus' requires torch-cluster, which is not installed; "
                          'no HEM fallback is performed')
    elif method == 'metis':
        raise ImportError("cluster='metis' requires pymetis, which is not installed; "
                          'no HEM fallback is performed')
    elif hem_hierarchy is None and exact_recompute and torch.cuda.is_available():
        labels = hem_labels_gpu(pat, target, max_size, max_nnz, hub_degree, topk, feasible_first)
    else:
        from ._hem import hem_labels
        labels = hem_labels(pat, target, max_size, max_nnz, hub_degree, topk, exact_recompute,
                            feasible_first=feasible_first, hierarchy=hem_hierarchy)
    labels = _enforce_caps(labels, row_nnz, max_size, max_nnz)
    return _relabel_consecutive(labels).astype(np.int32)


def cluster_axes(mat, method: str = 'hem', target_nr: int = 32, target_nc: int = 32,
                 max_nr: Optional[int] = None, max_nc: Optional[int] = None,
                 max_block_nnz: Optional[int] = None, seed: int = 0,
                 symmetric: Optional[bool] = None, hub_degree: int = DEFAULT_HUB_DEGREE,
                 topk: Optional[int] = DEFAULT_TOPK, exact_recompute: bool = True,
                 feasible_first: bool = False) -> Tuple[np.ndarray, np.ndarray]:
    """(row_labels, col_labels); one clustering serves both axes when the
    pattern is symmetric and the targets agree (clustering.py:512-545)."""
    csr = sp.csr_matrix(mat)
    if symmetric is None:
        symmetric = (target_nr == target_nc) and is_pattern_symmetric(csr)
    kw = dict(method=method, max_nnz=max_block_nnz, seed=seed, hub_degree=hub_degree, topk=topk,
              exact_recompute=exact_recompute, feasible_first=feasible_first)
    row_labels = cluster_axis(csr, target=target_nr, max_size=max_nr, **kw)
    if symmetric:
        return row_labels, row_labels.copy()
    col_labels = cluster_axis(csr.T.tocsr(), target=target_nc, max_size=max_nc, **kw)
    return row_labels, col_labels
