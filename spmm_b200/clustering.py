"""Row / column grouping labels for the BOO format.

``csr_to_boo`` takes one int32 group label per row and per column.  This
module produces them with the methods the reference offers
(``torch_fast_spdmm/torch_fast_spdmm/clustering.py``: ``cluster_axis``
:454-509, ``cluster_axes`` :512-545):

* ``identity`` -- consecutive runs of ``target`` rows;
* ``random`` / ``degree`` -- runs of a seeded permutation / of the rows
  sorted by nonzero count (stable);
* ``rcm`` -- runs of the reverse Cuthill-McKee order of the symmetrised
  pattern (square matrices);
* ``hem`` -- multilevel heavy-edge matching, computed on the GPU
  (``spmm_hem_labels`` / ``spmm_hem_hierarchy``; there is no host
  implementation in the product -- ``oracle/hem_oracle.c`` is its checker);
* ``graclus`` / ``metis`` need packages this image lacks and raise
  ``ImportError`` (the reference does not fall back either).

Every method's labels then go through the reference's cap enforcement
(groups split into pieces of at most ``max_size`` members / ``max_nnz`` row
nonzeros, members taken in ascending index order) and are renumbered
consecutively in ascending label order.
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


def _pattern(mat) -> sp.csr_matrix:
    """Canonical binary CSR of the sparsity pattern: each (row, col) that
    appears at least once, columns ascending, value 1 (int32).  A canonical
    input (sorted, no duplicates) is used as it is; others are canonicalised
    first."""
    a = sp.csr_matrix(mat)
    if not a.has_canonical_format:
        a = a.copy()
        a.sum_duplicates()             # sorts each row and merges repeats
    return sp.csr_matrix((np.ones(a.nnz, dtype=np.int32), a.indices, a.indptr), shape=a.shape)


def is_pattern_symmetric(mat) -> bool:
    """True for a square matrix whose (row, col) set equals its transpose's."""
    n, m = mat.shape
    if n != m:
        return False
    p = _pattern(mat)
    t = p.T.tocsr()                    # canonical: the transpose's rows come out sorted
    t.sort_indices()
    return np.array_equal(p.indptr, t.indptr) and np.array_equal(p.indices, t.indices)


def _runs_of(perm: np.ndarray, target: int) -> np.ndarray:
    """Vertex perm[i] gets label i // target."""
    labels = np.empty(perm.size, dtype=np.int64)
    labels[perm] = np.arange(perm.size, dtype=np.int64) // max(target, 1)
    return labels


def _dense_rank(labels: np.ndarray) -> np.ndarray:
    """Labels renumbered 0, 1, ... in ascending label order (labels are
    nonnegative; a presence count when they are bounded by the member count,
    as every method's are, else a sort)."""
    if labels.size and 0 <= labels.min() and labels.max() < 4 * labels.size:
        present = np.bincount(labels, minlength=1) > 0
        rank = np.cumsum(present) - 1
        return rank[labels].astype(np.int64)
    u = np.unique(labels)
    return np.searchsorted(u, labels).astype(np.int64)


def _enforce_caps(labels: np.ndarray, row_nnz: Optional[np.ndarray], max_size: Optional[int],
                  max_nnz: Optional[int]) -> np.ndarray:
    """Split every group into pieces that respect the caps.

    Inside a group, members are taken in ascending index order; a member
    starts a new piece when adding it would exceed ``max_size`` members or
    ``max_nnz`` row nonzeros (a piece holds at least one member).  Pieces are
    numbered by (group label, piece order).  Vectorised over groups: one pass
    per member position, so the loop runs as many times as the largest group
    has members.
    """
    if max_size is None and max_nnz is None:
        return labels
    if max_nnz is None and labels.size and labels.max() < 4 * labels.size \
            and np.bincount(labels).max() <= max_size:
        return labels                                  # no group over the size cap
    n = labels.size
    order = np.lexsort((np.arange(n), labels))          # by group, members ascending
    g = labels[order]
    heads = np.flatnonzero(np.r_[True, g[1:] != g[:-1]])
    glen = np.diff(np.r_[heads, n])
    piece = np.zeros(n, dtype=np.int64)                # piece index inside its group, sorted order
    if max_nnz is None:                                # size cap alone: fixed-size pieces
        pos = np.arange(n) - np.repeat(heads, glen)
        piece = pos // max(int(max_size), 1)
    else:
        nz = np.asarray(row_nnz, dtype=np.int64)[order]
        cur = np.zeros(heads.size, dtype=np.int64)     # per group: current piece, members, load
        cnt = np.ones(heads.size, dtype=np.int64)
        load = nz[heads].copy()
        live = np.arange(heads.size)
        for k in range(1, int(glen.max())):
            live = live[glen[live] > k]
            at = heads[live] + k
            add = nz[at]
            brk = load[live] + add > max_nnz
            if max_size is not None:
                brk |= cnt[live] + 1 > max_size
            cur[live] += brk
            cnt[live] = np.where(brk, 1, cnt[live] + 1)
            load[live] = np.where(brk, add, load[live] + add)
            piece[at] = cur[live]
    npieces = np.maximum.reduceat(piece, heads) + 1
    first = np.r_[0, np.cumsum(npieces)[:-1]]
    out = np.empty(n, dtype=np.int64)
    out[order] = np.repeat(first, glen) + piece
    return out


_COUNT_METHODS = ('identity', 'random', 'degree')


def _axis_nnz(csr: sp.csr_matrix, axis: int) -> np.ndarray:
    """Distinct nonzero columns per row (axis 0) or rows per column (axis 1)."""
    a = csr if csr.has_canonical_format else _pattern(csr)
    return np.diff(a.indptr) if axis == 0 else np.bincount(a.indices, minlength=a.shape[1])


def _count_labels(method: str, n: int, counts, target: int, max_size: Optional[int],
                  max_nnz: Optional[int], seed: int) -> np.ndarray:
    """Labels of the methods that need only the members' nonzero counts;
    `counts()` gives them and is called only when needed (degree order, or
    a nonzero cap)."""
    if n == 0:
        return np.zeros(0, dtype=np.int32)
    row_nnz = counts() if method == 'degree' or max_nnz is not None else None
    if method == 'identity':
        labels = np.arange(n, dtype=np.int64) // max(target, 1)
    elif method == 'random':
        labels = _runs_of(np.random.default_rng(seed).permutation(n), target)
    else:
        labels = _runs_of(np.argsort(row_nnz, kind='stable'), target)
    return _dense_rank(_enforce_caps(labels, row_nnz, max_size, max_nnz)).astype(np.int32)


def hem_labels_gpu(pat: sp.csr_matrix, target: int, max_size: Optional[int], max_nnz: Optional[int],
                   hub_degree: int = DEFAULT_HUB_DEGREE, topk: Optional[int] = DEFAULT_TOPK,
                   feasible_first: bool = False, residual_rounds: int = 3,
                   hierarchy: Optional[list] = None) -> np.ndarray:
    """HEM labels of the rows of a canonical binary pattern, before cap
    enforcement, on the current CUDA device (the reference's _hem_labels,
    clustering.py:271-351).  With ``hierarchy`` (a list), the identity labels
    and the labels after each level that matched are appended to it."""
    import ctypes as C

    from . import _lib
    from ._device import default_device, ptr, stream_handle, to_device
    if not torch.cuda.is_available():
        raise RuntimeError("cluster='hem' runs on the GPU (spmm_hem_labels); no CUDA device is available")
    n, m = pat.shape
    if n == 0:
        if hierarchy is not None:
            hierarchy.append(np.zeros(0, dtype=np.int64))
        return np.zeros(0, dtype=np.int64)
    L = _lib.lib()
    dev = default_device()
    with torch.cuda.device(dev):
        indptr = to_device(pat.indptr, dev, np.int64)
        indices = to_device(pat.indices, dev, np.int32)
        labels = torch.empty(n, dtype=torch.int64, device=dev)
        slots = int(L.spmm_hem_level_slots(int(target))) if hierarchy is not None else 0
        levels = torch.empty((slots, n), dtype=torch.int64, device=dev) if slots else None
        nlev = C.c_int64(0)
        rc = L.spmm_hem_hierarchy(
            n, m, ptr(indptr), ptr(indices), int(target), -1 if max_size is None else int(max_size),
            -1 if max_nnz is None else int(max_nnz), int(hub_degree), -1 if topk is None else int(topk),
            int(residual_rounds), 1 if feasible_first else 0, ptr(labels),
            ptr(levels) if levels is not None else None, slots, C.byref(nlev), stream_handle(dev))
        _lib.check(rc, 'hem_labels')
        if hierarchy is not None:
            hierarchy.extend(list(levels[:nlev.value].cpu().numpy()))
        return labels.cpu().numpy()


def cluster_axis(mat, method: str = 'hem', target: int = 32, max_size: Optional[int] = None,
                 max_nnz: Optional[int] = None, seed: int = 0,
                 hub_degree: int = DEFAULT_HUB_DEGREE, topk: Optional[int] = DEFAULT_TOPK,
                 exact_recompute: bool = True, feasible_first: bool = False,
                 hem_hierarchy: Optional[list] = None) -> np.ndarray:
    """int32 group label per ROW of `mat` (pass ``mat.T`` for columns).

    ``exact_recompute`` is accepted and always honoured as True: the similarity
    graph is rebuilt from the contracted pattern at every level (the reference
    with False reuses the first level's graph after contraction and raises
    IndexError as soon as a level has matched)."""
    if hem_hierarchy is not None and (method != 'hem' or len(hem_hierarchy)):
        raise ValueError('hem_hierarchy must be an empty list with method=hem')
    if method not in CLUSTER_METHODS:
        raise ValueError(f'unknown clustering method {method!r}; expected one of {CLUSTER_METHODS}')
    if method == 'graclus':
        raise ImportError("cluster='graclus' requires torch-cluster, which is not installed; "
                          'no HEM fallback is performed')
    if method == 'metis':
        raise ImportError("cluster='metis' requires pymetis, which is not installed; "
                          'no HEM fallback is performed')
    if method in _COUNT_METHODS:
        csr = sp.csr_matrix(mat)
        return _count_labels(method, csr.shape[0], lambda: _axis_nnz(csr, 0), target, max_size, max_nnz, seed)
    pat = _pattern(mat)
    n = pat.shape[0]
    if n == 0:
        if hem_hierarchy is not None:
            hem_hierarchy.append(np.zeros(0, dtype=np.int64))
        return np.zeros(0, dtype=np.int32)
    row_nnz = np.diff(pat.indptr)
    if method == 'rcm':
        if pat.shape[0] != pat.shape[1]:
            raise ValueError("cluster method 'rcm' requires a square matrix")
        from scipy.sparse.csgraph import reverse_cuthill_mckee
        both = (pat + pat.T).tocsr()
        both.data[:] = 1
        labels = _runs_of(reverse_cuthill_mckee(both, symmetric_mode=True).astype(np.int64), target)
    else:
        labels = hem_labels_gpu(pat, target, max_size, max_nnz, hub_degree, topk, feasible_first,
                                hierarchy=hem_hierarchy)
    return _dense_rank(_enforce_caps(labels, row_nnz, max_size, max_nnz)).astype(np.int32)


def cluster_axes(mat, method: str = 'hem', target_nr: int = 32, target_nc: int = 32,
                 max_nr: Optional[int] = None, max_nc: Optional[int] = None,
                 max_block_nnz: Optional[int] = None, seed: int = 0,
                 symmetric: Optional[bool] = None, hub_degree: int = DEFAULT_HUB_DEGREE,
                 topk: Optional[int] = DEFAULT_TOPK, exact_recompute: bool = True,
                 feasible_first: bool = False) -> Tuple[np.ndarray, np.ndarray]:
    """(row_labels, col_labels).  A square matrix with a symmetric pattern and
    equal targets is a graph: its vertex clustering serves both axes;
    otherwise rows and columns (the transpose's rows) are clustered apart.
    ``symmetric`` overrides the detection."""
    csr = sp.csr_matrix(mat)
    if method in _COUNT_METHODS:
        # These labels depend on each axis's member count and nonzero counts
        # only: a symmetric pattern gives equal row and column counts, so the
        # columns' own labels equal the rows' and no symmetry test is needed.
        rows = _count_labels(method, csr.shape[0], lambda: _axis_nnz(csr, 0), target_nr, max_nr, max_block_nnz,
                             seed)
        if symmetric:
            return rows, rows.copy()
        return rows, _count_labels(method, csr.shape[1], lambda: _axis_nnz(csr, 1), target_nc, max_nc,
                                   max_block_nnz, seed)
    if symmetric is None:
        symmetric = target_nr == target_nc and is_pattern_symmetric(csr)
    common = dict(method=method, max_nnz=max_block_nnz, seed=seed, hub_degree=hub_degree, topk=topk,
                  exact_recompute=exact_recompute, feasible_first=feasible_first)
    rows = cluster_axis(csr, target=target_nr, max_size=max_nr, **common)
    if symmetric:
        return rows, rows.copy()
    return rows, cluster_axis(csr.T.tocsr(), target=target_nc, max_size=max_nc, **common)
