"""Multilevel heavy-edge matching (HEM) labels -- the reference's default BOO
clustering (torch_fast_spdmm/torch_fast_spdmm/clustering.py:128-351),
restated.

Vertices are the rows of a binary pattern P.  Edge weight between rows i and j
is their shared-column count (P P^T), after dropping hub columns (degree >
``hub_degree``) and keeping each row's ``topk`` heaviest edges (ties by column
id), then symmetrising with max (:128-185).  A level matches vertices by
mutual-max ("locally dominant") pairs -- each vertex picks its heaviest live
edge, ties broken by a symmetric splitmix64 hash of the vertex pair, and
mutual picks are merged if the merged size / nnz respect the caps (:188-268);
up to ``residual_rounds`` matching rounds per level; the coarse graph is
recomputed from the contracted pattern (support union) each level, until a
level matches nothing (:271-351).  No randomness anywhere.
"""

from __future__ import annotations

from typing import Optional

import numpy as np
import scipy.sparse as sp

_M1 = np.uint64(0x9E3779B97F4A7C15)   # splitmix64 / golden-ratio increment
_M2 = np.uint64(0xC2B2AE3D27D4EB4F)
_F1 = np.uint64(0xBF58476D1CE4E5B9)   # splitmix64 finaliser multipliers
_F2 = np.uint64(0x94D049BB133111EB)


def pair_hash(a: np.ndarray, b: np.ndarray) -> np.ndarray:
    """Symmetric 63-bit hash of the unordered pair {a, b} (splitmix64 mix)."""
    lo = np.minimum(a, b).astype(np.uint64)
    hi = np.maximum(a, b).astype(np.uint64)
    with np.errstate(over='ignore'):
        h = (lo * _M1) ^ (hi * _M2)
        h ^= h >> np.uint64(30)
        h *= _F1
        h ^= h >> np.uint64(27)
        h *= _F2
        h ^= h >> np.uint64(31)
    return (h >> np.uint64(1)).astype(np.int64)


def similarity_graph(pat: sp.csr_matrix, hub_degree: int, topk: Optional[int],
                     chunk_rows: int = 4096) -> sp.csr_matrix:
    n, m = pat.shape
    if n <= 1:
        return sp.csr_matrix((n, n), dtype=np.int64)
    col_deg = np.bincount(pat.indices, minlength=m)
    keep = col_deg <= hub_degree
    if keep.all():
        pruned = sp.csr_matrix((pat.data.astype(np.int64), pat.indices, pat.indptr), shape=pat.shape)
    else:
        sel = keep[pat.indices]
        owner = np.repeat(np.arange(n), np.diff(pat.indptr))
        per_row = np.bincount(owner[sel], minlength=n)
        pruned = sp.csr_matrix((pat.data[sel].astype(np.int64), pat.indices[sel],
                                np.r_[0, np.cumsum(per_row)]), shape=pat.shape)
    pt = pruned.T.tocsr()
    rr, cc, dd = [], [], []
    for s in range(0, n, chunk_rows):
        e = min(s + chunk_rows, n)
        blk = (pruned[s:e] @ pt).tocoo()
        if blk.nnz == 0:
            continue
        r, c, d = blk.row, blk.col, blk.data
        off = c != r + s
        r, c, d = r[off], c[off], d[off]
        if topk is not None and r.size:
            o = np.lexsort((c, -d, r))          # row asc, weight desc, col asc
            rs = r[o]
            first = np.searchsorted(rs, np.arange(e - s))
            rank = np.arange(rs.size) - first[rs]
            o = o[rank < topk]
            r, c, d = r[o], c[o], d[o]
        rr.append(r + s)
        cc.append(c)
        dd.append(d)
    if not rr:
        return sp.csr_matrix((n, n), dtype=np.int64)
    g = sp.coo_matrix((np.concatenate(dd), (np.concatenate(rr), np.concatenate(cc))),
                      shape=(n, n)).tocsr()
    g.sum_duplicates()
    return g.maximum(g.T)


def mutual_max_pairs(graph: sp.csr_matrix, active, size, nnz, max_size, max_nnz,
                     feasible_first: bool = False):
    n = graph.shape[0]
    coo = graph.tocoo()
    empty = (np.empty(0, np.int64), np.empty(0, np.int64))
    if coo.nnz == 0:
        return empty
    live = active[coo.row] & active[coo.col]
    if feasible_first:
        if max_size is not None:
            live &= (size[coo.row] + size[coo.col]) <= max_size
        if max_nnz is not None:
            live &= (nnz[coo.row] + nnz[coo.col]) <= max_nnz
    r, c, d = coo.row[live], coo.col[live], coo.data[live]
    if r.size == 0:
        return empty
    o = np.lexsort((-pair_hash(r, c), -d, r))   # row asc, weight desc, hash desc
    r, c = r[o], c[o]
    head = np.flatnonzero(np.r_[True, r[1:] != r[:-1]])
    best = np.full(n, -1, dtype=np.int64)
    best[r[head]] = c[head]
    idx = np.arange(n, dtype=np.int64)
    partner = np.where(best >= 0, best, idx)
    mutual = (best >= 0) & (best[partner] == idx)
    left = idx[mutual & (idx < partner)]
    right = partner[left]
    if left.size == 0:
        return left, right
    ok = np.ones(left.size, dtype=bool)
    if max_size is not None:
        ok &= (size[left] + size[right]) <= max_size
    if max_nnz is not None:
        ok &= (nnz[left] + nnz[right]) <= max_nnz
    return left[ok], right[ok]


def hem_labels(pat: sp.csr_matrix, target: int, max_size, max_nnz, hub_degree: int,
               topk: Optional[int], exact_recompute: bool = True, residual_rounds: int = 3,
               feasible_first: bool = False, hierarchy: Optional[list] = None) -> np.ndarray:
    n = pat.shape[0]
    labels = np.arange(n, dtype=np.int64)
    if hierarchy is not None:
        hierarchy.append(labels.copy())
    if n <= 1 or target <= 1:
        return labels
    size = np.ones(n, dtype=np.int64)
    nnz = np.diff(pat.indptr).astype(np.int64)
    level_pat = pat
    graph = None
    max_levels = 8 * max(1, int(np.ceil(np.log2(target)))) + 16
    for _ in range(max_levels):
        n_cur = level_pat.shape[0]
        if n_cur <= 1:
            break
        if exact_recompute or graph is None:
            graph = similarity_graph(level_pat, hub_degree, topk)
        if graph.nnz == 0:
            break
        active = np.ones(n_cur, dtype=bool)
        lefts, rights = [], []
        for _round in range(residual_rounds):
            left, right = mutual_max_pairs(graph, active, size, nnz, max_size, max_nnz,
                                           feasible_first)
            if left.size == 0:
                break
            lefts.append(left)
            rights.append(right)
            active[left] = False
            active[right] = False
        if not lefts:
            break
        left = np.concatenate(lefts)
        right = np.concatenate(rights)
        parent = np.arange(n_cur, dtype=np.int64)
        parent[right] = left
        roots = np.flatnonzero(parent == np.arange(n_cur))
        remap = np.full(n_cur, -1, dtype=np.int64)
        remap[roots] = np.arange(roots.size, dtype=np.int64)
        new_id = remap[parent]
        n_new = roots.size
        size = np.bincount(new_id, weights=size, minlength=n_new).astype(np.int64)
        nnz = np.bincount(new_id, weights=nnz, minlength=n_new).astype(np.int64)
        labels = new_id[labels]
        if hierarchy is not None:
            hierarchy.append(labels.copy())
        contract = sp.csr_matrix((np.ones(n_cur, dtype=np.int64), (new_id, np.arange(n_cur))),
                                 shape=(n_new, n_cur))
        level_pat = contract @ level_pat
        level_pat.data[:] = 1
        graph = None if exact_recompute else graph
    return labels
