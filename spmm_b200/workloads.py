"""Seeded synthetic matrices for the five benchmark configurations.

No dataset is downloaded: each generator builds the matrix family the
configuration describes, deterministically from ``seed``, as a canonical
(sorted, duplicate-free) scipy CSR with int32 indices.  ``scale`` shrinks the
problem (grid edge / node count) for tests while keeping its structure.

* ``laplacian2d``  -- C1: 5-point Laplacian on an n x n grid, Dirichlet
  boundary (4 on the diagonal, -1 off it).
* ``fem3d``        -- C2: hex mesh of n^3 nodes x 3 DOF, 27-point node stencil
  expanded to dense 3x3 DOF blocks, values U(-1, 1), diagonal = 1 + sum of the
  row's off-diagonal magnitudes (strictly diagonally dominant).
* ``powerlaw``     -- C3: out-degrees Zipf(2.1) truncated to [1, 20000] and
  rescaled to mean 16, uniform targets, symmetrised (A | A^T), values
  1/sqrt(d_i d_j), random node relabelling.
* ``blockdiag``    -- C4: dense b x b diagonal blocks N(0, 1) plus 0.5% (of the
  block nonzeros) uniformly random off-block entries.
* ``uniform``      -- C5: exactly k distinct uniformly random columns per row,
  values U(-1, 1).
"""

from __future__ import annotations

import numpy as np
import scipy.sparse as sp


def _csr(rows, cols, r, c, v, n_rows, n_cols):
    m = sp.csr_matrix((v, (r, c)), shape=(n_rows, n_cols))
    m.sum_duplicates()
    m.sort_indices()
    m.indptr = m.indptr.astype(np.int32)
    m.indices = m.indices.astype(np.int32)
    return m


def laplacian2d(n: int = 256, dtype=np.float32) -> sp.csr_matrix:
    N = n * n
    idx = np.arange(N, dtype=np.int64)
    x, y = idx % n, idx // n
    rows, cols, vals = [idx], [idx], [np.full(N, 4.0)]
    for dx, dy in ((-1, 0), (1, 0), (0, -1), (0, 1)):
        ok = (x + dx >= 0) & (x + dx < n) & (y + dy >= 0) & (y + dy < n)
        rows.append(idx[ok])
        cols.append(idx[ok] + dx + dy * n)
        vals.append(np.full(int(ok.sum()), -1.0))
    return _csr(None, None, np.concatenate(rows), np.concatenate(cols),
                np.concatenate(vals).astype(dtype), N, N)


def fem3d(n: int = 64, dof: int = 3, seed: int = 0, dtype=np.float32) -> sp.csr_matrix:
    """Rows ordered node-major (node = (z*n + y)*n + x), DOF-minor."""
    rng = np.random.default_rng(seed)
    nodes = n ** 3
    node = np.arange(nodes, dtype=np.int64)
    x, y, z = node % n, (node // n) % n, node // (n * n)
    offs = [(dz, dy, dx) for dz in (-1, 0, 1) for dy in (-1, 0, 1) for dx in (-1, 0, 1)]
    valid = np.zeros((nodes, 27), dtype=bool)
    for o, (dz, dy, dx) in enumerate(offs):
        valid[:, o] = ((x + dx >= 0) & (x + dx < n) & (y + dy >= 0) & (y + dy < n) &
                       (z + dz >= 0) & (z + dz < n))
    off_lin = np.array([dz * n * n + dy * n + dx for dz, dy, dx in offs], dtype=np.int64)
    pn, po = np.nonzero(valid)                    # node-major, offsets ascending -> nbr ascending
    nbr = pn + off_lin[po]
    count = valid.sum(1).astype(np.int64)        # neighbours per node
    # one node's column list: its neighbours' DOFs, ascending
    node_cols = (dof * nbr[:, None] + np.arange(dof)[None, :]).reshape(-1)
    seg_len = dof * count
    seg_start = np.concatenate([[0], np.cumsum(seg_len)[:-1]])
    rows = nodes * dof
    rowlen = np.repeat(seg_len, dof)             # every DOF row of a node shares its columns
    indptr = np.concatenate([[0], np.cumsum(rowlen)]).astype(np.int64)
    total = int(indptr[-1])
    row_of = np.repeat(np.arange(rows, dtype=np.int64), rowlen)
    within = np.arange(total, dtype=np.int64) - indptr[:-1][row_of]
    indices = node_cols[seg_start[row_of // dof] + within]
    del within
    vals = rng.uniform(-1.0, 1.0, size=total)
    diag = indices == row_of
    vals[diag] = 0.0
    absrow = np.add.reduceat(np.abs(vals), indptr[:-1]) if total else np.zeros(rows)
    vals[diag] = 1.0 + absrow
    m = sp.csr_matrix((vals.astype(dtype), indices.astype(np.int32), indptr.astype(np.int32)),
                      shape=(rows, rows))
    m.has_sorted_indices = True
    return m


def powerlaw(n: int = 2_000_000, mean_degree: float = 16.0, exponent: float = 2.1,
             max_degree: int = 20_000, seed: int = 0, dtype=np.float32) -> sp.csr_matrix:
    rng = np.random.default_rng(seed)
    deg = rng.zipf(exponent, size=n).astype(np.float64)
    deg = np.clip(deg, 1, max_degree)
    deg = np.clip(np.rint(deg * (mean_degree / deg.mean())), 1, min(max_degree, n - 1)).astype(np.int64)
    src = np.repeat(np.arange(n, dtype=np.int64), deg)
    dst = rng.integers(0, n, size=src.size, dtype=np.int64)
    keep = src != dst
    src, dst = src[keep], dst[keep]
    a = sp.coo_matrix((np.ones(src.size, dtype=np.float32), (src, dst)), shape=(n, n)).tocsr()
    a = a + a.T
    a.data[:] = 1
    a.sum_duplicates()
    perm = rng.permutation(n)
    a = a[perm][:, perm].tocsr()
    a.sort_indices()
    d = np.diff(a.indptr).astype(np.float64)
    r = np.repeat(np.arange(n), np.diff(a.indptr))
    a.data = (1.0 / np.sqrt(d[r] * d[a.indices])).astype(dtype)
    a.indptr = a.indptr.astype(np.int32)
    a.indices = a.indices.astype(np.int32)
    return a


def blockdiag(n_blocks: int = 4096, b: int = 64, noise: float = 0.005, seed: int = 0,
              dtype=np.float32) -> sp.csr_matrix:
    rng = np.random.default_rng(seed)
    N = n_blocks * b
    blk = np.repeat(np.arange(n_blocks, dtype=np.int64), b * b)
    within = np.tile(np.arange(b * b, dtype=np.int64), n_blocks)
    r = blk * b + within // b
    c = blk * b + within % b
    v = rng.standard_normal(r.size)
    n_noise = int(round(noise * n_blocks * b * b))
    nr = rng.integers(0, N, size=4 * n_noise + 16)
    nc = rng.integers(0, N, size=nr.size)
    off = (nr // b) != (nc // b)
    key = np.unique(nr[off] * N + nc[off])
    key = rng.permutation(key)[:n_noise]
    r = np.concatenate([r, key // N])
    c = np.concatenate([c, key % N])
    v = np.concatenate([v, rng.standard_normal(key.size)])
    return _csr(None, None, r, c, v.astype(dtype), N, N)


def uniform(n: int = 8_388_608, k: int = 8, seed: int = 0, dtype=np.float32) -> sp.csr_matrix:
    """Exactly k distinct columns per row: k draws without replacement per row
    (rejection of in-row repeats)."""
    rng = np.random.default_rng(seed)
    cols = rng.integers(0, n, size=(n, k), dtype=np.int64)
    cols.sort(axis=1)
    while True:
        dup = np.zeros((n, k), dtype=bool)
        dup[:, 1:] = cols[:, 1:] == cols[:, :-1]
        bad = np.flatnonzero(dup.any(axis=1))
        if bad.size == 0:
            break
        redraw = rng.integers(0, n, size=(bad.size, k), dtype=np.int64)
        redraw.sort(axis=1)
        cols[bad] = redraw
    vals = rng.uniform(-1.0, 1.0, size=n * k).astype(dtype)
    indptr = (np.arange(n + 1, dtype=np.int64) * k).astype(np.int32)
    m = sp.csr_matrix((vals, cols.reshape(-1).astype(np.int32), indptr), shape=(n, n))
    m.has_sorted_indices = True
    return m


def dense_x(rows: int, k: int, seed: int = 0, dtype=np.float32, batch: int | None = None):
    """X ~ N(0, 1) from a seeded torch generator, [rows, k] (or [batch, rows, k])."""
    import torch
    g = torch.Generator().manual_seed(seed)
    shape = (rows, k) if batch is None else (batch, rows, k)
    tdt = torch.float32 if np.dtype(dtype) == np.float32 else torch.float64
    return torch.randn(shape, generator=g, dtype=tdt)


# name -> (generator, kwargs at full size, format, BOO target, K)
CONFIGS = {
    'c1_laplacian2d': dict(gen=laplacian2d, kw=dict(n=256), fmt='boo', target=32, K=128),
    'c2_fem3d': dict(gen=fem3d, kw=dict(n=64), fmt='boo', target=32, K=128),
    'c3_powerlaw': dict(gen=powerlaw, kw=dict(n=2_000_000), fmt='boo', target=32, K=256),
    'c4_blockdiag': dict(gen=blockdiag, kw=dict(n_blocks=4096, b=64), fmt='boo', target=64, K=512),
    'c5_uniform': dict(gen=uniform, kw=dict(n=8_388_608), fmt='pbr', target=32, K=64),
}
