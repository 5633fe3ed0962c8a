"""Multi-GPU SpMM: one process per GPU, ``torch.distributed`` for the plumbing.

The reference runs on one GPU; the product shards naturally, in two ways, and
neither needs a device-side remote load or a multicast:

* **feature split** -- A replicated, X / Y split by feature columns.  The
  format is built once on the source rank and broadcast array by array
  (:func:`broadcast_boo`); every rank multiplies its own slab of X columns, so
  the product has no collective.  Suits large K with a small A (C2, C4).
* **row split** -- BOO row groups or PBR stripes (``block_rows`` consecutive
  rows) partitioned by nonzero balance (a prefix over the per-group
  nonzeros, :func:`nnz_balanced_splits`).  Every rank builds the format of
  its own rows with global column ids (:class:`RowSplitBOO`,
  :class:`RowSplitPBR`), X reaches every rank once by a broadcast into local
  HBM (:func:`broadcast_dense`), and Y shards stay local; ``gather`` assembles
  a replicated Y when a caller wants one.  Suits random gathers with a large
  A (C3, C5).

Planning is host-side numpy, so the partition logic and the collectives are
tested with ``gloo`` ranks on CPU; products need CUDA.  Process groups get a
short timeout (:func:`init`), so a rank that dies makes the others' next
collective fail instead of hanging; every collective of this module turns
such a failure into ``SpmmError(SPMM_ENCCL)`` (a ``RuntimeError``).
"""

from __future__ import annotations

import dataclasses
import datetime
import os
import types
from typing import List, Optional

import numpy as np
import torch
import torch.distributed as dist

from . import _lib
from . import boo as _boo
from . import pbr as _pbr

DEFAULT_TIMEOUT_S = 60


def _collective(what: str, fn, *args, **kw):
    """Runs one torch.distributed collective; a failure (a peer that died, a
    timeout, a backend error) becomes SpmmError(SPMM_ENCCL)."""
    try:
        return fn(*args, **kw)
    except _lib.SpmmError:
        raise
    except (RuntimeError, ValueError) as e:
        raise _lib.SpmmError(_lib.SPMM_ENCCL, f'{what} ({type(e).__name__}: {str(e)[:200]})') from e


def barrier() -> None:
    _collective('barrier', dist.barrier)


def all_reduce_max(value: float, device) -> float:
    """max of `value` over ranks (the bench's step time)."""
    t = torch.tensor([float(value)], dtype=torch.float64, device=device)
    _collective('all_reduce', dist.all_reduce, t, op=dist.ReduceOp.MAX)
    return float(t.item())


def init(backend: Optional[str] = None, timeout_s: float = DEFAULT_TIMEOUT_S,
         device: Optional[torch.device] = None) -> None:
    """init_process_group from the torchrun environment with a bounded
    timeout (collectives waiting on a dead rank fail after `timeout_s`)."""
    if dist.is_initialized():
        return
    if backend is None:
        backend = 'nccl' if torch.cuda.is_available() else 'gloo'
    kw = dict(backend=backend, timeout=datetime.timedelta(seconds=timeout_s))
    if backend == 'nccl' and device is not None:
        kw['device_id'] = device
    dist.init_process_group(**kw)


# ---------------------------------------------------------------------------
# partition planning (host)
# ---------------------------------------------------------------------------

def nnz_balanced_splits(group_nnz: np.ndarray, parts: int) -> np.ndarray:
    """Boundaries b[0] = 0 <= b[1] <= ... <= b[parts] = len(group_nnz) of
    contiguous group ranges whose nonzero counts are as close as possible to
    total / parts: b[k] is the prefix end nearest the k-th target."""
    if parts < 1:
        raise ValueError('parts must be >= 1')
    g = np.asarray(group_nnz, dtype=np.int64)
    n = g.size
    cum = np.concatenate([[0], np.cumsum(g)])
    total = int(cum[-1])
    b = np.zeros(parts + 1, dtype=np.int64)
    b[parts] = n
    for k in range(1, parts):
        target = total * k / parts
        i = int(np.searchsorted(cum, target, side='left'))   # cum[i] >= target
        if i > 0 and abs(cum[i - 1] - target) <= abs(cum[min(i, n)] - target):
            i -= 1
        b[k] = min(max(i, b[k - 1]), n)
    return b


@dataclasses.dataclass
class RowShard:
    """Rows of one rank: row groups [g0, g1) of the global labelling."""
    rank: int
    g0: int
    g1: int
    rows: np.ndarray          # global row ids, ascending
    local_labels: np.ndarray  # row label within the shard (global label - g0)
    nnz: int


def stripe_labels(rows: int, block_rows: int) -> np.ndarray:
    """PBR stripe of every row (row // block_rows): the row-split unit of a
    PBR matrix, so every shard starts on a stripe boundary."""
    return np.arange(rows, dtype=np.int64) // max(int(block_rows), 1)


def plan_row_split(indptr: np.ndarray, row_labels: np.ndarray, parts: int) -> List[RowShard]:
    """Partition the row groups of `row_labels` (one label per row) into
    `parts` contiguous label ranges of balanced nonzeros."""
    indptr = np.asarray(indptr, dtype=np.int64)
    labels = np.asarray(row_labels, dtype=np.int64)
    if labels.size != indptr.size - 1:
        raise ValueError('row_labels must have one entry per row')
    if labels.size and labels.min() < 0:
        raise ValueError('row labels must be non-negative')
    n_groups = int(labels.max()) + 1 if labels.size else 0
    row_nnz = np.diff(indptr)
    gnnz = np.bincount(labels, weights=row_nnz, minlength=n_groups).astype(np.int64)
    bounds = nnz_balanced_splits(gnnz, parts)
    shards = []
    for r in range(parts):
        g0, g1 = int(bounds[r]), int(bounds[r + 1])
        rows = np.nonzero((labels >= g0) & (labels < g1))[0]
        shards.append(RowShard(r, g0, g1, rows, labels[rows] - g0, int(row_nnz[rows].sum())))
    return shards


def shard_csr(mat, shard: RowShard):
    """The shard's rows of a scipy CSR matrix (global column ids kept)."""
    sub = mat[shard.rows]
    sub.indptr = sub.indptr.astype(mat.indptr.dtype, copy=False)
    sub.indices = sub.indices.astype(mat.indices.dtype, copy=False)
    return sub


# ---------------------------------------------------------------------------
# collectives
# ---------------------------------------------------------------------------

def broadcast_dense(x: Optional[torch.Tensor], shape, dtype, device, src: int = 0) -> torch.Tensor:
    """X from `src` into every rank's memory on `device` (one broadcast).
    Ranks other than `src` pass x=None and the shape / dtype to allocate."""
    if dist.get_rank() == src:
        out = x.to(device).contiguous()
    else:
        out = torch.empty(tuple(shape), dtype=dtype, device=device)
    _collective('broadcast', dist.broadcast, out, src)
    return out


_BOO_SIZE_KEYS = ('rows', 'cols', 'total_nnz', 'n_rg', 'n_cg', 'nb', 'nnz_c', 'rem_nnz', 'tail_nnz',
                  'max_nr', 'max_nc', 'max_nnz_blk', 'nz_order')


def _boo_lengths(sz: dict) -> dict:
    return {'row_grp_ptr': sz['n_rg'] + 1, 'row_ids': sz['rows'], 'col_grp_ptr': sz['n_cg'] + 1,
            'col_ids': sz['cols'], 'blk_row_grp': sz['nb'], 'blk_col_grp': sz['nb'],
            'blk_nz_ptr': sz['nb'] + 1, 'blk_shift': sz['nb'], 'nz_idx': sz['nnz_c'],
            'nz_val': sz['nnz_c'], 'rem_indptr': sz['rows'] + 1, 'rem_col_ind': sz['rem_nnz'],
            'rem_vals': sz['rem_nnz'], 'tail_row': sz['tail_nnz'], 'tail_col': sz['tail_nnz'],
            'tail_val': sz['tail_nnz']}


def broadcast_boo(mat: Optional['_boo._BOOMatrix'], device, src: int = 0):
    """A BOO matrix built on rank `src` replicated on every rank's `device`:
    sizes first, then each staged array (the feature split's A staging)."""
    rank = dist.get_rank()
    meta = torch.zeros(len(_BOO_SIZE_KEYS) + 2, dtype=torch.int64, device=device)
    if rank == src:
        d = mat._gpu_meta if mat._gpu_meta is not None else mat._dev
        vals = [mat._sizes[k] for k in _BOO_SIZE_KEYS]
        vals += [0 if mat._index_dtype == np.int32 else 1, 0 if mat._scalar_dtype == np.float32 else 1]
        meta.copy_(torch.tensor(vals, dtype=torch.int64))
    _collective('broadcast', dist.broadcast, meta, src)
    m = [int(v) for v in meta.cpu()]
    sizes = dict(zip(_BOO_SIZE_KEYS, m[:len(_BOO_SIZE_KEYS)]))
    idt = np.int32 if m[-2] == 0 else np.int64
    sdt = np.float32 if m[-1] == 0 else np.float64
    tsdt = torch.float32 if sdt == np.float32 else torch.float64
    lengths = _boo_lengths(sizes)
    arrays = {}
    for name, tdt in _boo._DEV_DTYPES.items():
        dt = tsdt if tdt is None else tdt
        if rank == src:
            t = getattr(d, name).to(device).contiguous()
        else:
            t = torch.empty(lengths[name], dtype=dt, device=device)
        if t.numel():
            _collective('broadcast', dist.broadcast, t.view(torch.uint8), src)   # bytes: no int16 collectives
        arrays[name] = t
    cls = _boo._boo_class(idt, sdt)
    out = cls(sizes, types.SimpleNamespace(**arrays))
    if torch.device(device).type == 'cuda':
        out._gpu_meta = out._dev
    return out


_PBR_SIZE_KEYS = ('rows', 'cols', 'block_rows', 'block_cols', 'total_nnz', 'nb', 'nnz_c', 'rem_nnz')
_PBR_ARRAYS = ('codes', 'coords', 'offsets', 'data', 'rem_indptr', 'rem_col_ind', 'rem_vals')


def _pbr_lengths(sz: dict) -> dict:
    return {'codes': sz['nb'], 'coords': 2 * sz['nb'], 'offsets': sz['nb'] + 1, 'data': sz['nnz_c'],
            'rem_indptr': sz['rows'] + 1, 'rem_col_ind': sz['rem_nnz'], 'rem_vals': sz['rem_nnz']}


def broadcast_pbr(mat: Optional['_pbr._PBRMatrix'], device, src: int = 0):
    """A PBR matrix built on rank `src` replicated on every rank's `device`
    (the feature split's A staging for the PBR format)."""
    rank = dist.get_rank()
    meta = torch.zeros(len(_PBR_SIZE_KEYS) + 2, dtype=torch.int64, device=device)
    if rank == src:
        d = mat._gpu_meta if mat._gpu_meta is not None else mat._dev
        vals = [mat._sizes[k] for k in _PBR_SIZE_KEYS]
        vals += [0 if d.coords.dtype == torch.int32 else 1, 0 if mat._scalar_dtype == np.float32 else 1]
        meta.copy_(torch.tensor(vals, dtype=torch.int64))
    _collective('broadcast', dist.broadcast, meta, src)
    m = [int(v) for v in meta.cpu()]
    sizes = dict(zip(_PBR_SIZE_KEYS, m[:len(_PBR_SIZE_KEYS)]))
    tidt = torch.int32 if m[-2] == 0 else torch.int64
    tsdt = torch.float32 if m[-1] == 0 else torch.float64
    dtypes = {'codes': torch.int64, 'coords': tidt, 'offsets': tidt, 'data': tsdt, 'rem_indptr': tidt,
              'rem_col_ind': tidt, 'rem_vals': tsdt}
    lengths = _pbr_lengths(sizes)
    arrays = {}
    for name in _PBR_ARRAYS:
        if rank == src:
            t = getattr(d, name).to(device).contiguous()
        else:
            t = torch.empty(lengths[name], dtype=dtypes[name], device=device)
        if t.numel():
            _collective('broadcast', dist.broadcast, t.view(torch.uint8), src)
        arrays[name] = t
    cls = _pbr._pbr_class(np.int32 if m[-2] == 0 else np.int64, np.float32 if m[-1] == 0 else np.float64)
    out = cls(sizes, types.SimpleNamespace(**arrays))
    if torch.device(device).type == 'cuda':
        out._gpu_meta = out._dev
    return out


# ---------------------------------------------------------------------------
# row split
# ---------------------------------------------------------------------------

class RowSplitBOO:
    """This rank's share of a row-split BOO product.

    Every rank passes the same CSR matrix and labels (or rebuilds them from
    the same seed); each builds the BOO format of its own row groups with
    global column ids on its GPU.  ``matmul(x)`` takes the full X resident on
    this rank (see :func:`broadcast_dense`) and returns the Y rows of the
    shard, in ``self.shard.rows`` order."""

    def __init__(self, mat, row_labels, col_labels, device, rank: Optional[int] = None,
                 world: Optional[int] = None, **boo_kw):
        rank = dist.get_rank() if rank is None else rank
        world = dist.get_world_size() if world is None else world
        self.shards = plan_row_split(mat.indptr, row_labels, world)
        self.shard = self.shards[rank]
        self.rows_total = mat.shape[0]
        sub = shard_csr(mat, self.shard)
        self.boo = _boo.csr_to_boo(sub, row_labels=self.shard.local_labels, col_labels=col_labels,
                                   **boo_kw).to(device)
        self.device = torch.device(device)

    def matmul(self, x: torch.Tensor, **kw) -> torch.Tensor:
        return _boo.boo_matmul(self.boo, x, **kw)

    def gather(self, y_local: torch.Tensor) -> torch.Tensor:
        """Replicated Y [rows_total, K] from every rank's shard."""
        return gather_rows(y_local, self.shards, self.rows_total)


class RowSplitPBR:
    """This rank's share of a row-split PBR product: stripes of
    ``block_rows`` rows partitioned by nonzero balance, so every shard starts
    on a stripe boundary and its blocks are the global matrix's blocks of
    those stripes (same codes, coordinates shifted by the shard's first row).
    ``matmul(x)`` takes the full X on this rank and returns the shard's Y
    rows (``self.shard.rows``, ascending and contiguous)."""

    def __init__(self, mat, block_rows: int, block_cols: int, min_nnz_per_block: int, device,
                 rank: Optional[int] = None, world: Optional[int] = None):
        rank = dist.get_rank() if rank is None else rank
        world = dist.get_world_size() if world is None else world
        self.shards = plan_row_split(mat.indptr, stripe_labels(mat.shape[0], block_rows), world)
        self.shard = self.shards[rank]
        self.rows_total = mat.shape[0]
        sub = shard_csr(mat, self.shard)
        self.pbr = _pbr.csr_to_pbr(sub, block_rows, block_cols, min_nnz_per_block).to(device)
        self.device = torch.device(device)

    def matmul(self, x: torch.Tensor, **kw) -> torch.Tensor:
        return _pbr.pbr_matmul(self.pbr, x, **kw)

    def gather(self, y_local: torch.Tensor) -> torch.Tensor:
        return gather_rows(y_local, self.shards, self.rows_total)


def gather_rows(y_local: torch.Tensor, shards: List[RowShard], rows_total: int) -> torch.Tensor:
    """Y [rows_total, K] on every rank from the row shards (all_gather of
    equal-size padded shards, then a scatter by global row id)."""
    world = dist.get_world_size()
    K = y_local.shape[-1]
    width = max(len(s.rows) for s in shards)
    pad = torch.zeros((width, K), dtype=y_local.dtype, device=y_local.device)
    pad[:y_local.shape[0]] = y_local
    parts = [torch.empty_like(pad) for _ in range(world)]
    _collective('all_gather', dist.all_gather, parts, pad)
    y = torch.empty((rows_total, K), dtype=y_local.dtype, device=y_local.device)
    for s, part in zip(shards, parts):
        idx = torch.from_numpy(s.rows).to(y.device)
        y.index_copy_(0, idx, part[:len(s.rows)])
    return y


def local_rank() -> int:
    return int(os.environ.get('LOCAL_RANK', '0'))
