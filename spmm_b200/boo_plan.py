"""BOO execution plans (the reference's ``boo_plan.py:11-123`` API).

In the reference a plan reorders blocks into shared-memory size buckets and
precomputes per-block row tables for its sm_86 row-segmented kernels.  The
sm_100a products here need neither: the tensor-core kernel's workers walk
row groups directly and the CUDA-core kernel builds its row tables in shared
memory.  A plan is still accepted -- same construction, validation and fields
-- so code written against the reference runs unchanged: ``buckets`` records
the reference's bucket boundaries (information only), no device tables are
staged (``extra_device_bytes`` is 0) and ``boo_matmul(..., execution_plan=)``
validates the plan exactly as the reference does and runs the usual product.
"""

from dataclasses import dataclass
import time

import numpy as np
import torch


@dataclass(frozen=True)
class BOOExecutionPlan:
    """Prepared metadata tied to one matrix's current CUDA staging (field by
    field as the reference's, boo_plan.py:11-33)."""

    matrix: object
    source_meta: object
    meta: object
    buckets: tuple
    row_ptr: torch.Tensor
    row_starts: torch.Tensor
    p: int
    bucketed: bool
    precomputed_rows: bool
    build_ms: float
    staging_ms: float
    extra_device_bytes: int


def _buckets(boo, bucketed: bool, p: int) -> tuple:
    """The reference's bucket table (boo_plan.py:36-60): blocks split at the
    median and 90th percentile of their estimated shared-memory need; per
    bucket (start, count, max rows, max cols, max nonzeros)."""
    nb = boo.num_blocks()
    if nb == 0:
        return ()
    nr = np.diff(np.asarray(boo.row_grp_ptr, dtype=np.int64))[boo.blk_row_grp]
    nc = np.diff(np.asarray(boo.col_grp_ptr, dtype=np.int64))[boo.blk_col_grp]
    nnz = np.diff(np.asarray(boo.blk_nz_ptr, dtype=np.int64))
    if not bucketed:
        return (0, nb, int(boo.max_nr), int(boo.max_nc), int(boo.max_nnz_blk))
    scalar_bytes = np.asarray(boo.nz_val).dtype.itemsize
    required = (scalar_bytes + 2) * nnz + 4 * (2 * nr + nc + 1) + scalar_bytes * p * nc + 16
    cuts = np.unique(np.quantile(required, [0.5, 0.9], method='nearest'))
    labels = np.searchsorted(cuts, required, side='left')
    order = np.argsort(labels, kind='stable')
    out, start = [], 0
    for label in np.unique(labels):
        sel = order[labels[order] == label]
        out.extend((start, len(sel), int(nr[sel].max()), int(nc[sel].max()), int(nnz[sel].max())))
        start += len(sel)
    return tuple(out)


def prepare_boo_cuda(boo, *, bucketed: bool = False, precomputed_rows: bool = False, p: int = 64):
    """A plan for ``boo`` in its current CUDA staging (boo_plan.py:83-123:
    same arguments and errors)."""
    source = getattr(boo, '_gpu_meta', None)
    if source is None:
        raise ValueError("Call boo.to('cuda') before preparing an execution plan")
    if int(boo.nz_order) != 0:
        raise ValueError('BOO execution plans require rowmajor nonzeros')
    if p not in (8, 16, 32, 64, 128):
        raise ValueError('p must be one of 8, 16, 32, 64, 128')
    start = time.perf_counter()
    buckets = _buckets(boo, bucketed, p)
    build_ms = (time.perf_counter() - start) * 1000
    empty = torch.empty(0, dtype=torch.int32, device=source.nz_val.device)
    return BOOExecutionPlan(boo, source, source, buckets, empty, empty, p, bool(bucketed),
                            bool(precomputed_rows), build_ms, 0.0, 0)
