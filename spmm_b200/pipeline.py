"""Host-operand BOO products with the PCIe copies overlapped.

``boo_matmul(A, x)`` with ``x`` in (pinned) host memory must copy X to the
GPU, multiply, and copy Y back.  Done one after the other, the two copies
dominate (C2: 403 MB each way at ~55 GB/s, about 7 ms each, around a 1.8 ms
product).  The rows of Y depend on a bounded window of X rows when the
matrix is banded, so the call is split into row-group chunks:

* X goes up in pieces, in row order, on a copy stream;
* chunk i is multiplied (``spmm_boo_matmul_groups``) on a compute stream as
  soon as the pieces holding every X row it uses have arrived;
* its Y rows go down on a second copy stream while later chunks compute and
  later X pieces arrive.

So the H2D and D2H copies run at the same time on the two directions of the
link, and the call takes about the larger of them plus one chunk.  The plan
(chunk boundaries and the largest X row each chunk uses) is computed once per
matrix from the format's own arrays and cached on the matrix.  Applies to
matrices whose rows are in identity order (``row_ids`` ascending, so a chunk's
Y rows are one contiguous range) and that are not remainder-major; others
take the one-shot path.
"""

from __future__ import annotations

import ctypes as C
import types
from typing import Optional

import numpy as np
import torch

from . import _lib
from ._device import ptr

MIN_X_BYTES = 32 << 20     # below this the copies are short and a plain call is as fast
CHUNKS = 32                # row-group chunks per call
PIECES = 16                # H2D pieces of X per call (C2 end to end, measured: 32 / 16 9.4-9.5 ms,
                           # 16 / 32 10.5 ms, 64 / 8 10.3 ms)


def _group_max_col(boo_mat) -> np.ndarray:
    """Largest X row (column of A) each row group uses, -1 for none: over its
    blocks (the largest column id of the block's column group), its rows'
    CSR remainder and their COO tail entries."""
    h = boo_mat._host_arrays()
    s = boo_mat._sizes
    n_rg = s['n_rg']
    out = np.full(n_rg, -1, dtype=np.int64)
    cgp = h['col_grp_ptr'].astype(np.int64)
    col_ids = h['col_ids'].astype(np.int64)
    if s['nb']:
        sizes = np.diff(cgp)
        gmax = np.full(s['n_cg'], -1, dtype=np.int64)
        nz = sizes > 0
        if col_ids.size:
            gmax[nz] = np.maximum.reduceat(col_ids, cgp[:-1][nz])
        np.maximum.at(out, h['blk_row_grp'].astype(np.int64), gmax[h['blk_col_grp'].astype(np.int64)])
    rgp = h['row_grp_ptr'].astype(np.int64)
    row_group = np.empty(s['rows'], dtype=np.int64)
    row_group[h['row_ids'].astype(np.int64)] = np.repeat(np.arange(n_rg), np.diff(rgp))
    if s['rem_nnz']:
        rp = h['rem_indptr'].astype(np.int64)
        has = np.diff(rp) > 0
        rmax = np.maximum.reduceat(h['rem_col_ind'].astype(np.int64), rp[:-1][has])
        np.maximum.at(out, row_group[np.flatnonzero(has)], rmax)
    if s['tail_nnz']:
        np.maximum.at(out, row_group[h['tail_row'].astype(np.int64)], h['tail_col'].astype(np.int64))
    return out


def plan(boo_mat) -> Optional[types.SimpleNamespace]:
    """The chunk plan of a matrix (cached), or None when it does not apply."""
    cached = getattr(boo_mat, '_pipe_plan', False)
    if cached is not False:
        return cached
    s = boo_mat._sizes
    result = None
    rem_major = s['rem_nnz'] > 0 and 2 * s['rem_nnz'] >= s['total_nnz']
    h = boo_mat._host_arrays()
    if not rem_major and s['n_rg'] >= CHUNKS and np.array_equal(h['row_ids'], np.arange(s['rows'])):
        rgp = h['row_grp_ptr'].astype(np.int64)
        gnnz = np.zeros(s['n_rg'], dtype=np.int64)
        if s['nb']:
            np.add.at(gnnz, h['blk_row_grp'].astype(np.int64), np.diff(h['blk_nz_ptr'].astype(np.int64)))
        rp = h['rem_indptr'].astype(np.int64)      # rows in identity order: a group's rows are
        gnnz += rp[rgp[1:]] - rp[rgp[:-1]]          # contiguous, so is its remainder
        gnnz += np.diff(rgp)                        # every row costs its Y write
        from .distributed import nnz_balanced_splits
        bounds = nnz_balanced_splits(gnnz, CHUNKS)
        bounds = np.unique(bounds)
        gmax = _group_max_col(boo_mat)
        need = np.array([gmax[bounds[i]:bounds[i + 1]].max(initial=-1) + 1 for i in range(len(bounds) - 1)])
        need = np.maximum.accumulate(need)          # chunks run in order
        result = types.SimpleNamespace(rg_bounds=bounds, row_bounds=rgp[bounds], x_need=need)
    boo_mat._pipe_plan = result
    return result


_STREAMS = {}


def _streams(device: torch.device):
    key = device.index
    if key not in _STREAMS:
        _STREAMS[key] = tuple(torch.cuda.Stream(device) for _ in range(3))
    return _STREAMS[key]


def applies(boo_mat, x: torch.Tensor) -> bool:
    return (x.dim() == 2 or x.shape[0] == 1) and x.is_pinned() and x.is_contiguous() \
        and x.numel() * x.element_size() >= MIN_X_BYTES and plan(boo_mat) is not None


def host_product(boo_mat, meta, x: torch.Tensor, device: torch.device, engine: str,
                 slab_features: int) -> torch.Tensor:
    """Y (pinned host) = A @ x (pinned host, one batch) with the copies
    overlapped as the module docstring describes."""
    pl = plan(boo_mat)
    x2 = x.reshape(x.shape[-2], x.shape[-1])
    cols, K = x2.shape
    rows = boo_mat.rows
    h2d, comp, d2h = _streams(device)
    L = _lib.lib()
    with torch.cuda.device(device):
        cur = torch.cuda.current_stream(device)
        x_dev = torch.empty((cols, K), dtype=x.dtype, device=device)
        y_dev = torch.empty((rows, K), dtype=x.dtype, device=device)
        y_host = torch.empty((rows, K), dtype=x.dtype, pin_memory=True)
        st = boo_mat._dev_struct(meta)
        from .boo import product_plan
        cfg = _lib.launch_cfg(engine, slab_features=slab_features, plan=product_plan(boo_mat, meta).data_ptr())
        ws_bytes = L.spmm_boo_matmul_workspace_size(C.byref(st), 1, K, C.byref(cfg))
        n_chunks = len(pl.rg_bounds) - 1
        off = (ws_bytes + 255) // 256 * 256
        buf = torch.empty(off + 256 * n_chunks, dtype=torch.uint8, device=device)
        words = buf[off:].view(torch.int32).view(n_chunks, 64)
        if ws_bytes:
            cfg.workspace, cfg.workspace_bytes = buf.data_ptr(), ws_bytes
        # X up in pieces
        cuts = np.linspace(0, cols, PIECES + 1).astype(np.int64)
        h2d.wait_stream(cur)
        arrived = []
        for j in range(PIECES):
            a, b = int(cuts[j]), int(cuts[j + 1])
            with torch.cuda.stream(h2d):
                if b > a:
                    x_dev[a:b].copy_(x2[a:b], non_blocking=True)
                ev = torch.cuda.Event()
                ev.record(h2d)
            arrived.append(ev)
        comp.wait_stream(cur)
        d2h.wait_stream(cur)
        for i in range(n_chunks):
            need = int(pl.x_need[i])
            piece = int(np.searchsorted(cuts, need, side='left')) - 1 if need > 0 else -1
            if piece >= 0:
                comp.wait_event(arrived[min(piece, PIECES - 1)])
            cfg.status = words[i].data_ptr()
            rc = L.spmm_boo_matmul_groups(C.byref(st), ptr(x_dev), ptr(y_dev), 1, K, int(pl.rg_bounds[i]),
                                          int(pl.rg_bounds[i + 1]), C.byref(cfg), comp.cuda_stream)
            _lib.check(rc, 'boo_matmul')
            done = torch.cuda.Event()
            done.record(comp)
            d2h.wait_event(done)
            r0, r1 = int(pl.row_bounds[i]), int(pl.row_bounds[i + 1])
            with torch.cuda.stream(d2h):
                if r1 > r0:
                    y_host[r0:r1].copy_(y_dev[r0:r1], non_blocking=True)
        h2d.synchronize()
        comp.synchronize()
        d2h.synchronize()
        bad = int(words[:, 0].abs().max().item()) if n_chunks else 0
        if bad:
            raise _lib.SpmmError(int(words[:, 0][words[:, 0] != 0][0].item()), 'boo_matmul')
    return y_host.view(x.shape[:-2] + (rows, K))
