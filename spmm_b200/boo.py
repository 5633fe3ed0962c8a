"""BOO (Blocked COO) front end: the reference's Python API over the C ABI.

Same names, arguments, returned classes and exceptions as the reference's
``torch_fast_spdmm/torch_fast_spdmm/boo.py``:

* ``csr_to_boo`` (boo.py:108-210) validates, clusters on the host, then builds
  the format ON THE GPU (``spmm_boo_build_analyze`` / ``_emit``); the result is
  bit-identical to the reference's CPU builder (boo_matrix.cpp:53-274).
* ``BOOMatrix*.to(device)`` (boo.py:54-96) stages / drops the device copy.
* ``boo_matmul`` (boo.py:230-354) runs ``spmm_boo_matmul`` on X's device and
  stream.  A CPU ``x`` is copied to the current CUDA device, multiplied there
  and the result copied back: there is no CPU implementation.
* ``boo_to_csr`` runs on the GPU (``spmm_boo_to_csr``); ``boo_info`` and
  ``boo_arena_bytes`` are host utilities.
"""

from __future__ import annotations

import ctypes as C
import enum
import types
from dataclasses import dataclass
from typing import Optional, Tuple

import numpy as np
import scipy.sparse as sp
import torch

from . import _lib
from ._device import default_device, ptr, require_cuda, stream_handle, to_device
from .clustering import cluster_axes

__all__ = ['csr_to_boo', 'boo_to_csr', 'boo_info', 'boo_matmul', 'boo_arena_bytes', 'BOOInfo',
           'SMALL_BLOCK_POLICIES', 'NZ_ORDERS', 'BooNzOrder', 'BooSmallBlockPolicy',
           'BOOMatrixInt32Float', 'BOOMatrixInt64Float', 'BOOMatrixInt32Double',
           'BOOMatrixInt64Double']

SMALL_BLOCK_POLICIES = ('keep', 'merge', 'remainder', 'tail_batch')
NZ_ORDERS = ('rowmajor', 'colmajor')
_POLICY_CODE = {'keep': 0, 'merge': 1, 'remainder': 2, 'tail_batch': 3}
_ORDER_CODE = {'rowmajor': 0, 'colmajor': 1}


class BooNzOrder(enum.IntEnum):
    ROWMAJOR = 0
    COLMAJOR = 1


class BooSmallBlockPolicy(enum.IntEnum):
    KEEP = 0
    MERGE = 1
    REMAINDER = 2
    TAIL_BATCH = 3


# device arrays: name -> torch dtype on the GPU (int32 indices, the reference's
# staging types, boo.py:71-90); nz_idx is an int16 bit view of uint16
_DEV_DTYPES = {
    'row_grp_ptr': torch.int32, 'row_ids': torch.int32, 'col_grp_ptr': torch.int32,
    'col_ids': torch.int32, 'blk_row_grp': torch.int32, 'blk_col_grp': torch.int32,
    'blk_nz_ptr': torch.int32, 'blk_shift': torch.uint8, 'nz_idx': torch.int16, 'nz_val': None,
    'rem_indptr': torch.int32, 'rem_col_ind': torch.int32, 'rem_vals': None,
    'tail_row': torch.int32, 'tail_col': torch.int32, 'tail_val': None,
}


class _BOOMatrix:
    """A BOO matrix.  Host arrays are numpy (index dtype of the input CSR);
    the device copy, when staged, is ``_gpu_meta``."""

    _index_dtype = np.int64
    _scalar_dtype = np.float32

    def __init__(self, sizes: dict, dev: types.SimpleNamespace):
        self.rows = int(sizes['rows'])
        self.cols = int(sizes['cols'])
        self.total_nnz = int(sizes['total_nnz'])
        self.max_nr = int(sizes['max_nr'])
        self.max_nc = int(sizes['max_nc'])
        self.max_nnz_blk = int(sizes['max_nnz_blk'])
        self.nz_order = BooNzOrder(int(sizes['nz_order']))
        self._sizes = {k: int(v) for k, v in sizes.items()}
        self._host = None          # dict of numpy arrays, materialised lazily
        self._dev = dev            # device arrays (build result or staged copy)
        self._gpu_meta = None

    # ---- host arrays -------------------------------------------------------
    def _host_arrays(self) -> dict:
        if self._host is None:
            d = self._dev
            h = {}
            for name, tdt in _DEV_DTYPES.items():
                a = getattr(d, name).cpu().numpy()
                if name == 'nz_idx':
                    a = a.view(np.uint16)
                elif name == 'blk_shift':
                    a = a.astype(np.uint8)
                elif tdt is None:
                    a = a.astype(self._scalar_dtype, copy=False)
                else:
                    a = a.astype(self._index_dtype)
                a.setflags(write=False)
                h[name] = a
            self._host = h
        return self._host

    def _array(self, name):
        return self._host_arrays()[name].copy()

    row_grp_ptr = property(lambda s: s._array('row_grp_ptr'))
    row_ids = property(lambda s: s._array('row_ids'))
    col_grp_ptr = property(lambda s: s._array('col_grp_ptr'))
    col_ids = property(lambda s: s._array('col_ids'))
    blk_row_grp = property(lambda s: s._array('blk_row_grp'))
    blk_col_grp = property(lambda s: s._array('blk_col_grp'))
    blk_nz_ptr = property(lambda s: s._array('blk_nz_ptr'))
    blk_shift = property(lambda s: s._array('blk_shift'))
    nz_idx = property(lambda s: s._array('nz_idx'))
    nz_val = property(lambda s: s._array('nz_val'))
    rem_indptr = property(lambda s: s._array('rem_indptr'))
    rem_col_ind = property(lambda s: s._array('rem_col_ind'))
    rem_vals = property(lambda s: s._array('rem_vals'))
    tail_row = property(lambda s: s._array('tail_row'))
    tail_col = property(lambda s: s._array('tail_col'))
    tail_val = property(lambda s: s._array('tail_val'))

    def num_blocks(self) -> int:
        return self._sizes['nb']

    def num_row_groups(self) -> int:
        return self._sizes['n_rg']

    def num_col_groups(self) -> int:
        return self._sizes['n_cg']

    def compressed_nnz(self) -> int:
        return self._sizes['nnz_c']

    def remainder_nnz(self) -> int:
        return self._sizes['rem_nnz']

    def tail_nnz(self) -> int:
        return self._sizes['tail_nnz']

    def __repr__(self):
        return (f'BOOMatrix({self.rows}x{self.cols}, blocks={self.num_blocks()}, '
                f'grid={self.num_row_groups()}x{self.num_col_groups()}, max_nr={self.max_nr}, '
                f'max_nc={self.max_nc}, max_nnz_blk={self.max_nnz_blk}, '
                f'compressed_nnz={self.compressed_nnz()}, remainder_nnz={self.remainder_nnz()}, '
                f'tail_nnz={self.tail_nnz()})')

    # ---- staging (boo.py:54-96) --------------------------------------------
    def to(self, device='cuda'):
        device = torch.device('cpu' if device is None else device)
        if device.type not in ('cpu', 'cuda'):
            raise ValueError('BOO supports only CPU and CUDA devices')
        if device.type == 'cuda' and device.index is None:
            device = torch.device('cuda', torch.cuda.current_device())
        current = str(self._gpu_meta.nz_val.device) if self._gpu_meta is not None else 'cpu'
        if current == str(device):
            return self
        if device.type == 'cuda':
            if max(self.rows, self.cols, self.total_nnz) > np.iinfo(np.int32).max:
                raise ValueError('BOO CUDA metadata must fit int32')
            if self._dev is not None and self._dev.nz_val.device == device:
                self._gpu_meta = self._dev
            else:
                h = self._host_arrays()
                meta = {}
                for name, tdt in _DEV_DTYPES.items():
                    a = h[name]
                    if name == 'nz_idx':
                        a = np.ascontiguousarray(a).view(np.int16)
                    elif tdt is torch.int32:
                        a = a.astype(np.int32)
                    meta[name] = to_device(a, device)
                self._gpu_meta = types.SimpleNamespace(**meta)
                torch.cuda.synchronize(device)
        else:
            if self._host is None and self._dev is not None:
                self._host_arrays()
            self._gpu_meta = None
            self._dev = None
        return self

    def _staged_on(self, device: torch.device) -> types.SimpleNamespace:
        """Device arrays on `device` for a call with host operands: the staged
        copy, the build result, or a fresh temporary staging."""
        for d in (self._gpu_meta, self._dev):
            if d is not None and d.nz_val.device == device:
                return d
        tmp = _BOOMatrix.__new__(type(self))
        tmp.__dict__.update(self.__dict__)
        tmp._gpu_meta = None
        tmp.to(device)
        return tmp._gpu_meta

    def _dev_struct(self, d: types.SimpleNamespace) -> _lib.BooDev:
        st = _lib.BooDev()
        for k in _lib.BOO_SIZE_FIELDS:
            setattr(st, k, self._sizes[k])
        st.nz_order = int(self.nz_order)
        st.scalar_type = _lib.F32 if self._scalar_dtype == np.float32 else _lib.F64
        for name in _lib.BOO_PTR_FIELDS:
            setattr(st, name, ptr(getattr(d, name)))
        return st


def _boo_class(index_dtype, scalar_dtype):
    i = 'Int32' if np.dtype(index_dtype) == np.int32 else 'Int64'
    s = 'Float' if np.dtype(scalar_dtype) == np.float32 else 'Double'
    return globals()[f'BOOMatrix{i}{s}']


class BOOMatrixInt64Float(_BOOMatrix):
    _index_dtype, _scalar_dtype = np.int64, np.float32


class BOOMatrixInt32Float(_BOOMatrix):
    _index_dtype, _scalar_dtype = np.int32, np.float32


class BOOMatrixInt64Double(_BOOMatrix):
    _index_dtype, _scalar_dtype = np.int64, np.float64


class BOOMatrixInt32Double(_BOOMatrix):
    _index_dtype, _scalar_dtype = np.int32, np.float64


_BOO_TYPE_MAP = {c.__name__: (c._index_dtype, c._scalar_dtype)
                 for c in (BOOMatrixInt64Float, BOOMatrixInt32Float, BOOMatrixInt64Double,
                           BOOMatrixInt32Double)}


# ---------------------------------------------------------------------------
# build
# ---------------------------------------------------------------------------

def _as_scipy_csr(mat) -> sp.csr_matrix:
    if isinstance(mat, torch.Tensor):
        if mat.device.type != 'cpu':
            raise ValueError('Input tensor must be on CPU')
        if mat.layout != torch.sparse_csr or mat.dim() != 2:
            raise ValueError('Input tensor must be a 2D sparse CSR tensor')
        return sp.csr_matrix(
            (mat.values().cpu().numpy(), mat.col_indices().numpy(), mat.crow_indices().numpy()),
            shape=tuple(mat.shape))
    if isinstance(mat, sp.csr_matrix):
        return mat
    raise TypeError(f'Unsupported type {type(mat)}')


def _index_dtype_of(csr) -> np.dtype:
    if csr.indptr.dtype == np.int32 and csr.indices.dtype == np.int32:
        return np.dtype(np.int32)
    return np.dtype(np.int64)


def _stage_csr(csr, device, idt):
    d_indptr = to_device(csr.indptr, device, idt)
    d_indices = to_device(csr.indices, device, idt)
    d_vals = to_device(csr.data, device)
    A = _lib.CsrDev()
    A.rows, A.cols, A.nnz = int(csr.shape[0]), int(csr.shape[1]), int(csr.data.size)
    A.indptr, A.indices, A.values = ptr(d_indptr), ptr(d_indices), ptr(d_vals)
    A.index_type = _lib.I32 if idt == np.int32 else _lib.I64
    A.scalar_type = _lib.F32 if csr.data.dtype == np.float32 else _lib.F64
    return A, (d_indptr, d_indices, d_vals)


def _raise_build_error(status: int, where: str):
    if status == _lib.SPMM_ELABEL:
        raise ValueError(f'{where}: cluster label out of range')
    if status == _lib.SPMM_EOVERFLOW_U16:
        raise ValueError('csr_to_boo: block local index space exceeds uint16 -- '
                         'reduce max_nr/max_nc in the clustering')
    if status == _lib.SPMM_EINVAL:
        raise ValueError(f'{where}: invalid input ({_lib.status_string(status)})')
    raise _lib.SpmmError(status, where)


def _gpu_build_boo(csr, row_labels, col_labels, policy: int, threshold: int, order: int):
    require_cuda('csr_to_boo')
    L = _lib.lib()
    device = default_device()
    idt = _index_dtype_of(csr)
    sdt = csr.data.dtype
    with torch.cuda.device(device):
        A, keep = _stage_csr(csr, device, idt)
        d_rl = to_device(row_labels, device, np.int32)
        d_cl = to_device(col_labels, device, np.int32)
        ws_bytes = int(L.spmm_boo_build_workspace_size(A.rows, A.cols, A.nnz))
        ws = torch.empty(ws_bytes, dtype=torch.uint8, device=device)
        sizes = _lib.BooDev()
        s = stream_handle(device)
        st = L.spmm_boo_build_analyze(C.byref(A), ptr(d_rl), ptr(d_cl), policy, threshold, order,
                                      ws.data_ptr(), ws_bytes, C.byref(sizes), s)
        if st:
            _raise_build_error(st, 'csr_to_boo')
        n = {k: int(getattr(sizes, k)) for k in _lib.BOO_SIZE_FIELDS}
        vdt = torch.float32 if sdt == np.float32 else torch.float64
        shapes = {'row_grp_ptr': n['n_rg'] + 1, 'row_ids': n['rows'], 'col_grp_ptr': n['n_cg'] + 1,
                  'col_ids': n['cols'], 'blk_row_grp': n['nb'], 'blk_col_grp': n['nb'],
                  'blk_nz_ptr': n['nb'] + 1, 'blk_shift': n['nb'], 'nz_idx': n['nnz_c'],
                  'nz_val': n['nnz_c'], 'rem_indptr': n['rows'] + 1, 'rem_col_ind': n['rem_nnz'],
                  'rem_vals': n['rem_nnz'], 'tail_row': n['tail_nnz'], 'tail_col': n['tail_nnz'],
                  'tail_val': n['tail_nnz']}
        dev = types.SimpleNamespace(**{
            name: torch.empty(shapes[name], dtype=_DEV_DTYPES[name] or vdt, device=device)
            for name in _DEV_DTYPES})
        for name in _lib.BOO_PTR_FIELDS:
            setattr(sizes, name, ptr(getattr(dev, name)))
        st = L.spmm_boo_build_emit(C.byref(A), ptr(d_rl), ptr(d_cl), policy, threshold, order,
                                   ws.data_ptr(), ws_bytes, C.byref(sizes), s)
        if st:
            _raise_build_error(st, 'csr_to_boo')
        torch.cuda.current_stream(device).synchronize()
        del keep, ws
    n['nz_order'] = order
    cls = _boo_class(idt, sdt)
    return cls(n, dev)


def csr_to_boo(mat, cluster: str = 'hem', target_nr: int = 32, target_nc: int = 32,
               max_nr: Optional[int] = None, max_nc: Optional[int] = None,
               max_block_nnz: Optional[int] = None,
               small_block_policy: str = 'remainder', small_block_threshold: int = 4,
               nz_order: str = 'rowmajor', seed: int = 0,
               symmetric: Optional[bool] = None,
               row_labels: Optional[np.ndarray] = None,
               col_labels: Optional[np.ndarray] = None,
               hem_feasible_first: bool = True):
    """Cluster both axes on the host, then build the BOO format on the GPU.

    Argument checks and messages follow the reference (boo.py:149-200).
    ``row_labels``/``col_labels`` bypass clustering.  The returned object is
    in the CPU state (no ``_gpu_meta``) like the reference's; ``.to('cuda')``
    on the build device reuses the built device arrays without a copy.
    """
    if small_block_policy not in SMALL_BLOCK_POLICIES:
        raise ValueError(f'small_block_policy must be one of {SMALL_BLOCK_POLICIES}')
    if nz_order not in NZ_ORDERS:
        raise ValueError(f'nz_order must be one of {NZ_ORDERS}')
    for name, value in (('target_nr', target_nr), ('target_nc', target_nc),
                        ('max_nr', max_nr), ('max_nc', max_nc),
                        ('max_block_nnz', max_block_nnz)):
        if value is not None and (not isinstance(value, (int, np.integer)) or value <= 0):
            raise ValueError(f'{name} must be a positive integer')
    if not isinstance(small_block_threshold, (int, np.integer)) or small_block_threshold < 0:
        raise ValueError('small_block_threshold must be a nonnegative integer')
    if (row_labels is None) != (col_labels is None):
        raise ValueError('row_labels and col_labels must be supplied together')

    csr = _as_scipy_csr(mat)
    if csr.dtype not in (np.dtype(np.float32), np.dtype(np.float64)):
        raise TypeError('BOO supports float32/float64 matrix values')
    csr.check_format(full_check=True)

    if max_nr is None:
        max_nr = target_nr
    if max_nc is None:
        max_nc = target_nc

    if row_labels is None or col_labels is None:
        row_labels, col_labels = cluster_axes(
            csr, method=cluster, target_nr=target_nr, target_nc=target_nc,
            max_nr=max_nr, max_nc=max_nc, max_block_nnz=max_block_nnz,
            seed=seed, symmetric=symmetric, feasible_first=hem_feasible_first)

    for name, labels, size in (('row_labels', row_labels, csr.shape[0]),
                               ('col_labels', col_labels, csr.shape[1])):
        labels = np.asarray(labels)
        if labels.ndim != 1 or labels.size != size:
            raise ValueError(f'{name} must be a 1D array matching the matrix dimension')
        if not np.issubdtype(labels.dtype, np.integer):
            raise TypeError(f'{name} must contain integer labels')
        if labels.size and (labels.min() < 0 or labels.max() >= size):
            raise ValueError(f'{name} labels must be in [0, {size})')

    if small_block_policy == 'merge':
        # boo_matrix.cpp:65-76
        raise ValueError("csr_to_boo: 'merge' policy is a clustering-level column relabel, "
                         'not a builder policy -- merge the column groups before building')
    return _gpu_build_boo(csr, np.ascontiguousarray(row_labels, dtype=np.int32),
                          np.ascontiguousarray(col_labels, dtype=np.int32),
                          _POLICY_CODE[small_block_policy], int(small_block_threshold),
                          _ORDER_CODE[nz_order])


def _csr_from_device(rows, cols, n, index_dtype, scalar_dtype, device, run) -> sp.csr_matrix:
    """Allocates the CSR outputs and scratch on `device`, lets `run` fill them
    through the C ABI, and returns the host scipy matrix."""
    itype = _lib.I64 if index_dtype == np.int64 else _lib.I32
    tidx = torch.int64 if itype == _lib.I64 else torch.int32
    tval = torch.float64 if scalar_dtype == np.float64 else torch.float32
    with torch.cuda.device(device):
        indptr = torch.empty(rows + 1, dtype=tidx, device=device)
        indices = torch.empty(max(n, 1), dtype=tidx, device=device)
        values = torch.empty(max(n, 1), dtype=tval, device=device)
        run(indptr, indices, values, itype)
        return sp.csr_matrix((values[:n].cpu().numpy(), indices[:n].cpu().numpy(), indptr.cpu().numpy()),
                             shape=(rows, cols))


def boo_to_csr(boo_mat) -> sp.csr_matrix:
    """Rows collected from blocks, remainder and tail, each row sorted by
    (col, value) -- boo_matrix.cpp:277-333 -- on the GPU (spmm_boo_to_csr)."""
    index_dtype, scalar_dtype = _BOO_TYPE_MAP[type(boo_mat).__name__]
    require_cuda('boo_to_csr')
    meta = boo_mat._gpu_meta
    device = meta.nz_val.device if meta is not None else default_device()
    if meta is None:
        meta = boo_mat._staged_on(device)
    st = boo_mat._dev_struct(meta)
    n = int(boo_mat._sizes['nnz_c'] + boo_mat._sizes['rem_nnz'] + boo_mat._sizes['tail_nnz'])
    L = _lib.lib()

    def run(indptr, indices, values, itype):
        ws_bytes = L.spmm_boo_to_csr_workspace_size(C.byref(st))
        ws = torch.empty(ws_bytes, dtype=torch.uint8, device=device)
        _lib.check(L.spmm_boo_to_csr(C.byref(st), ptr(indptr), ptr(indices), ptr(values), itype, ptr(ws),
                                     ws_bytes, stream_handle(device)), 'boo_to_csr')

    return _csr_from_device(boo_mat.rows, boo_mat.cols, n, index_dtype, scalar_dtype, device, run)


# ---------------------------------------------------------------------------
# SpMM
# ---------------------------------------------------------------------------

def product_plan(boo_mat, meta) -> torch.Tensor:
    """The matrix's product plan on the device of ``meta`` (spmm_boo_plan_build:
    each row group's first block, and for remainder-major matrices with
    scattered blocks a row-ordered copy of every entry), built on first use
    and kept with the staging."""
    plan = getattr(meta, 'plan', None)
    if plan is not None:
        return plan
    L = _lib.lib()
    st = boo_mat._dev_struct(meta)
    n = L.spmm_boo_plan_size(C.byref(st))
    w = L.spmm_boo_plan_workspace_size(C.byref(st))
    device = meta.nz_val.device
    with torch.cuda.device(device):
        plan = torch.empty(max(n, 256), dtype=torch.uint8, device=device)
        ws = torch.empty(max(w, 16), dtype=torch.uint8, device=device) if w else None
        rc = L.spmm_boo_plan_build(C.byref(st), ptr(plan), n, ptr(ws), w, stream_handle(device))
        _lib.check(rc, 'boo_plan')
        del ws
    meta.plan = plan
    return plan


def _run_boo(boo_mat, meta, x: torch.Tensor, engine: str = 'auto', slab_features: int = 0,
             wait_us: int = 0) -> Tuple[torch.Tensor, Optional[torch.Tensor]]:
    """(Y, the call's device status word).  One scratch buffer per call from
    torch's caching allocator: the product's workspace, then the status word."""
    device = x.device
    status = None
    with torch.cuda.device(device):
        x3 = x if x.dim() == 3 else x.unsqueeze(0)
        x3 = x3.contiguous()
        batch, _, K = x3.shape
        y = torch.empty((batch, boo_mat.rows, K), dtype=x.dtype, device=device)
        if y.numel():
            st = boo_mat._dev_struct(meta)
            L = _lib.lib()
            cfg = _lib.launch_cfg(engine, slab_features=slab_features, wait_us=wait_us,
                                  plan=product_plan(boo_mat, meta).data_ptr())
            ws_bytes = L.spmm_boo_matmul_workspace_size(C.byref(st), batch, K, C.byref(cfg))
            off = (ws_bytes + 255) // 256 * 256
            buf = torch.empty(off + 256, dtype=torch.uint8, device=device)
            status = buf[off:off + 4].view(torch.int32)
            cfg.status = status.data_ptr()
            if ws_bytes:
                cfg.workspace, cfg.workspace_bytes = buf.data_ptr(), ws_bytes
            rc = L.spmm_boo_matmul(C.byref(st), ptr(x3), ptr(y), batch, K, C.byref(cfg),
                                   stream_handle(device))
            _lib.check(rc, 'boo_matmul')
    return y, status


def product_status(y: torch.Tensor) -> int:
    """Device-side outcome of the product that returned `y` (not in the
    reference): SPMM_OK (0), or SPMM_ETIMEOUT when one of its bounded waits
    expired and `y` is incomplete.  Synchronises `y`'s device."""
    status = getattr(y, '_spmm_status', None)
    if status is None:
        return 0
    return int(status.item())


def check_product(y: torch.Tensor) -> torch.Tensor:
    """Raises SpmmError(SPMM_ETIMEOUT) when the product that returned `y` did
    not complete; returns `y`.  Synchronises `y`'s device."""
    rc = product_status(y)
    if rc:
        raise _lib.SpmmError(rc, 'boo_matmul')
    return y


def _to_host(y: torch.Tensor, like: torch.Tensor) -> torch.Tensor:
    """D2H of a result; into pinned memory when the caller's X is pinned."""
    out = torch.empty(y.shape, dtype=y.dtype, pin_memory=like.is_pinned())
    out.copy_(y, non_blocking=True)
    torch.cuda.current_stream(y.device).synchronize()
    return out


def boo_matmul(boo_mat, x: torch.Tensor, threads: int = 256, p: int = 64,
               csr_mode: int = 0, row_seg: Optional[bool] = None,
               launch_mode: str = 'legacy', execution_plan=None,
               features_per_thread: int = 1,
               nnzflat_impl: Optional[str] = None, *, engine: str = 'auto',
               slab_features: int = 0, wait_us: int = 0) -> torch.Tensor:
    """Y = A @ X (boo.py:230-354).

    ``engine`` (not in the reference) picks the units that multiply the
    blocks: 'auto' (tensor cores for float32 with K a multiple of 128 and
    blocks up to 64 x 64, else CUDA cores), 'cuda_cores', 'tensor_cores'
    (three-term tf32 split, float32 accuracy; an error where not applicable)
    or 'tensor_cores_tf32' (opt-in, one tf32 product: tf32 accuracy, about
    2e-3 relative, never chosen by 'auto').  ``slab_features`` (not in the
    reference) selects the remainder kernels of a remainder-major matrix: 0
    (default) the nnz-flat chunks, or half a warp per row for a remainder of
    at most 16 entries per row with K up to 64 (float32) / 32 (float64); a
    positive value the nnz-flat chunks; a negative value the register path.  ``wait_us`` (not in the reference) bounds the tensor-core
    product's device waits (0: about 2 s); a product whose wait expired
    leaves Y incomplete and reports SPMM_ETIMEOUT through
    ``product_status(y)`` / ``check_product(y)`` (GPU ``x``; a CPU ``x``
    raises ``SpmmError`` directly).

    The launch knobs of the reference's sm_86 kernels (``threads``, ``p``,
    ``csr_mode``, ``features_per_thread``, ``nnzflat_impl``, ``launch_mode``)
    are validated exactly as there and otherwise have no effect: one fused
    sm_100a kernel serves every setting.  ``row_seg=True`` still requires a
    rowmajor matrix.  A CPU ``x`` runs on the current CUDA device with host
    copies in and out.
    """
    if launch_mode not in ('legacy', 'auto'):
        raise ValueError("launch_mode must be 'legacy' or 'auto'")
    if x.dim() not in (2, 3):
        raise ValueError(f'Expected 2D or 3D input, got {x.dim()}D')
    if x.layout != torch.strided or x.device.type not in ('cpu', 'cuda'):
        raise ValueError('X must be a dense CPU or CUDA tensor')
    if x.size(-2) != boo_mat.cols:
        raise ValueError(f'X has {x.size(-2)} rows, expected {boo_mat.cols}')
    expected_dtype = {np.float32: torch.float32, np.float64: torch.float64}[
        _BOO_TYPE_MAP[type(boo_mat).__name__][1]]
    if x.dtype != expected_dtype:
        raise TypeError(f'X dtype must match BOO values ({expected_dtype}), got {x.dtype}')
    if execution_plan is not None and not x.is_cuda:
        raise ValueError('BOO execution plans require CUDA inputs')
    if not x.is_cuda:
        require_cuda('boo_matmul')
        device = default_device()
        meta = boo_mat._staged_on(device)
        from . import pipeline
        if pipeline.applies(boo_mat, x):     # copies in both directions overlapped with the product
            y = pipeline.host_product(boo_mat, meta, x, device, engine, slab_features)
            return y
        yd, status = _run_boo(boo_mat, meta, x.to(device, non_blocking=True), engine, slab_features)
        y = _to_host(yd, x)                      # synchronises: the status word is final
        if status is not None and int(status.item()):
            raise _lib.SpmmError(int(status.item()), 'boo_matmul')
        return y.squeeze(0) if x.dim() == 2 else y

    meta = boo_mat._gpu_meta
    if meta is None:
        raise RuntimeError("[boo_matmul] X is on GPU but BOOMatrix is not. Call .to('cuda') first.")
    if meta.nz_val.device != x.device:
        raise ValueError('BOO metadata and X must be on the same CUDA device')
    if threads not in (128, 256, 512):
        raise ValueError('threads must be one of 128, 256, 512')
    if p not in (8, 16, 32, 64, 128):
        raise ValueError('p must be one of 8, 16, 32, 64, 128')
    if csr_mode not in (0, 1, 2):
        raise ValueError('csr_mode must be one of 0, 1, 2')
    if features_per_thread not in (1, 2, 4):
        raise ValueError('features_per_thread must be one of 1, 2, 4')
    if features_per_thread == 4 and x.dtype != torch.float32:
        raise ValueError('features_per_thread=4 requires float32')
    if nnzflat_impl not in (None, 'reference', 'template'):
        raise ValueError("nnzflat_impl must be None, 'reference' or 'template'")
    if row_seg is None:
        row_seg = int(boo_mat.nz_order) == _ORDER_CODE['rowmajor']
    elif row_seg and int(boo_mat.nz_order) != _ORDER_CODE['rowmajor']:
        raise ValueError('row_seg=True requires a matrix built with nz_order="rowmajor"')
    if row_seg:
        if nnzflat_impl is not None:
            raise ValueError('nnzflat_impl applies only to row_seg=False')
    else:
        if features_per_thread == 4:
            raise ValueError('nnzflat (row_seg=False) supports features_per_thread 1 or 2')
        if nnzflat_impl == 'reference' and features_per_thread != 1:
            raise ValueError("nnzflat_impl='reference' is the FPT=1 kernel; use 'template'")
    if execution_plan is not None:   # validated as boo.py:334-340; the product needs no tables
        from .boo_plan import BOOExecutionPlan
        plan = execution_plan
        if not isinstance(plan, BOOExecutionPlan) or plan.matrix is not boo_mat or plan.source_meta is not meta:
            raise ValueError('Execution plan does not match this matrix and its current CUDA staging')
        if launch_mode != 'auto' or not row_seg or p != plan.p:
            raise ValueError('Execution plans require launch_mode="auto", row_seg=True and the prepared p')
    y, status = _run_boo(boo_mat, meta, x, engine, slab_features, wait_us)
    y = y.squeeze(0) if x.dim() == 2 else y
    y._spmm_status = status      # read by product_status / check_product
    return y


# ---------------------------------------------------------------------------
# offline metrics (boo.py:361-500)
# ---------------------------------------------------------------------------

# The reference's occupancy model is calibrated for sm_86 (boo.py:41-47); it is
# kept so boo_info's fields mean the same thing.
_SMEM_PER_SM = 102400
_DRIVER_SMEM_PER_CTA = 1024
_MAX_THREADS_PER_SM = 1536
_MAX_CTAS_PER_SM = 16


@dataclass(frozen=True)
class BOOInfo:
    shape: Tuple[int, int]
    total_nnz: int
    compressed_nnz: int
    remainder_nnz: int
    tail_nnz: int
    compressed_fraction: float
    boo_fraction: float
    num_blocks: int
    num_row_groups: int
    num_col_groups: int
    n_r_mean: float
    n_r_max: int
    n_c_mean: float
    n_c_max: int
    nnz_per_block_mean: float
    nnz_per_block_max: int
    nnz_per_block_hist: dict
    x_loads: int
    y_writes: int
    arithmetic_intensity: float
    scalar_bytes: int
    p: int
    threads: int
    arena_bytes: int
    ctas_per_sm: int
    occupancy_pct: float


def _occupancy(arena_bytes: int, threads: int) -> Tuple[int, float]:
    by_smem = _SMEM_PER_SM // (arena_bytes + _DRIVER_SMEM_PER_CTA)
    by_warps = _MAX_THREADS_PER_SM // threads
    ctas = max(0, min(by_smem, by_warps, _MAX_CTAS_PER_SM))
    return ctas, 100.0 * ctas * threads / _MAX_THREADS_PER_SM


def boo_arena_bytes(max_nr: int, max_nc: int, max_nnz_blk: int, p: int,
                    scalar_bytes: int, row_seg: bool = True) -> int:
    """Shared-memory arena of the reference's sm_86 kernels (boo.py:428-444)."""
    data = max_nnz_blk * (scalar_bytes + 2)
    if row_seg:
        ids = 4 * (max_nr + max_nc) + 4 * (max_nr + 1)
        tiles = scalar_bytes * p * max_nc
    else:
        ids = 4 * (max_nr + max_nc)
        tiles = scalar_bytes * p * (max_nr + max_nc)
    return data + ids + tiles


def boo_info(boo_mat, p: int = 64, threads: int = 256, row_seg: bool = True) -> BOOInfo:
    """Structural summary derived from the built format (boo.py:447-500)."""
    _, scalar_dtype = _BOO_TYPE_MAP[type(boo_mat).__name__]
    scalar_bytes = np.dtype(scalar_dtype).itemsize
    h = boo_mat._host_arrays()
    row_grp_ptr = h['row_grp_ptr'].astype(np.int64)
    col_grp_ptr = h['col_grp_ptr'].astype(np.int64)
    blk_row_grp = h['blk_row_grp'].astype(np.int64)
    blk_col_grp = h['blk_col_grp'].astype(np.int64)
    blk_nz_ptr = h['blk_nz_ptr'].astype(np.int64)
    rg_size = np.diff(row_grp_ptr)
    cg_size = np.diff(col_grp_ptr)
    nb = int(blk_row_grp.size)
    if nb:
        n_r = rg_size[blk_row_grp]
        n_c = cg_size[blk_col_grp]
        nnz_per_block = np.diff(blk_nz_ptr)
        x_loads = int(n_c.sum())
        y_writes = int(n_r.sum())
        buckets = np.where(nnz_per_block > 0,
                           np.floor(np.log2(np.maximum(nnz_per_block, 1))).astype(int), 0)
        hist = {f'{1 << b}-{(1 << (b + 1)) - 1}': int(count)
                for b, count in zip(*np.unique(buckets, return_counts=True))}
    else:
        n_r = n_c = nnz_per_block = np.zeros(0, dtype=np.int64)
        x_loads = y_writes = 0
        hist = {}
    compressed = int(boo_mat.compressed_nnz())
    tail = int(boo_mat.tail_nnz())
    total = int(boo_mat.total_nnz)
    arena = boo_arena_bytes(int(boo_mat.max_nr), int(boo_mat.max_nc), int(boo_mat.max_nnz_blk),
                            p, scalar_bytes, row_seg)
    ctas, occupancy = _occupancy(arena, threads)
    return BOOInfo(
        shape=(int(boo_mat.rows), int(boo_mat.cols)), total_nnz=total, compressed_nnz=compressed,
        remainder_nnz=int(boo_mat.remainder_nnz()), tail_nnz=tail,
        compressed_fraction=compressed / total if total else 0.0,
        boo_fraction=(compressed + tail) / total if total else 0.0,
        num_blocks=nb, num_row_groups=int(rg_size.size), num_col_groups=int(cg_size.size),
        n_r_mean=float(n_r.mean()) if nb else 0.0, n_r_max=int(n_r.max()) if nb else 0,
        n_c_mean=float(n_c.mean()) if nb else 0.0, n_c_max=int(n_c.max()) if nb else 0,
        nnz_per_block_mean=float(nnz_per_block.mean()) if nb else 0.0,
        nnz_per_block_max=int(nnz_per_block.max()) if nb else 0,
        nnz_per_block_hist=hist, x_loads=x_loads, y_writes=y_writes,
        arithmetic_intensity=compressed / x_loads if x_loads else 0.0,
        scalar_bytes=scalar_bytes, p=p, threads=threads, arena_bytes=arena,
        ctas_per_sm=ctas, occupancy_pct=occupancy)
