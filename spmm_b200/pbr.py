"""PBR (packed 64-bit-bitset blocks) front end: the reference's Python API over
the C ABI.

Same names, arguments, classes and exceptions as the reference's
``torch_fast_spdmm/torch_fast_spdmm/__init__.py``:

* ``csr_to_pbr`` (__init__.py:255-274) builds the format ON THE GPU
  (``spmm_pbr_build_analyze`` / ``_emit``), equal to the reference's CPU builder
  (pbr_matrix.cpp:333-448) with blocks in (stripe, block column) order.
* ``PBRMatrix*.to(device)`` (__init__.py:17-40) stages codes as int64 and
  coordinates / offsets / remainder in the host index dtype.
* ``pbr_matmul`` (__init__.py:218-252): every ``kernel=`` value runs the one
  sm_100a kernel ``spmm_pbr_matmul``.  A CPU ``x`` is multiplied on the current
  CUDA device with host copies in and out: there is no CPU implementation.
* ``pbr_to_csr``, ``pbr_info``, ``pbr_analyze_csr`` are host utilities.
"""

from __future__ import annotations

import ctypes as C
import types
from dataclasses import dataclass

import numpy as np
import scipy.sparse as sp
import torch

from . import _lib
from ._device import default_device, ptr, require_cuda, stream_handle, to_device

__all__ = ['csr_to_pbr', 'pbr_to_csr', 'pbr_matmul', 'pbr_info', 'PBRInfo', 'BlockFillStats',
           'BlockStripeStats', 'pbr_analyze_csr', 'pbr_batched_matmul_cuda',
           'pbr_batched_matmul_cpu', 'pbr_batched_matmul_chunkcols_cuda',
           'pbr_batched_matmul_nnzflat_cuda', 'pbr_batched_matmul_variant_cuda',
           'PBRMatrixInt32Float', 'PBRMatrixInt64Float', 'PBRMatrixInt32Double',
           'PBRMatrixInt64Double', 'DataOrder']

PBR_KERNELS = ('block', 'chunkcols', 'nnzflat', 'nnzflat_shared', 'nnzflat_onthefly')


class DataOrder:
    BLOCK_ROW_MAJOR = 0
    BLOCK_COLUMN_MAJOR = 1
    INTERLEAVED_ROW_MAJOR = 2
    INTERLEAVED_COLUMN_MAJOR = 3


class _PBRMatrix:
    _index_dtype = np.int64
    _scalar_dtype = np.float32

    def __init__(self, sizes: dict, dev: types.SimpleNamespace):
        self.rows = int(sizes['rows'])
        self.cols = int(sizes['cols'])
        self.block_rows = int(sizes['block_rows'])
        self.block_cols = int(sizes['block_cols'])
        self.total_nnz = int(sizes['total_nnz'])
        self.data_order = DataOrder.BLOCK_ROW_MAJOR
        self._sizes = {k: int(v) for k, v in sizes.items()}
        self._host = None
        self._dev = dev
        self._gpu_meta = None

    def _host_arrays(self) -> dict:
        if self._host is None:
            d = self._dev
            h = {'block_codes': d.codes.cpu().numpy().view(np.uint64),
                 'block_coords': d.coords.cpu().numpy().astype(self._index_dtype),
                 'block_offsets': d.offsets.cpu().numpy().astype(self._index_dtype),
                 'block_data': d.data.cpu().numpy(),
                 'remainder_indptr': d.rem_indptr.cpu().numpy().astype(self._index_dtype),
                 'remainder_col_ind': d.rem_col_ind.cpu().numpy().astype(self._index_dtype),
                 'remainder_data': d.rem_vals.cpu().numpy()}
            for a in h.values():
                a.setflags(write=False)
            self._host = h
        return self._host

    def _array(self, name):
        return self._host_arrays()[name].copy()

    block_codes = property(lambda s: s._array('block_codes'))
    block_coords = property(lambda s: s._array('block_coords'))
    block_offsets = property(lambda s: s._array('block_offsets'))
    block_data = property(lambda s: s._array('block_data'))
    remainder_indptr = property(lambda s: s._array('remainder_indptr'))
    remainder_col_ind = property(lambda s: s._array('remainder_col_ind'))
    remainder_data = property(lambda s: s._array('remainder_data'))

    def accounted_blocks(self) -> int:
        return self._sizes['nb']

    def compressed_nnz(self) -> int:
        return self._sizes['nnz_c']

    def remainder_nnz(self) -> int:
        return self._sizes['rem_nnz']

    def __repr__(self):
        return (f'PBRMatrix({self.rows}x{self.cols}, blocks={self.accounted_blocks()}, '
                f'compressed_nnz={self.compressed_nnz()}, remainder_nnz={self.remainder_nnz()}, '
                f'total_nnz={self.total_nnz})')

    def to(self, device='cuda'):
        target = 'cpu' if device is None else str(torch.device(device))
        current = str(self._gpu_meta.codes.device) if self._gpu_meta is not None else 'cpu'
        if current == target:
            return self
        if target != 'cpu':
            dev = torch.device(target)
            if dev.index is None:
                dev = torch.device('cuda', torch.cuda.current_device())
            if self._dev is not None and self._dev.codes.device == dev:
                self._gpu_meta = self._dev
            else:
                h = self._host_arrays()
                self._gpu_meta = types.SimpleNamespace(
                    codes=to_device(h['block_codes'].view(np.int64), dev),
                    coords=to_device(h['block_coords'], dev),
                    offsets=to_device(h['block_offsets'], dev),
                    data=to_device(h['block_data'], dev),
                    rem_indptr=to_device(h['remainder_indptr'], dev),
                    rem_col_ind=to_device(h['remainder_col_ind'], dev),
                    rem_vals=to_device(h['remainder_data'], dev))
                torch.cuda.synchronize(dev)
        else:
            if self._host is None and self._dev is not None:
                self._host_arrays()
            self._gpu_meta = None
            self._dev = None
        return self

    def _staged_on(self, device: torch.device) -> types.SimpleNamespace:
        for d in (self._gpu_meta, self._dev):
            if d is not None and d.codes.device == device:
                return d
        tmp = _PBRMatrix.__new__(type(self))
        tmp.__dict__.update(self.__dict__)
        tmp._gpu_meta = None
        tmp.to(device)
        return tmp._gpu_meta

    def _dev_struct(self, d: types.SimpleNamespace) -> _lib.PbrDev:
        st = _lib.PbrDev()
        for k in _lib.PBR_SIZE_FIELDS:
            setattr(st, k, self._sizes[k])
        st.index_type = _lib.I32 if d.coords.dtype == torch.int32 else _lib.I64
        st.scalar_type = _lib.F32 if self._scalar_dtype == np.float32 else _lib.F64
        for name in _lib.PBR_PTR_FIELDS:
            setattr(st, name, ptr(getattr(d, name)))
        return st


class PBRMatrixInt64Float(_PBRMatrix):
    _index_dtype, _scalar_dtype = np.int64, np.float32


class PBRMatrixInt32Float(_PBRMatrix):
    _index_dtype, _scalar_dtype = np.int32, np.float32


class PBRMatrixInt64Double(_PBRMatrix):
    _index_dtype, _scalar_dtype = np.int64, np.float64


class PBRMatrixInt32Double(_PBRMatrix):
    _index_dtype, _scalar_dtype = np.int32, np.float64


_PBR_TYPE_MAP = {c.__name__: (c._index_dtype, c._scalar_dtype)
                 for c in (PBRMatrixInt64Float, PBRMatrixInt32Float, PBRMatrixInt64Double,
                           PBRMatrixInt32Double)}


def _pbr_class(index_dtype, scalar_dtype):
    i = 'Int32' if np.dtype(index_dtype) == np.int32 else 'Int64'
    s = 'Float' if np.dtype(scalar_dtype) == np.float32 else 'Double'
    return globals()[f'PBRMatrix{i}{s}']


def _gpu_build_pbr(indptr, indices, data, rows, cols, block_rows, block_cols, min_nnz):
    require_cuda('csr_to_pbr')
    L = _lib.lib()
    device = default_device()
    if indptr.dtype == np.int32 and indices.dtype == np.int32:
        idt = np.dtype(np.int32)
    else:
        idt = np.dtype(np.int64)
    data = np.asarray(data)
    if data.dtype not in (np.dtype(np.float32), np.dtype(np.float64)):
        raise TypeError('PBR supports float32/float64 matrix values')
    with torch.cuda.device(device):
        d_indptr = to_device(indptr, device, idt)
        d_indices = to_device(indices, device, idt)
        d_vals = to_device(data, device)
        A = _lib.CsrDev()
        A.rows, A.cols, A.nnz = int(rows), int(cols), int(data.size)
        A.indptr, A.indices, A.values = ptr(d_indptr), ptr(d_indices), ptr(d_vals)
        A.index_type = _lib.I32 if idt == np.int32 else _lib.I64
        A.scalar_type = _lib.F32 if data.dtype == np.float32 else _lib.F64
        ws_bytes = int(L.spmm_pbr_build_workspace_size(A.rows, A.cols, A.nnz))
        ws = torch.empty(ws_bytes, dtype=torch.uint8, device=device)
        sizes = _lib.PbrDev()
        s = stream_handle(device)
        st = L.spmm_pbr_build_analyze(C.byref(A), block_rows, block_cols, min_nnz, ws.data_ptr(),
                                      ws_bytes, C.byref(sizes), s)
        if st == _lib.SPMM_EDUPLICATE:
            raise ValueError('csr_to_pbr: the CSR has duplicate (row, col) entries; the PBR '
                             'bitset cannot represent them (sum duplicates first)')
        if st == _lib.SPMM_EINVAL:
            raise ValueError('csr_to_pbr: invalid input')
        _lib.check(st, 'csr_to_pbr')
        n = {k: int(getattr(sizes, k)) for k in _lib.PBR_SIZE_FIELDS}
        tdt = torch.int32 if idt == np.int32 else torch.int64
        vdt = torch.float32 if data.dtype == np.float32 else torch.float64
        dev = types.SimpleNamespace(
            codes=torch.empty(n['nb'], dtype=torch.int64, device=device),
            coords=torch.empty(2 * n['nb'], dtype=tdt, device=device),
            offsets=torch.empty(n['nb'] + 1, dtype=tdt, device=device),
            data=torch.empty(n['nnz_c'], dtype=vdt, device=device),
            rem_indptr=torch.empty(n['rows'] + 1, dtype=tdt, device=device),
            rem_col_ind=torch.empty(n['rem_nnz'], dtype=tdt, device=device),
            rem_vals=torch.empty(n['rem_nnz'], dtype=vdt, device=device))
        sizes.index_type = A.index_type
        for name in _lib.PBR_PTR_FIELDS:
            setattr(sizes, name, ptr(getattr(dev, name)))
        st = L.spmm_pbr_build_emit(C.byref(A), block_rows, block_cols, min_nnz, ws.data_ptr(),
                                   ws_bytes, C.byref(sizes), s)
        _lib.check(st, 'csr_to_pbr')
        torch.cuda.current_stream(device).synchronize()
        del d_indptr, d_indices, d_vals, ws
    return _pbr_class(idt, data.dtype)(n, dev)


def csr_to_pbr(mat, block_rows: int = 8, block_cols: int = 8, min_nnz_per_block: int = 4):
    """Build PBR on the GPU (__init__.py:255-274).  ``min_nnz_per_block`` is the
    reference's uint8_t parameter: values outside [0, 255] raise TypeError like
    its pybind conversion does; block_rows * block_cols must be <= 64."""
    if isinstance(mat, torch.Tensor):
        if mat.device.type != 'cpu':
            raise ValueError('Input tensor must be on CPU')
        indptr = mat.crow_indices().numpy()
        indices = mat.col_indices().numpy()
        data = mat.values().cpu().numpy()
        rows, cols = mat.shape
    elif isinstance(mat, sp.csr_matrix):
        indptr, indices, data = mat.indptr, mat.indices, mat.data
        rows, cols = mat.shape
    else:
        raise TypeError(f'Unsupported type {type(mat)}')
    if not isinstance(min_nnz_per_block, (int, np.integer)) or not 0 <= min_nnz_per_block <= 255:
        raise TypeError('min_nnz_per_block must be an integer in [0, 255] (uint8_t)')
    if block_rows <= 0 or block_cols <= 0 or block_rows * block_cols > 64:
        raise ValueError('block_rows * block_cols must be in [1, 64] (one 64-bit code per block)')
    return _gpu_build_pbr(np.asarray(indptr), np.asarray(indices), data, rows, cols,
                          int(block_rows), int(block_cols), int(min_nnz_per_block))


def pbr_to_csr(pbr_mat) -> sp.csr_matrix:
    """Blocks (bit order) + remainder, rows sorted by (col, value)
    (pbr_matrix.cpp:279-331), on the GPU (spmm_pbr_to_csr)."""
    from .boo import _csr_from_device
    index_dtype, scalar_dtype = _PBR_TYPE_MAP[type(pbr_mat).__name__]
    require_cuda('pbr_to_csr')
    meta = pbr_mat._gpu_meta
    device = meta.codes.device if meta is not None else default_device()
    if meta is None:
        meta = pbr_mat._staged_on(device)
    st = pbr_mat._dev_struct(meta)
    n = int(pbr_mat._sizes['nnz_c'] + pbr_mat._sizes['rem_nnz'])
    L = _lib.lib()

    def run(indptr, indices, values, itype):
        ws_bytes = L.spmm_pbr_to_csr_workspace_size(C.byref(st))
        ws = torch.empty(ws_bytes, dtype=torch.uint8, device=device)
        rc = L.spmm_pbr_to_csr(C.byref(st), ptr(indptr), ptr(indices), ptr(values), itype, ptr(ws), ws_bytes,
                               stream_handle(device))
        if rc == _lib.SPMM_EINVAL:
            raise RuntimeError('Block has a nonzero past the last matrix row. Check block size and '
                               'matrix dimensions for compatibility.')
        _lib.check(rc, 'pbr_to_csr')

    return _csr_from_device(pbr_mat.rows, pbr_mat.cols, n, index_dtype, scalar_dtype, device, run)


def _run_pbr(pbr_mat, meta, x: torch.Tensor) -> torch.Tensor:
    device = x.device
    with torch.cuda.device(device):
        x3 = (x if x.dim() == 3 else x.unsqueeze(0)).contiguous()
        batch, _, K = x3.shape
        y = torch.empty((batch, pbr_mat.rows, K), dtype=x.dtype, device=device)
        if y.numel():
            st = pbr_mat._dev_struct(meta)
            rc = _lib.lib().spmm_pbr_matmul(C.byref(st), ptr(x3), ptr(y), batch, K, None,
                                             stream_handle(device))
            _lib.check(rc, 'pbr_matmul')
    return y


def _check_x(pbr_mat, x):
    expected = torch.float32 if _PBR_TYPE_MAP[type(pbr_mat).__name__][1] == np.float32 else torch.float64
    if x.layout != torch.strided:
        raise ValueError('X must be a dense tensor')
    if x.dtype != expected:
        raise TypeError(f'X dtype must match PBR values ({expected}), got {x.dtype}')
    if x.size(-2) != pbr_mat.cols:
        raise ValueError(f'X has {x.size(-2)} rows, expected {pbr_mat.cols}')


def pbr_batched_matmul_cuda(pbr_mat, x: torch.Tensor, csr_mode: int = 0,
                            smem_size: int = 2048) -> torch.Tensor:
    """Batched Y = A @ X on X's device (__init__.py:122-153): Y is [B, rows, K]
    for 3-D X."""
    meta = getattr(pbr_mat, '_gpu_meta', None)
    if meta is None:
        raise RuntimeError("PBRMatrix is not on GPU. Call .to('cuda') first.")
    _check_x(pbr_mat, x)
    if meta.codes.device != x.device:
        raise ValueError('PBR metadata and X must be on the same CUDA device')
    return _run_pbr(pbr_mat, meta, x)


pbr_batched_matmul_chunkcols_cuda = pbr_batched_matmul_cuda
pbr_batched_matmul_nnzflat_cuda = pbr_batched_matmul_cuda


def pbr_batched_matmul_variant_cuda(pbr_mat, x, prefix, csr_mode=0, smem_size=2048):
    return pbr_batched_matmul_cuda(pbr_mat, x, csr_mode, smem_size)


def pbr_batched_matmul_cpu(pbr_mat, x: torch.Tensor) -> torch.Tensor:
    """Host operands in and out; the product itself runs on the current CUDA
    device (there is no CPU implementation)."""
    require_cuda('pbr_batched_matmul_cpu')
    _check_x(pbr_mat, x)
    device = default_device()
    meta = pbr_mat._staged_on(device)
    y = _run_pbr(pbr_mat, meta, x.to(device, non_blocking=True))
    out = torch.empty(y.shape, dtype=y.dtype, pin_memory=x.is_pinned())
    out.copy_(y, non_blocking=True)
    torch.cuda.current_stream(device).synchronize()
    return out


def pbr_matmul(pbr_mat, x: torch.Tensor, csr_mode: int = 0, smem_size: int = 2048,
               kernel: str = 'block') -> torch.Tensor:
    """Y = A @ X (__init__.py:218-252).  ``csr_mode``, ``smem_size`` and
    ``kernel`` select among the reference's sm_86 kernels; here one kernel
    serves all of them.  A CPU ``x`` is multiplied on the current CUDA device."""
    if x.dim() not in (2, 3):
        raise ValueError(f"Expected 2D or 3D input, got {x.dim()}D")
    if x.is_cuda:
        meta = getattr(pbr_mat, '_gpu_meta', None)
        if meta is None:
            raise RuntimeError("[pbr_matmul] X is on GPU but PBRMatrix is not. Call .to('cuda') first.")
        y = pbr_batched_matmul_cuda(pbr_mat, x, csr_mode=csr_mode, smem_size=smem_size)
    else:
        y = pbr_batched_matmul_cpu(pbr_mat, x)
    return y.squeeze(0) if x.dim() == 2 else y


@dataclass(frozen=True)
class BlockFillStats:
    min: int
    max: int
    mean: float
    max_possible: int


@dataclass(frozen=True)
class BlockStripeStats:
    min: int
    max: int
    mean: float


@dataclass(frozen=True)
class PBRInfo:
    shape: tuple
    block_size: tuple
    total_nnz: int
    compressed_nnz: int
    remainder_nnz: int
    compressed_fraction: float
    num_blocks: int
    num_unique_patterns: int
    avg_reuse: float
    block_fill: BlockFillStats
    blocks_per_stripe: BlockStripeStats


def pbr_info(pbr_mat) -> PBRInfo:
    """Structural summary of a built PBR matrix (__init__.py:344-397)."""
    codes = np.asarray(pbr_mat.block_codes, dtype=np.uint64)
    num_blocks = len(codes)
    total_nnz = int(pbr_mat.total_nnz)
    compressed_nnz = int(pbr_mat.compressed_nnz())
    remainder_nnz = int(pbr_mat.remainder_nnz())
    max_possible = pbr_mat.block_rows * pbr_mat.block_cols
    if num_blocks > 0:
        popcounts = np.array([bin(int(c)).count('1') for c in codes], dtype=np.int32)
        num_unique = int(np.unique(codes).size)
        rows_abs = np.asarray(pbr_mat.block_coords).reshape(-1, 2)[:, 0]
        _, stripe_counts = np.unique(rows_abs // pbr_mat.block_rows, return_counts=True)
        block_fill = BlockFillStats(min=int(popcounts.min()), max=int(popcounts.max()),
                                    mean=float(popcounts.mean()), max_possible=max_possible)
        blocks_per_stripe = BlockStripeStats(min=int(stripe_counts.min()),
                                             max=int(stripe_counts.max()),
                                             mean=float(stripe_counts.mean()))
    else:
        num_unique = 0
        block_fill = BlockFillStats(min=0, max=0, mean=0.0, max_possible=max_possible)
        blocks_per_stripe = BlockStripeStats(min=0, max=0, mean=0.0)
    return PBRInfo(shape=(pbr_mat.rows, pbr_mat.cols),
                   block_size=(pbr_mat.block_rows, pbr_mat.block_cols), total_nnz=total_nnz,
                   compressed_nnz=compressed_nnz, remainder_nnz=remainder_nnz,
                   compressed_fraction=compressed_nnz / total_nnz if total_nnz > 0 else 0.0,
                   num_blocks=num_blocks, num_unique_patterns=num_unique,
                   avg_reuse=num_blocks / num_unique if num_unique > 0 else 0.0,
                   block_fill=block_fill, blocks_per_stripe=blocks_per_stripe)


@dataclass(frozen=True)
class PBRStats:
    """Block-pattern statistics of a CSR (pbr_matrix.cpp:71-146, 265-277)."""
    rows: int
    cols: int
    nnz: int
    block_rows: int
    block_cols: int
    min_nnz_coverage: int
    accounted_nnz: int
    remainder_nnz: int
    accounted_patterns: int
    accounted_blocks: int
    remainder_coo_overhead: float
    csr_index_size: float
    pbr_index_size: float
    block_stats: list


def pbr_analyze_csr(mat, block_rows: int = 8, block_cols: int = 8, min_nnz_coverage=1000,
                    index_bytes: int | None = None, scalar_bytes: int = 4) -> PBRStats:
    """Pattern statistics: for every distinct block code, its occurrences and
    whether occurrence * popcount reaches ``min_nnz_coverage``."""
    if isinstance(mat, torch.Tensor):
        if mat.device.type != 'cpu':
            raise ValueError('Input tensor must be on CPU')
        csr = sp.csr_matrix((mat.values().numpy(), mat.col_indices().numpy(),
                             mat.crow_indices().numpy()), shape=tuple(mat.shape))
    elif isinstance(mat, sp.csr_matrix):
        csr = mat
    else:
        raise TypeError(f'Unsupported type {type(mat)}')
    rows, cols = csr.shape
    if index_bytes is None:
        index_bytes = 4 if csr.indices.dtype == np.int32 else 8
    r = np.repeat(np.arange(rows, dtype=np.int64), np.diff(csr.indptr))
    c = csr.indices.astype(np.int64)
    n_bcol = (cols + block_cols - 1) // block_cols
    key = (r // block_rows) * n_bcol + c // block_cols
    bit = ((r % block_rows) * block_cols + c % block_cols).astype(np.uint64)
    ukey, inv = np.unique(key, return_inverse=True)
    codes = np.zeros(ukey.size, dtype=np.uint64)
    np.bitwise_or.at(codes, inv, np.uint64(1) << bit)
    ucode, occ = np.unique(codes, return_counts=True)
    pop = np.array([bin(int(x)).count('1') for x in ucode], dtype=np.int64)
    cover = occ * pop
    compress = cover >= min_nnz_coverage
    remainder_nnz = int(cover[~compress].sum())
    accounted_blocks = int(occ[compress].sum())
    nnz = int(csr.nnz)
    overhead = float(remainder_nnz * (2.0 * index_bytes + scalar_bytes))
    stats = [{'code': int(ucode[i]), 'occurrence': int(occ[i]), 'compress': bool(compress[i])}
             for i in range(ucode.size)]
    return PBRStats(rows=rows, cols=cols, nnz=nnz, block_rows=block_rows, block_cols=block_cols,
                    min_nnz_coverage=min_nnz_coverage, accounted_nnz=nnz - remainder_nnz,
                    remainder_nnz=remainder_nnz, accounted_patterns=int(compress.sum()),
                    accounted_blocks=accounted_blocks, remainder_coo_overhead=overhead,
                    csr_index_size=float((nnz + cols + 1) * index_bytes),
                    pbr_index_size=float((2.0 * accounted_blocks + overhead) * index_bytes),
                    block_stats=stats)
