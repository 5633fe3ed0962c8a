"""Paired timing harnesses, the counterparts of the reference's C++-level
timed classes (torch_fast_spdmm/bindings/bindings_boo_timed.cu:294-314,
bindings_pbr_timed.cu:198-210, bindings_cusparse.cu:154-160).

Everything a measurement must not include -- the output, the product's
scratch, the CUDA events, the choice of stream -- is set up once at
construction; ``timed_run()`` brackets exactly the product call (one C-ABI
call that launches this library's kernels) with CUDA events on the
construction stream and returns milliseconds.  ``run()`` does the same work
untimed and returns the output, which aliases a persistent tensor that later
runs overwrite (as in the reference).  Calls must come from the construction
stream (the reference raises the same error otherwise).

``DirectSpMM`` is the cuSPARSE reference point (``cusparseSpMM`` on a CSR
matrix with a persistent descriptor, workspace and preprocessing), loaded
from the CUDA toolkit's libcusparse: benchmark-only code, never on the
product path.
"""

from __future__ import annotations

import ctypes as C
import glob
import os
from typing import Optional, Sequence

import numpy as np
import torch

from . import _lib
from ._device import ptr, stream_handle

__all__ = ['BOOTimedSpMM', 'PBRTimedSpMM', 'DirectSpMM']


class _Timed:
    """Construction stream, events and the timing bracket shared by the harnesses."""

    def _setup(self, x: torch.Tensor):
        self._device = x.device
        self._stream = torch.cuda.current_stream(x.device)
        self._start = torch.cuda.Event(enable_timing=True)
        self._end = torch.cuda.Event(enable_timing=True)

    def _check_stream(self, name: str):
        if torch.cuda.current_stream(self._device) != self._stream:
            raise RuntimeError(f'{name} must run on its construction stream')

    def _launch(self):
        raise NotImplementedError

    def run(self) -> torch.Tensor:
        self._check_stream(type(self).__name__)
        with torch.cuda.device(self._device):
            self._launch()
        return self.output

    def timed_run(self) -> float:
        self._check_stream(type(self).__name__)
        with torch.cuda.device(self._device):
            self._start.record(self._stream)
            self._launch()                 # the only work between the events
            self._end.record(self._stream)
            self._end.synchronize()
            return float(self._start.elapsed_time(self._end))


def _check_device_tensors(name: str, x: torch.Tensor, tensors):
    for t in tensors:
        if t is not None and (t.device != x.device or not t.is_contiguous()):
            raise RuntimeError(f'{name}: format tensors must be contiguous and on X\'s device')


class BOOTimedSpMM(_Timed):
    """Y = A @ X for a BOO matrix given by its staged device arrays (the
    fields of ``BOOMatrix._gpu_meta``), argument order and checks as the
    reference's ``BOOTimedSpMM`` (bindings_boo_timed.cu:163-210).  The sm_86
    launch knobs are validated and otherwise ignored, as in ``boo_matmul``;
    ``diagnostic_raw_store`` times the whole product (the fused kernels have
    no separate block-only leg) and makes ``output`` raise, as there."""

    def __init__(self, rows, cols, max_nr, max_nc, max_nnz_blk, row_grp_ptr, row_ids, col_grp_ptr, col_ids,
                 blk_row_grp, blk_col_grp, blk_nz_ptr, blk_shift, nz_idx, nz_val, rem_indptr, rem_col_ind,
                 rem_vals, tail_row, tail_col, tail_val, x, threads: int = 256, p: int = 64, csr_mode: int = 0,
                 row_seg: bool = True, diagnostic_raw_store: bool = False, nnzflat_fpt: int = 1,
                 nnzflat_reference: bool = True, launch_mode: str = 'legacy', buckets: Sequence[int] = (),
                 plan_row_ptr: Optional[torch.Tensor] = None, plan_row_starts: Optional[torch.Tensor] = None,
                 *, engine: str = 'auto'):
        if launch_mode not in ('auto', 'legacy'):
            raise RuntimeError("BOOTimedSpMM: launch_mode must be 'auto' or 'legacy'")
        if len(buckets) and not (launch_mode == 'auto' and row_seg):
            raise RuntimeError('BOOTimedSpMM: buckets require launch_mode="auto" and row_seg=True')
        if (plan_row_ptr is None) != (plan_row_starts is None):
            raise RuntimeError('BOOTimedSpMM: plan_row_ptr and plan_row_starts go together')
        if not (x.is_cuda and x.dtype == torch.float32):
            raise RuntimeError('BOOTimedSpMM: X must be a float32 CUDA tensor')
        if x.dim() not in (2, 3):
            raise RuntimeError('BOOTimedSpMM: X must be 2D or 3D')
        if threads not in (128, 256, 512):
            raise RuntimeError('BOOTimedSpMM: threads must be 128, 256 or 512')
        if p not in (8, 16, 32, 64, 128):
            raise RuntimeError('BOOTimedSpMM: p must be one of 8, 16, 32, 64, 128')
        if csr_mode not in (0, 1, 2):
            raise RuntimeError('BOOTimedSpMM: csr_mode must be 0, 1 or 2')
        if nnzflat_fpt not in (1, 2):
            raise RuntimeError('BOOTimedSpMM: nnzflat_fpt must be 1 or 2')
        if row_seg and not (nnzflat_fpt == 1 and nnzflat_reference):
            raise RuntimeError('BOOTimedSpMM: nnzflat options apply only to row_seg=False')
        if not (nnzflat_fpt == 1 or not nnzflat_reference):
            raise RuntimeError('BOOTimedSpMM: the reference nnzflat kernel is the FPT=1 kernel')
        if diagnostic_raw_store and not row_seg:
            raise RuntimeError('BOOTimedSpMM: diagnostic_raw_store requires row_seg=True')
        arrays = dict(row_grp_ptr=row_grp_ptr, row_ids=row_ids, col_grp_ptr=col_grp_ptr, col_ids=col_ids,
                      blk_row_grp=blk_row_grp, blk_col_grp=blk_col_grp, blk_nz_ptr=blk_nz_ptr,
                      blk_shift=blk_shift, nz_idx=nz_idx, nz_val=nz_val, rem_indptr=rem_indptr,
                      rem_col_ind=rem_col_ind, rem_vals=rem_vals, tail_row=tail_row, tail_col=tail_col,
                      tail_val=tail_val)
        _check_device_tensors('BOOTimedSpMM', x, arrays.values())
        if nz_val.dtype != torch.float32 or rem_vals.dtype != torch.float32:
            raise RuntimeError('BOOTimedSpMM: float32 values only')
        self._arrays = arrays                      # keeps the device arrays alive
        self._setup(x)
        self._diag = bool(diagnostic_raw_store)
        self._squeeze = x.dim() == 2
        self._x = (x.unsqueeze(0) if x.dim() == 2 else x).contiguous()
        batch, _, K = self._x.shape
        self._batch, self._K = batch, K
        nb = int(blk_row_grp.numel())
        st = _lib.BooDev()
        sizes = dict(rows=rows, cols=cols, total_nnz=int(nz_val.numel() + rem_vals.numel() + tail_val.numel()),
                     n_rg=int(row_grp_ptr.numel()) - 1, n_cg=int(col_grp_ptr.numel()) - 1, nb=nb,
                     nnz_c=int(nz_val.numel()), rem_nnz=int(rem_vals.numel()), tail_nnz=int(tail_val.numel()),
                     max_nr=max_nr, max_nc=max_nc, max_nnz_blk=max_nnz_blk)
        for k, v in sizes.items():
            setattr(st, k, int(v))
        # row_seg=True promises row-major blocks (as the reference requires);
        # otherwise the order-agnostic column-major treatment is used
        st.nz_order = 0 if row_seg else 1
        st.scalar_type = _lib.F32
        for name, t in arrays.items():
            setattr(st, name, ptr(t))
        self._st = st
        self._info = dict(diagnostic=self._diag, row_seg=bool(row_seg), nnzflat_fpt=int(nnzflat_fpt),
                          nnzflat_reference=bool(nnzflat_reference), engine=engine)
        L = _lib.lib()
        with torch.cuda.device(self._device):   # the product plan, built once (spmm_boo_plan_build)
            n, w = L.spmm_boo_plan_size(C.byref(st)), L.spmm_boo_plan_workspace_size(C.byref(st))
            self._plan = torch.empty(max(n, 256), dtype=torch.uint8, device=self._device)
            pws = torch.empty(max(w, 16), dtype=torch.uint8, device=self._device)
            _lib.check(L.spmm_boo_plan_build(C.byref(st), self._plan.data_ptr(), n, pws.data_ptr(), w,
                                             stream_handle(self._device)), 'BOOTimedSpMM')
            del pws
        self._cfg = _lib.launch_cfg(engine, plan=self._plan.data_ptr())
        ws = L.spmm_boo_matmul_workspace_size(C.byref(st), batch, K, C.byref(self._cfg))
        with torch.cuda.device(self._device):
            self._y = torch.empty((batch, rows, K), dtype=torch.float32, device=self._device)
            self._ws = torch.empty(max(ws, 1), dtype=torch.uint8, device=self._device)
        self._cfg.workspace, self._cfg.workspace_bytes = self._ws.data_ptr(), ws
        self._sh = stream_handle(self._device)

    def _launch(self):
        if self._y.numel() == 0:
            return
        rc = _lib.lib().spmm_boo_matmul(C.byref(self._st), ptr(self._x), ptr(self._y), self._batch, self._K,
                                        C.byref(self._cfg), self._sh)
        _lib.check(rc, 'BOOTimedSpMM')

    @property
    def output(self) -> torch.Tensor:
        if self._diag:
            raise RuntimeError("BOOTimedSpMM(diagnostic_raw_store=True)'s output is not meaningful")
        return self._y.squeeze(0) if self._squeeze else self._y

    def run(self) -> torch.Tensor:
        self._check_stream('BOOTimedSpMM')
        with torch.cuda.device(self._device):
            self._launch()
        return self._y.squeeze(0) if self._squeeze else self._y

    def info(self) -> dict:
        return dict(self._info)


class PBRTimedSpMM(_Timed):
    """Y = A @ X for a PBR matrix given by its staged device arrays (argument
    order as the reference's ``PBRTimedSpMM``, bindings_pbr_timed.cu:198-206;
    ``kernel`` / ``csr_mode`` / ``smem_size`` validated as in ``pbr_matmul``
    and otherwise ignored)."""

    _KERNELS = ('block', 'chunkcols', 'nnzflat', 'nnzflat_shared', 'nnzflat_onthefly')

    def __init__(self, cols, rows, block_rows, block_cols, block_codes, block_coords, block_offsets, block_data,
                 rem_indptr, rem_col_ind, rem_vals, x, csr_mode: int = 0, smem_size: int = 2048,
                 diagnostic_raw_store: bool = False, kernel: str = 'block'):
        if kernel not in self._KERNELS:
            raise RuntimeError(f'PBRTimedSpMM: unknown kernel {kernel!r}')
        if not (x.is_cuda and x.dtype == torch.float32 and x.dim() in (2, 3)):
            raise RuntimeError('PBRTimedSpMM: X must be a 2D or 3D float32 CUDA tensor')
        if csr_mode not in (0, 1, 2):
            raise RuntimeError('PBRTimedSpMM: csr_mode must be 0, 1 or 2')
        arrays = dict(codes=block_codes, coords=block_coords, offsets=block_offsets, data=block_data,
                      rem_indptr=rem_indptr, rem_col_ind=rem_col_ind, rem_vals=rem_vals)
        _check_device_tensors('PBRTimedSpMM', x, arrays.values())
        self._arrays = arrays
        self._setup(x)
        self._diag = bool(diagnostic_raw_store)
        self._squeeze = x.dim() == 2
        self._x = (x.unsqueeze(0) if x.dim() == 2 else x).contiguous()
        batch, _, K = self._x.shape
        self._batch, self._K = batch, K
        st = _lib.PbrDev()
        nb = int(block_codes.numel())
        sizes = dict(rows=rows, cols=cols, block_rows=block_rows, block_cols=block_cols,
                     total_nnz=int(block_data.numel() + rem_vals.numel()), nb=nb, nnz_c=int(block_data.numel()),
                     rem_nnz=int(rem_vals.numel()))
        for k, v in sizes.items():
            setattr(st, k, int(v))
        st.index_type = _lib.I32 if block_coords.dtype == torch.int32 else _lib.I64
        st.scalar_type = _lib.F32
        for name, t in arrays.items():
            setattr(st, name, ptr(t))
        self._st = st
        self._cfg = _lib.launch_cfg('auto')
        with torch.cuda.device(self._device):
            self._y = torch.empty((batch, rows, K), dtype=torch.float32, device=self._device)
        self._sh = stream_handle(self._device)
        self._info = dict(diagnostic=self._diag, kernel=kernel)

    def _launch(self):
        if self._y.numel() == 0:
            return
        rc = _lib.lib().spmm_pbr_matmul(C.byref(self._st), ptr(self._x), ptr(self._y), self._batch, self._K,
                                        C.byref(self._cfg), self._sh)
        _lib.check(rc, 'PBRTimedSpMM')

    @property
    def output(self) -> torch.Tensor:
        if self._diag:
            raise RuntimeError("PBRTimedSpMM(diagnostic_raw_store=True)'s output is not meaningful")
        return self._y.squeeze(0) if self._squeeze else self._y

    def run(self) -> torch.Tensor:
        self._check_stream('PBRTimedSpMM')
        with torch.cuda.device(self._device):
            self._launch()
        return self._y.squeeze(0) if self._squeeze else self._y

    def info(self) -> dict:
        return dict(self._info)


# ---------------------------------------------------------------------------
# cuSPARSE reference point
# ---------------------------------------------------------------------------

_CUSPARSE = None
# enum values of the public cusparse.h / library_types.h
_SPMM_ALGS = {'DEFAULT': 0, 'CSR_ALG1': 4, 'CSR_ALG2': 6, 'CSR_ALG3': 12}
_INDEX_32I, _BASE_ZERO, _R_32F, _ORDER_ROW, _NON_TRANSPOSE = 2, 0, 0, 2, 0
_STATUS_NOT_SUPPORTED = 10


def _cusparse() -> C.CDLL:
    global _CUSPARSE
    if _CUSPARSE is None:
        cands = []
        try:
            import nvidia.cusparse.lib as _nv
            cands += glob.glob(os.path.join(os.path.dirname(_nv.__file__), 'libcusparse.so*'))
        except ImportError:
            pass
        cands += glob.glob('/usr/local/cuda/lib64/libcusparse.so*')
        if not cands:
            raise RuntimeError('DirectSpMM: libcusparse not found')
        L = C.CDLL(cands[0])
        vp, i64 = C.c_void_p, C.c_int64
        L.cusparseCreate.argtypes = [C.POINTER(vp)]
        L.cusparseSetStream.argtypes = [vp, vp]
        L.cusparseCreateCsr.argtypes = [C.POINTER(vp), i64, i64, i64, vp, vp, vp, C.c_int, C.c_int, C.c_int, C.c_int]
        L.cusparseCreateDnMat.argtypes = [C.POINTER(vp), i64, i64, i64, vp, C.c_int, C.c_int]
        spmm_args = [vp, C.c_int, C.c_int, vp, vp, vp, vp, vp, C.c_int, C.c_int]
        L.cusparseSpMM_bufferSize.argtypes = spmm_args + [C.POINTER(C.c_size_t)]
        L.cusparseSpMM_preprocess.argtypes = spmm_args + [vp]
        L.cusparseSpMM.argtypes = spmm_args + [vp]
        for n in ('cusparseDestroySpMat', 'cusparseDestroyDnMat', 'cusparseDestroy'):
            getattr(L, n).argtypes = [vp]
        _CUSPARSE = L
    return _CUSPARSE


class DirectSpMM(_Timed):
    """cusparseSpMM on an int32 / float32 CSR matrix and a row-major X, with
    the descriptors, workspace and preprocessing made once (the reference's
    DirectSpMM, bindings_cusparse.cu:20-160).  ``algorithm`` in DEFAULT /
    CSR_ALG1 / CSR_ALG2 / CSR_ALG3."""

    def __init__(self, crow: torch.Tensor, col: torch.Tensor, val: torch.Tensor, x: torch.Tensor,
                 algorithm: str = 'DEFAULT'):
        if not (x.is_cuda and x.dim() == 2 and x.is_contiguous() and x.dtype == torch.float32):
            raise RuntimeError('X must be contiguous CUDA FP32, two-dimensional')
        for t in (crow, col, val):
            if t.device != x.device or t.dim() != 1 or not t.is_contiguous():
                raise RuntimeError("CSR arrays must be contiguous 1D tensors on X's device")
        if crow.dtype != torch.int32 or col.dtype != torch.int32 or val.dtype != torch.float32:
            raise RuntimeError('CSR must use int32 indices and FP32 values')
        if crow.numel() < 1 or col.numel() != val.numel():
            raise RuntimeError('Invalid CSR dimensions')
        if algorithm not in _SPMM_ALGS:
            raise RuntimeError(f'Unknown cuSPARSE algorithm: {algorithm}')
        self._setup(x)
        self._keep = (crow, col, val, x)
        self._alg = _SPMM_ALGS[algorithm]
        L = _cusparse()
        rows = crow.numel() - 1
        with torch.cuda.device(x.device):
            self._y = torch.empty((rows, x.size(1)), dtype=torch.float32, device=x.device)
            self._h, self._a, self._b, self._c = C.c_void_p(), C.c_void_p(), C.c_void_p(), C.c_void_p()
            self._alpha, self._beta = C.c_float(1.0), C.c_float(0.0)
            self._ok(L.cusparseCreate(C.byref(self._h)))
            self._ok(L.cusparseSetStream(self._h, C.c_void_p(stream_handle(x.device))))
            self._ok(L.cusparseCreateCsr(C.byref(self._a), rows, x.size(0), val.numel(), crow.data_ptr(),
                                         col.data_ptr(), val.data_ptr(), _INDEX_32I, _INDEX_32I, _BASE_ZERO,
                                         _R_32F))
            self._ok(L.cusparseCreateDnMat(C.byref(self._b), x.size(0), x.size(1), x.size(1), x.data_ptr(),
                                           _R_32F, _ORDER_ROW))
            self._ok(L.cusparseCreateDnMat(C.byref(self._c), rows, x.size(1), x.size(1), self._y.data_ptr(),
                                           _R_32F, _ORDER_ROW))
            nbytes = C.c_size_t(0)
            st = L.cusparseSpMM_bufferSize(self._h, _NON_TRANSPOSE, _NON_TRANSPOSE, C.byref(self._alpha), self._a,
                                           self._b, C.byref(self._beta), self._c, _R_32F, self._alg,
                                           C.byref(nbytes))
            self.supported = st != _STATUS_NOT_SUPPORTED
            self.reason = '' if self.supported else 'CUSPARSE_STATUS_NOT_SUPPORTED at bufferSize'
            if self.supported:
                self._ok(st)
                self._ws = torch.empty(max(nbytes.value, 1), dtype=torch.uint8, device=x.device)
                pre = L.cusparseSpMM_preprocess(self._h, _NON_TRANSPOSE, _NON_TRANSPOSE, C.byref(self._alpha),
                                                self._a, self._b, C.byref(self._beta), self._c, _R_32F,
                                                self._alg, self._ws.data_ptr())
                if pre != _STATUS_NOT_SUPPORTED:
                    self._ok(pre)
                self._bytes = nbytes.value
                torch.cuda.current_stream(x.device).synchronize()

    @staticmethod
    def _ok(status: int):
        if status != 0:
            raise RuntimeError(f'cuSPARSE error {status}')

    def _launch(self):
        if not self.supported:
            raise RuntimeError(self.reason)
        self._ok(_cusparse().cusparseSpMM(self._h, _NON_TRANSPOSE, _NON_TRANSPOSE, C.byref(self._alpha), self._a,
                                          self._b, C.byref(self._beta), self._c, _R_32F, self._alg,
                                          self._ws.data_ptr()))

    @property
    def output(self) -> torch.Tensor:
        return self._y

    def info(self) -> dict:
        return dict(supported=self.supported, reason=self.reason, algorithm=self._alg,
                    workspace_bytes=getattr(self, '_bytes', 0))

    def __del__(self):
        try:
            L = _cusparse()
            torch.cuda.current_stream(self._device).synchronize()
            for h, fn in ((self._c, 'cusparseDestroyDnMat'), (self._b, 'cusparseDestroyDnMat'),
                          (self._a, 'cusparseDestroySpMat'), (self._h, 'cusparseDestroy')):
                if h:
                    getattr(L, fn)(h)
        except Exception:   # noqa: BLE001 -- interpreter shutdown
            pass
