"""On-disk BOO / PBR formats: one ``.npz`` file per matrix holding the
format's arrays (exactly the arrays the formats define, in their host dtypes),
the size record and the class name, so a format built once -- HEM
clustering included -- is reloaded without rebuilding.  Loading gives a host
object; ``.to('cuda')`` stages it as any built matrix."""

from __future__ import annotations

import json

import numpy as np

from . import boo as _boo
from . import pbr as _pbr

__all__ = ['save_boo', 'load_boo', 'save_pbr', 'load_pbr']

_FORMAT_VERSION = 1


def _save(path, kind: str, obj, arrays: dict):
    meta = dict(kind=kind, version=_FORMAT_VERSION, cls=type(obj).__name__, sizes=obj._sizes)
    np.savez(path, __meta__=np.frombuffer(json.dumps(meta).encode(), dtype=np.uint8), **arrays)


def _load(path, kind: str):
    with np.load(path, allow_pickle=False) as f:
        meta = json.loads(bytes(f['__meta__']).decode())
        if meta.get('kind') != kind or meta.get('version') != _FORMAT_VERSION:
            raise ValueError(f'{path}: not a version-{_FORMAT_VERSION} {kind.upper()} file')
        arrays = {k: f[k] for k in f.files if k != '__meta__'}
    return meta, arrays


def save_boo(path, boo_mat) -> None:
    """Writes a BOO matrix (host or device resident) to `path` (.npz)."""
    if type(boo_mat).__name__ not in _boo._BOO_TYPE_MAP:
        raise TypeError('save_boo expects a BOOMatrix')
    _save(path, 'boo', boo_mat, boo_mat._host_arrays())


def load_boo(path):
    """A BOOMatrix from a file written by save_boo (host resident)."""
    meta, arrays = _load(path, 'boo')
    if meta['cls'] not in _boo._BOO_TYPE_MAP:
        raise ValueError(f'{path}: unknown BOO class {meta["cls"]!r}')
    cls = getattr(_boo, meta['cls'])
    idt, sdt = _boo._BOO_TYPE_MAP[meta['cls']]
    want = set(_boo._DEV_DTYPES)
    if set(arrays) != want:
        raise ValueError(f'{path}: BOO arrays {sorted(arrays)} do not match {sorted(want)}')
    obj = cls(meta['sizes'], None)
    host = {}
    for name, a in arrays.items():
        if name == 'nz_idx':
            a = a.astype(np.uint16)
        elif name == 'blk_shift':
            a = a.astype(np.uint8)
        elif _boo._DEV_DTYPES[name] is None:
            a = a.astype(sdt)
        else:
            a = a.astype(idt)
        a.setflags(write=False)
        host[name] = a
    obj._host = host
    return obj


_PBR_ARRAYS = ('block_codes', 'block_coords', 'block_offsets', 'block_data', 'remainder_indptr',
               'remainder_col_ind', 'remainder_data')


def save_pbr(path, pbr_mat) -> None:
    """Writes a PBR matrix (host or device resident) to `path` (.npz)."""
    if type(pbr_mat).__name__ not in _pbr._PBR_TYPE_MAP:
        raise TypeError('save_pbr expects a PBRMatrix')
    _save(path, 'pbr', pbr_mat, pbr_mat._host_arrays())


def load_pbr(path):
    """A PBRMatrix from a file written by save_pbr (host resident)."""
    meta, arrays = _load(path, 'pbr')
    if meta['cls'] not in _pbr._PBR_TYPE_MAP:
        raise ValueError(f'{path}: unknown PBR class {meta["cls"]!r}')
    if set(arrays) != set(_PBR_ARRAYS):
        raise ValueError(f'{path}: PBR arrays {sorted(arrays)} do not match {sorted(_PBR_ARRAYS)}')
    idt, sdt = _pbr._PBR_TYPE_MAP[meta['cls']]
    obj = getattr(_pbr, meta['cls'])(meta['sizes'], None)
    host = {}
    for name, a in arrays.items():
        if name == 'block_codes':
            a = a.astype(np.uint64)
        elif name in ('block_data', 'remainder_data'):
            a = a.astype(sdt)
        else:
            a = a.astype(idt)
        a.setflags(write=False)
        host[name] = a
    obj._host = host
    return obj
