"""Generates the golden fixtures in this directory from the REFERENCE itself.

Run here, where the reference sources exist:
    python oracle/build_ref.py          # reference core -> oracle/_ref/
    python tests/golden/gen_golden.py   # -> tests/golden/*.npz

Inputs are seeded; outputs come from the reference's compiled core
(torch_fast_spdmm_core: csr_to_boo, boo_batched_matmul_cpu, boo_to_csr,
csr_to_pbr, pbr_batched_matmul_cpu, pbr_to_csr) and its clustering module
(torch_fast_spdmm/torch_fast_spdmm/clustering.py, loaded by file path).  The
fixtures are what the oracle and the GPU path are checked against on a machine
without the reference.
"""

from __future__ import annotations

import importlib.util
import json
import os
import sys

import numpy as np
import scipy.sparse as sp
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)
from oracle.build_ref import DEFAULT_REFERENCE, load_reference  # noqa: E402

BOO_FIELDS = ('row_grp_ptr', 'row_ids', 'col_grp_ptr', 'col_ids', 'blk_row_grp', 'blk_col_grp',
              'blk_nz_ptr', 'blk_shift', 'nz_idx', 'nz_val', 'rem_indptr', 'rem_col_ind',
              'rem_vals', 'tail_row', 'tail_col', 'tail_val')
PBR_FIELDS = ('block_codes', 'block_coords', 'block_offsets', 'block_data',
              'remainder_indptr', 'remainder_col_ind', 'remainder_data')


def _rand_csr(rng, rows, cols, density, dtype, idt, unsorted=False, dups=False):
    m = sp.random(rows, cols, density=density, format='csr', random_state=int(rng.integers(1 << 30)),
                  dtype=np.float64)
    m.data = rng.standard_normal(m.nnz)
    m = m.astype(dtype)
    indptr, indices, data = m.indptr.astype(idt), m.indices.astype(idt), m.data
    if unsorted or dups:
        ind, dat, ptr = [], [], [0]
        for r in range(rows):
            c = list(indices[indptr[r]:indptr[r + 1]])
            v = list(data[indptr[r]:indptr[r + 1]])
            if dups and c:
                k = int(rng.integers(len(c)))
                c.append(c[k])
                v.append(dtype(rng.standard_normal()))
            if unsorted and len(c) > 1:
                p = rng.permutation(len(c))
                c = [c[i] for i in p]
                v = [v[i] for i in p]
            ind += c
            dat += v
            ptr.append(len(ind))
        indptr = np.array(ptr, dtype=idt)
        indices = np.array(ind, dtype=idt)
        data = np.array(dat, dtype=dtype)
    return indptr, indices, data


def main():
    core = load_reference()
    if core is None:
        sys.exit('build the reference core first: python oracle/build_ref.py')
    spec = importlib.util.spec_from_file_location(
        'ref_clustering', os.path.join(DEFAULT_REFERENCE, 'torch_fast_spdmm', 'torch_fast_spdmm',
                                       'clustering.py'))
    clus = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(clus)

    rng = np.random.default_rng(20261201)
    boo, pbr, cl, manifest = {}, {}, {}, {'boo': [], 'pbr': [], 'clustering': []}

    # ---- BOO -----------------------------------------------------------------
    policies = (0, 2, 3)
    for i in range(36):
        rows, cols = int(rng.integers(1, 90)), int(rng.integers(1, 90))
        dtype = np.float32 if i % 2 == 0 else np.float64
        idt = np.int32 if i % 3 else np.int64
        unsorted, dups = i % 9 == 4, i % 9 == 7
        ip, ix, dv = _rand_csr(rng, rows, cols, float(rng.uniform(0.02, 0.4)), dtype, idt,
                               unsorted, dups)
        rl = rng.integers(0, max(1, rows // int(rng.integers(1, 9))), size=rows).astype(np.int32)
        clab = rng.integers(0, max(1, cols // int(rng.integers(1, 9))), size=cols).astype(np.int32)
        pol, thr, order = policies[i % 3], int(rng.integers(0, 7)), (i // 3) % 2
        b = core.csr_to_boo(ip, ix, dv, rows, cols, rl, clab, pol, thr, order)
        x = rng.standard_normal((2, cols, int(rng.integers(1, 20)))).astype(dtype)
        y = core.boo_batched_matmul_cpu(b, torch.from_numpy(x)).numpy()
        cp = np.zeros(rows + 1, idt)
        ci = np.zeros(dv.size, idt)
        cd = np.zeros(dv.size, dtype)
        core.boo_to_csr(b, cp, ci, cd)
        p = f'b{i}/'
        boo.update({p + 'indptr': ip, p + 'indices': ix, p + 'data': dv, p + 'row_labels': rl,
                    p + 'col_labels': clab, p + 'x': x, p + 'y': y, p + 'csr_indptr': cp,
                    p + 'csr_indices': ci, p + 'csr_data': cd})
        for f in BOO_FIELDS:
            boo[p + f] = np.asarray(getattr(b, f)).copy()
        manifest['boo'].append(dict(case=i, rows=rows, cols=cols, policy=pol, threshold=thr,
                                    order=order, max_nr=int(b.max_nr), max_nc=int(b.max_nc),
                                    max_nnz_blk=int(b.max_nnz_blk), total_nnz=int(b.total_nnz),
                                    unsorted=unsorted, dups=dups))
    # the uint16 overflow case must be rejected by both
    manifest['boo_overflow'] = dict(rows=257, cols=256, entry=[256, 255])

    # ---- PBR -----------------------------------------------------------------
    shapes = ((8, 8), (4, 4), (2, 2), (4, 16), (1, 64), (3, 5))
    for i in range(30):
        rows, cols = int(rng.integers(1, 70)), int(rng.integers(1, 70))
        dtype = np.float32 if i % 2 == 0 else np.float64
        idt = np.int32 if i % 3 else np.int64
        ip, ix, dv = _rand_csr(rng, rows, cols, float(rng.uniform(0.02, 0.6)), dtype, idt,
                               unsorted=(i % 10 == 3))
        br, bc = shapes[i % len(shapes)]
        mn = int(rng.integers(1, 9))
        m = core.csr_to_pbr(ip, ix, dv, rows, cols, br, bc, mn)
        x = rng.standard_normal((2, cols, int(rng.integers(1, 20)))).astype(dtype)
        y = core.pbr_batched_matmul_cpu(m, torch.from_numpy(x)).numpy()
        cp = np.zeros(rows + 1, idt)
        ci = np.zeros(dv.size, idt)
        cd = np.zeros(dv.size, dtype)
        core.pbr_to_csr(m, cp, ci, cd)
        p = f'p{i}/'
        pbr.update({p + 'indptr': ip, p + 'indices': ix, p + 'data': dv, p + 'x': x, p + 'y': y,
                    p + 'csr_indptr': cp, p + 'csr_indices': ci, p + 'csr_data': cd})
        for f in PBR_FIELDS:
            pbr[p + f] = np.asarray(getattr(m, f)).copy()
        manifest['pbr'].append(dict(case=i, rows=rows, cols=cols, block_rows=br, block_cols=bc,
                                    min_nnz=mn, total_nnz=int(m.total_nnz)))

    # ---- clustering --------------------------------------------------------------
    k = 0
    for meth in ('identity', 'random', 'degree', 'rcm', 'hem'):
        for j in range(3):
            n = int(rng.integers(20, 160))
            a = sp.random(n, n, density=float(rng.uniform(0.02, 0.15)), format='csr',
                          random_state=int(rng.integers(1 << 30)))
            if j == 1:
                a = (a + a.T).tocsr()
            kw = dict(method=meth, target_nr=8 + 4 * j, target_nc=8, max_nr=8 + 4 * j, max_nc=8,
                      max_block_nnz=(None if j else 120), seed=j, feasible_first=bool(j % 2))
            r_l, c_l = clus.cluster_axes(a, **kw)
            p = f'c{k}/'
            cl.update({p + 'indptr': a.indptr.astype(np.int32), p + 'indices': a.indices.astype(np.int32),
                       p + 'data': a.data.astype(np.float32), p + 'row_labels': r_l, p + 'col_labels': c_l})
            manifest['clustering'].append(dict(case=k, n=n, **kw))
            k += 1
    # HEM on structured graphs (grids, meshes, skewed and uniform degrees,
    # dense blocks): many equal similarity weights, so the tie-break order is
    # what decides the labels.  Inputs from this package's seeded generators.
    from spmm_b200 import workloads as W
    structured = (('laplacian2d', W.laplacian2d(12)), ('fem3d', W.fem3d(3)),
                  ('powerlaw', W.powerlaw(400)), ('uniform', W.uniform(300, k=6)),
                  ('blockdiag', W.blockdiag(8, 16)))
    for gname, a in structured:
        for tgt, ff in ((8, True), (16, False)):
            kw = dict(method='hem', target_nr=tgt, target_nc=tgt, max_nr=tgt, max_nc=tgt,
                      max_block_nnz=None, seed=0, feasible_first=ff)
            r_l, c_l = clus.cluster_axes(a, **kw)
            p = f'c{k}/'
            cl.update({p + 'indptr': a.indptr.astype(np.int32), p + 'indices': a.indices.astype(np.int32),
                       p + 'data': a.data.astype(np.float32), p + 'row_labels': r_l, p + 'col_labels': c_l})
            manifest['clustering'].append(dict(case=k, n=int(a.shape[0]), graph=gname, **kw))
            k += 1

    np.savez_compressed(os.path.join(HERE, 'boo_golden.npz'), **boo)
    np.savez_compressed(os.path.join(HERE, 'pbr_golden.npz'), **pbr)
    np.savez_compressed(os.path.join(HERE, 'clustering_golden.npz'), **cl)
    with open(os.path.join(HERE, 'manifest.json'), 'w') as f:
        json.dump(manifest, f, indent=1)
    print('wrote', len(manifest['boo']), 'BOO,', len(manifest['pbr']), 'PBR,',
          len(manifest['clustering']), 'clustering cases')


if __name__ == '__main__':
    main()
