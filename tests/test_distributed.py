"""Multi-GPU plumbing on CPU: the row-split partition, the format broadcast,
X broadcast / Y gather over gloo (world_size 2), and a dead rank making the
survivor's next collective fail within the process-group timeout.  Products
on the shards are the oracle's (the GPU product itself is covered by the gpu
tests); the distributed logic is what is checked here."""

import os
import socket
import types

import numpy as np
import pytest
import scipy.sparse as sp
import torch
import torch.multiprocessing as mp

from oracle import oracle as O
from spmm_b200 import boo as B
from spmm_b200 import distributed as D
from spmm_b200 import workloads


def test_nnz_balanced_splits_properties():
    rng = np.random.default_rng(0)
    for trial in range(200):
        n = int(rng.integers(0, 60))
        g = rng.integers(0, 50, size=n)
        parts = int(rng.integers(1, 10))
        b = D.nnz_balanced_splits(g, parts)
        assert b[0] == 0 and b[-1] == n and len(b) == parts + 1
        assert np.all(np.diff(b) >= 0)
        cum = np.concatenate([[0], np.cumsum(g)])
        total = cum[-1]
        gmax = g.max() if n else 0
        for k in range(1, parts):
            assert abs(cum[b[k]] - total * k / parts) <= gmax   # nearest prefix end
    np.testing.assert_array_equal(D.nnz_balanced_splits([5, 5, 5, 5], 2), [0, 2, 4])
    np.testing.assert_array_equal(D.nnz_balanced_splits([], 3), [0, 0, 0, 0])


@pytest.mark.parametrize('labels', ['identity', 'random'])
def test_plan_row_split_covers_rows(labels):
    mat = workloads.powerlaw(n=4000, seed=3)
    rows = mat.shape[0]
    rng = np.random.default_rng(1)
    rl = np.arange(rows) // 32 if labels == 'identity' else rng.permutation(np.arange(rows) // 16)
    for parts in (1, 2, 3, 8):
        shards = D.plan_row_split(mat.indptr, rl, parts)
        allrows = np.concatenate([s.rows for s in shards])
        assert np.array_equal(np.sort(allrows), np.arange(rows))
        assert sum(s.nnz for s in shards) == mat.nnz
        for s in shards:
            assert np.all(np.diff(s.rows) > 0)
            assert np.all((rl[s.rows] >= s.g0) & (rl[s.rows] < s.g1))
            np.testing.assert_array_equal(s.local_labels, rl[s.rows] - s.g0)
        gn = np.bincount(rl, weights=np.diff(mat.indptr))
        assert max(s.nnz for s in shards) <= mat.nnz / parts + gn.max() + 1


def _free_port():
    with socket.socket() as s:
        s.bind(('127.0.0.1', 0))
        return s.getsockname()[1]


def _boo_cpu(ob: dict, sizes: dict):
    """A BOOMatrix whose 'device' arrays are CPU tensors, from oracle arrays."""
    arrays = {}
    for name, tdt in B._DEV_DTYPES.items():
        a = np.asarray(ob[name])
        if name == 'nz_idx':
            a = a.astype(np.uint16).view(np.int16)
        elif name == 'blk_shift':
            a = a.astype(np.uint8)
        elif tdt is None:
            a = a.astype(np.float32)
        else:
            a = a.astype(np.int32)
        arrays[name] = torch.from_numpy(np.ascontiguousarray(a))
    return B._boo_class(np.int32, np.float32)(sizes, types.SimpleNamespace(**arrays))


def _worker(rank, world, port, case, q):
    os.environ.update(MASTER_ADDR='127.0.0.1', MASTER_PORT=str(port), RANK=str(rank),
                      WORLD_SIZE=str(world))
    try:
        D.init(backend='gloo', timeout_s=10 if case == 'fault' else 60)
        import torch.distributed as dist
        if case == 'fault':
            if rank == 1:
                os._exit(3)                      # dies before the collective
            from spmm_b200 import _lib
            try:
                D.all_reduce_max(1.0, 'cpu')
                D.barrier()
                q.put((rank, 'no error'))
            except _lib.SpmmError as e:         # the module's collectives report SPMM_ENCCL
                q.put((rank, f'error: SpmmError {e.status}'))
            except Exception as e:              # noqa: BLE001
                q.put((rank, 'unexpected: ' + type(e).__name__))
            return
        mat = workloads.fem3d(n=6)
        rows, cols = mat.shape
        rl = np.arange(rows) // 32
        cl = np.arange(cols) // 32
        x_full = torch.from_numpy(np.random.default_rng(4).standard_normal((cols, 16)).astype(np.float32))
        if case == 'rowsplit':
            x = D.broadcast_dense(x_full if rank == 0 else None, (cols, 16), torch.float32, 'cpu')
            shards = D.plan_row_split(mat.indptr, rl, world)
            sh = shards[rank]
            sub = D.shard_csr(mat, sh)
            ob = O.boo_build(sub.indptr, sub.indices, sub.data, sub.shape[0], cols, sh.local_labels, cl)
            ob.update(rows=sub.shape[0], cols=cols)
            y_local = torch.from_numpy(O.boo_matmul(ob, x.numpy()))
            y = D.gather_rows(y_local, shards, rows)
            full = O.boo_build(mat.indptr, mat.indices, mat.data, rows, cols, rl, cl)
            full.update(rows=rows, cols=cols)
            ref = O.boo_matmul(full, x_full.numpy())
            bound = np.abs(mat) @ np.abs(x_full.numpy())
            ok = np.all(np.abs(y.numpy() - ref) <= 1e-5 * bound + 1e-30)
            q.put((rank, 'ok' if ok and sh.nnz > 0 else f'mismatch nnz={sh.nnz}'))
        elif case == 'rowsplit_pbr':
            mat = workloads.uniform(n=3000, k=8, seed=2)
            rows, cols = mat.shape
            x_full = torch.from_numpy(np.random.default_rng(5).standard_normal((cols, 24)).astype(np.float32))
            x = D.broadcast_dense(x_full if rank == 0 else None, (cols, 24), torch.float32, 'cpu')
            shards = D.plan_row_split(mat.indptr, D.stripe_labels(rows, 8), world)
            sh = shards[rank]
            assert sh.rows[0] % 8 == 0 and np.all(np.diff(sh.rows) == 1)   # stripe-aligned, contiguous
            sub = D.shard_csr(mat, sh)
            op = O.pbr_build(sub.indptr, sub.indices, sub.data, sub.shape[0], cols, 8, 8, 1)
            op.update(rows=sub.shape[0], cols=cols)
            y_local = torch.from_numpy(O.pbr_matmul(op, x.numpy()))
            y = D.gather_rows(y_local, shards, rows)
            full = O.pbr_build(mat.indptr, mat.indices, mat.data, rows, cols, 8, 8, 1)
            full.update(rows=rows, cols=cols)
            # the shards hold exactly the global matrix's blocks of their stripes
            same_blocks = op['nb'] == int(np.sum((full['block_coords'][0::2] >= sh.rows[0]) &
                                                  (full['block_coords'][0::2] <= sh.rows[-1])))
            ref = O.pbr_matmul(full, x_full.numpy())
            bound = np.abs(mat) @ np.abs(x_full.numpy())
            ok = np.all(np.abs(y.numpy() - ref) <= 1e-5 * bound + 1e-30)
            q.put((rank, 'ok' if ok and same_blocks and sh.nnz > 0 else f'mismatch nnz={sh.nnz} {same_blocks}'))
        elif case == 'broadcast_pbr':
            from spmm_b200 import pbr as P
            full = O.pbr_build(mat.indptr, mat.indices, mat.data, rows, cols, 8, 8, 4)
            src = None
            if rank == 0:
                arr = dict(codes=torch.from_numpy(full['block_codes'].view(np.int64)),
                           coords=torch.from_numpy(full['block_coords'].astype(np.int32)),
                           offsets=torch.from_numpy(full['block_offsets'].astype(np.int32)),
                           data=torch.from_numpy(full['block_data']),
                           rem_indptr=torch.from_numpy(full['remainder_indptr'].astype(np.int32)),
                           rem_col_ind=torch.from_numpy(full['remainder_col_ind'].astype(np.int32)),
                           rem_vals=torch.from_numpy(full['remainder_data']))
                sizes = dict(rows=rows, cols=cols, block_rows=8, block_cols=8,
                             total_nnz=int(mat.nnz), nb=int(full['nb']), nnz_c=int(full['nnz_c']),
                             rem_nnz=int(full['rem_nnz']))
                src = P.PBRMatrixInt32Float(sizes, types.SimpleNamespace(**arr))
            got = D.broadcast_pbr(src, 'cpu')
            same = all(np.array_equal(getattr(got, f), full[f]) for f in O.PBR_FIELDS) \
                and type(got).__name__ == 'PBRMatrixInt32Float'
            q.put((rank, 'ok' if same else 'mismatch'))
        elif case == 'broadcast':
            full = O.boo_build(mat.indptr, mat.indices, mat.data, rows, cols, rl, cl)
            sizes = {k: full[k] for k in D._BOO_SIZE_KEYS}
            src = _boo_cpu(full, sizes) if rank == 0 else None
            got = D.broadcast_boo(src, 'cpu')
            same = all(np.array_equal(np.asarray(getattr(got, f)).astype(np.int64) if f not in
                                      ('nz_val', 'rem_vals', 'tail_val') else getattr(got, f),
                                      np.asarray(full[f]).astype(np.int64) if f not in
                                      ('nz_val', 'rem_vals', 'tail_val') else full[f])
                       for f in O.BOO_FIELDS)
            q.put((rank, 'ok' if same and got.num_blocks() == full['nb'] else 'mismatch'))
        dist.destroy_process_group()
    except Exception as e:                      # noqa: BLE001
        q.put((rank, f'exception {type(e).__name__}: {e}'))


def _run(case, world=2, timeout=120):
    ctx = mp.get_context('spawn')
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, case, q)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout)
    for p in procs:
        if p.is_alive():
            p.kill()
            p.join()
            pytest.fail(f'{case}: rank process did not finish within {timeout} s')
    out = {}
    while not q.empty():
        r, msg = q.get()
        out[r] = msg
    return out, [p.exitcode for p in procs]


@pytest.mark.timeout(300)
def test_row_split_product_over_gloo():
    out, codes = _run('rowsplit')
    assert out == {0: 'ok', 1: 'ok'}, out
    assert codes == [0, 0]


@pytest.mark.timeout(300)
def test_broadcast_boo_over_gloo():
    out, codes = _run('broadcast')
    assert out == {0: 'ok', 1: 'ok'}, out


@pytest.mark.timeout(300)
def test_row_split_pbr_over_gloo():
    out, codes = _run('rowsplit_pbr')
    assert out == {0: 'ok', 1: 'ok'}, out
    assert codes == [0, 0]


@pytest.mark.timeout(300)
def test_broadcast_pbr_over_gloo():
    out, codes = _run('broadcast_pbr')
    assert out == {0: 'ok', 1: 'ok'}, out


@pytest.mark.timeout(300)
def test_dead_rank_fails_collective_within_timeout():
    """A rank that dies before a collective: the survivor's next collective
    fails within the process-group timeout as SpmmError(SPMM_ENCCL)."""
    from spmm_b200 import _lib
    out, codes = _run('fault', timeout=120)
    assert codes[1] == 3
    assert out.get(0, '') == f'error: SpmmError {_lib.SPMM_ENCCL}', out
