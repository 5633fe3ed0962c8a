"""Row split and format broadcast over NCCL on two GPUs (one process each),
for BOO and PBR, against the oracle.  NVLS is switched off (plain NCCL rings) and every
collective has a bounded process-group timeout."""

import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

from oracle import oracle as O
from tests.conftest import TOL, abs_bound

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(torch.cuda.device_count() < 2, reason='requires two GPUs')]


def _free_port():
    with socket.socket() as s:
        s.bind(('127.0.0.1', 0))
        return s.getsockname()[1]


def _worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR='127.0.0.1', MASTER_PORT=str(port), RANK=str(rank),
                      WORLD_SIZE=str(world), LOCAL_RANK=str(rank), NCCL_NVLS_ENABLE='0')
    try:
        import spmm_b200 as S
        from spmm_b200 import distributed as D
        from spmm_b200 import workloads
        dev = torch.device('cuda', rank)
        torch.cuda.set_device(dev)
        D.init('nccl', timeout_s=60, device=dev)
        import torch.distributed as dist
        mat = workloads.fem3d(n=9)
        rows, cols = mat.shape
        rl, cl = np.arange(rows) // 32, np.arange(cols) // 32
        xh = torch.from_numpy(np.random.default_rng(2).standard_normal((cols, 128)).astype(np.float32))
        full = O.boo_build(mat.indptr, mat.indices, mat.data, rows, cols, rl, cl)
        full.update(rows=rows, cols=cols)
        ref = O.boo_matmul(full, xh.numpy())
        bound = abs_bound(mat.indptr, mat.indices, mat.data, xh.numpy())
        msgs = []
        # row split: X broadcast once, shard products, Y gathered
        rs = D.RowSplitBOO(mat, rl, cl, dev)
        x = D.broadcast_dense(xh.to(dev) if rank == 0 else None, (cols, 128), torch.float32, dev)
        y = rs.gather(rs.matmul(x)).cpu().numpy()
        msgs.append(bool(np.all(np.abs(y - ref) <= TOL[np.dtype(np.float32)] * bound + 1e-30)))
        # feature split: A built on rank 0, broadcast; each rank its 64-column slab
        A = None
        if rank == 0:
            A = S.csr_to_boo(mat, cluster='identity', target_nr=32, target_nc=32).to(dev)
        A = D.broadcast_boo(A, dev)
        slab = xh[:, rank * 64:(rank + 1) * 64].contiguous().to(dev)
        ys = S.boo_matmul(A, slab).cpu().numpy()
        msgs.append(bool(np.all(np.abs(ys - ref[:, rank * 64:(rank + 1) * 64])
                                <= TOL[np.dtype(np.float32)] * bound[:, rank * 64:(rank + 1) * 64] + 1e-30)))
        # PBR: row split over stripes, and the format broadcast for a feature split
        um = workloads.uniform(n=6000, seed=4)
        ux = torch.from_numpy(np.random.default_rng(3).standard_normal((6000, 64)).astype(np.float32))
        ufull = O.pbr_build(um.indptr, um.indices, um.data, 6000, 6000, 8, 8, 1)
        ufull.update(rows=6000, cols=6000)
        uref = O.pbr_matmul(ufull, ux.numpy())
        ubound = abs_bound(um.indptr, um.indices, um.data, ux.numpy())
        rp = D.RowSplitPBR(um, 8, 8, 1, dev)
        uxd = D.broadcast_dense(ux.to(dev) if rank == 0 else None, (6000, 64), torch.float32, dev)
        uy = rp.gather(rp.matmul(uxd)).cpu().numpy()
        msgs.append(bool(np.all(np.abs(uy - uref) <= TOL[np.dtype(np.float32)] * ubound + 1e-30)))
        P = S.csr_to_pbr(um, 8, 8, 1).to(dev) if rank == 0 else None
        P = D.broadcast_pbr(P, dev)
        py = S.pbr_matmul(P, uxd).cpu().numpy()
        msgs.append(bool(np.all(np.abs(py - uref) <= TOL[np.dtype(np.float32)] * ubound + 1e-30)))
        D.barrier()
        dist.destroy_process_group()
        q.put((rank, 'ok' if all(msgs) else f'mismatch {msgs}'))
    except Exception as e:      # noqa: BLE001
        q.put((rank, f'exception {type(e).__name__}: {e}'))


@pytest.mark.timeout(600)
def test_row_split_and_feature_split_two_gpus():
    ctx = mp.get_context('spawn')
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(480)
    for p in procs:
        if p.is_alive():
            p.kill()
            p.join()
            pytest.fail('rank process did not finish')
    out = {}
    while not q.empty():
        r, m = q.get()
        out[r] = m
    assert out == {0: 'ok', 1: 'ok'}, out
