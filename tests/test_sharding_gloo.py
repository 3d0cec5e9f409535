"""The sharded sites' host logic on CPU: two gloo ranks, each taking its
range from the library's partitioning rule (mapal_gpu_shard_range), computing
its shard with the oracle, and combining the way the GPU path does:
concatenation for saxpy / gather / matmul row blocks (bit-exact with the
unsharded site), one f64 all-reduce for the sum (same result on every rank,
within the sum tolerance), and the gather's x replicated by a broadcast."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import flow_b200 as fb
import oracle as o


def _free_port() -> int:
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _gather_concat(local: np.ndarray, world: int) -> np.ndarray:
    parts = [None] * world
    dist.all_gather_object(parts, local)
    return np.concatenate(parts)


def _worker(rank: int, world: int, port: int, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        # saxpy shards (no exchange in the GPU path; concatenation here checks the split)
        n = 10007
        lo, hi = fb.shard_range(n, world, rank)
        x, y0 = o.gen(n, 3, 0), o.gen(n, 3, n)
        y_local = o.saxpy(2.5, x[lo:hi].copy(), y0[lo:hi].copy())
        ok_saxpy = np.array_equal(_gather_concat(y_local, world), o.saxpy(2.5, x, y0))

        # sum: one f64 partial per rank, all-reduced, seed added once
        xs = o.gen(1 << 16, 3, 0, o.U01)
        lo, hi = fb.shard_range(xs.size, world, rank)
        part = torch.tensor([o.sum_f64(0.0, xs[lo:hi].copy())], dtype=torch.float64)
        dist.all_reduce(part)
        total = float(np.float32(1.5 + part.item()))
        allv = [None] * world
        dist.all_gather_object(allv, total)
        exact = o.sum_f64(1.5, xs)
        ok_sum = len(set(allv)) == 1 and abs(total - exact) <= 1e-6 * (o.sum_abs_f64(xs) + 1.5)

        # gather: x replicated from rank 0, idx sharded
        nx = 5000
        xg = o.gen(nx, 4, 0) if rank == 0 else np.zeros(nx, np.float32)
        xt = torch.from_numpy(xg)
        dist.broadcast(xt, src=0)
        idx = o.gen_index(7001, 4, nx, nx)
        lo, hi = fb.shard_range(idx.size, world, rank)
        rc, g_local = o.gather(xt.numpy(), idx[lo:hi].copy())
        rc_full, g_full = o.gather(o.gen(nx, 4, 0), idx)
        ok_gather = rc == 0 and np.array_equal(_gather_concat(g_local, world), g_full)

        # matmul: A row blocks, B replicated, C row blocks; each cell's k order untouched
        M, N, K = 37, 29, 41
        A, B = o.gen(M * K, 5, 0), o.gen(K * N, 5, M * K)
        lo, hi = fb.shard_range(M, world, rank)
        C_local = o.matmul(A, B, M, N, K, row0=lo, row1=hi).reshape(M, N)[lo:hi].ravel().copy()
        ok_mm = np.array_equal(_gather_concat(C_local, world), o.matmul(A, B, M, N, K))
        q.put((rank, ok_saxpy, ok_sum, ok_gather, ok_mm))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2])
def test_sharded_host_logic_gloo(world):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = [q.get(timeout=120) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank, *oks in results:
        assert all(oks), (rank, oks)
