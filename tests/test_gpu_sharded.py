"""The sharded sites on real GPUs, through the C ABI.

Single process over every visible GPU (ncclCommInitAll when there are two or
more; the one-device context runs the same entry points without NCCL), and,
with two or more GPUs, one process per GPU joined by an NCCL unique id
(mapal_gpu_ctx_create_rank). Results are checked against the unsharded
oracle: bit-exact for saxpy, gather and strict matmul row blocks; the sum
within 1e-6 * sum|x| and identical on every device."""
import os
import socket

import numpy as np
import pytest
import torch

import flow_b200 as fb
import oracle as o

pytestmark = pytest.mark.gpu

NDEV = torch.cuda.device_count() if torch.cuda.is_available() else 0


def devs():
    return list(range(min(NDEV, 8)))


@pytest.fixture(scope="module")
def ctx():
    c = fb.Context(devs())
    yield c
    c.close()


def on(d, a):
    return torch.from_numpy(np.ascontiguousarray(a)).to(f"cuda:{d}")


def test_saxpy_sharded(ctx):
    n = (1 << 20) + 13
    x, y0 = o.gen(n, 3, 0), o.gen(n, 3, n)
    D = devs()
    spans = [fb.shard_range(n, len(D), i) for i in range(len(D))]
    xs = [on(d, x[lo:hi]) for d, (lo, hi) in zip(D, spans)]
    ys = [on(d, y0[lo:hi]) for d, (lo, hi) in zip(D, spans)]
    outs = [torch.empty(hi - lo, dtype=torch.float32, device=f"cuda:{d}") for d, (lo, hi) in zip(D, spans)]
    ctx.saxpy_sharded(2.5, xs, ys, outs)
    got = np.concatenate([t.cpu().numpy() for t in outs])
    assert np.array_equal(got, o.saxpy(2.5, x, y0))


def test_fold_sum_sharded(ctx):
    n = (1 << 22) + 5
    x = o.gen(n, 3, 0, o.U01)
    D = devs()
    spans = [fb.shard_range(n, len(D), i) for i in range(len(D))]
    xs = [on(d, x[lo:hi]) for d, (lo, hi) in zip(D, spans)]
    outs = [torch.empty(1, dtype=torch.float32, device=f"cuda:{d}") for d in D]
    ctx.fold_sum_sharded(xs, outs, seed=0.25)
    vals = {float(t.cpu().item()) for t in outs}
    assert len(vals) == 1
    got = vals.pop()
    assert abs(got - o.sum_f64(0.25, x)) <= 1e-6 * (o.sum_abs_f64(x) + 0.25)


@pytest.mark.skipif(NDEV < 2, reason="needs two GPUs")
def test_fold_sum_sharded_peer_combine_repeated(ctx, monkeypatch):
    # Back-to-back calls reuse the exchange slots by epoch parity: every call's
    # result is the same on every device and matches the ncclAllReduce path
    # within the reordering tolerance.
    D = devs()
    n = (1 << 20) + 333
    warm = [torch.ones(8, device=f"cuda:{d}") for d in D]
    ctx.fold_sum_sharded(warm, [torch.empty(1, device=f"cuda:{d}") for d in D])  # maps the peers
    monkeypatch.setenv("MAPAL_GPU_PEER_COMBINE", "0")  # the reference context takes ncclAllReduce
    ref_ctx = fb.Context(D)
    try:
        for call in range(12):
            x = o.gen(n, 40 + call, 0, o.U01 if call % 2 else o.U11)
            spans = [fb.shard_range(n, len(D), i) for i in range(len(D))]
            xs = [on(d, x[lo:hi]) for d, (lo, hi) in zip(D, spans)]
            outs = [torch.empty(1, dtype=torch.float32, device=f"cuda:{d}") for d in D]
            ctx.fold_sum_sharded(xs, outs, seed=0.5 * call)
            vals = {float(t.cpu().item()) for t in outs}
            assert len(vals) == 1, (call, vals)
            got = vals.pop()
            assert abs(got - o.sum_f64(0.5 * call, x)) <= 1e-6 * (o.sum_abs_f64(x) + 0.5 * call)
            ref = [torch.empty(1, dtype=torch.float32, device=f"cuda:{d}") for d in D]
            ref_ctx.fold_sum_sharded(xs, ref, seed=0.5 * call)
            assert abs(got - float(ref[0].cpu().item())) <= 1e-6 * (o.sum_abs_f64(x) + 0.5 * call)
    finally:
        ref_ctx.close()


def test_broadcast_then_gather_sharded(ctx):
    nx, n = 1 << 20, (1 << 20) + 3
    x = o.gen(nx, 3, 0)
    idx = o.gen_index(n, 3, nx, nx)
    D = devs()
    xb = [on(D[0], x)] + [torch.full((nx,), float("nan"), device=f"cuda:{d}") for d in D[1:]]
    ctx.broadcast(xb, root=0)
    spans = [fb.shard_range(n, len(D), i) for i in range(len(D))]
    idxs = [on(d, idx[lo:hi]) for d, (lo, hi) in zip(D, spans)]
    outs = [torch.empty(hi - lo, dtype=torch.float32, device=f"cuda:{d}") for d, (lo, hi) in zip(D, spans)]
    ctx.gather_sharded(xb, idxs, outs)
    rc, want = o.gather(x, idx)
    assert rc == 0 and np.array_equal(np.concatenate([t.cpu().numpy() for t in outs]), want)
    bad = idxs[-1].clone()
    bad[0] = nx
    with pytest.raises(fb.MapalTrap):
        ctx.gather_sharded(xb, idxs[:-1] + [bad], outs)


@pytest.mark.parametrize("mode", [fb.STRICT, fb.TF32X3])
def test_matmul_sharded(ctx, mode):
    M, N, K = 1000, 768, 640
    A, B = o.gen(M * K, 4, 0), o.gen(K * N, 4, M * K)
    D = devs()
    spans = [fb.shard_range(M, len(D), i) for i in range(len(D))]
    As = [on(d, A[lo * K:hi * K]) for d, (lo, hi) in zip(D, spans)]
    Bs = [on(D[0], B)] + [torch.full((K * N,), float("nan"), device=f"cuda:{d}") for d in D[1:]]
    Cs = [torch.empty((hi - lo) * N, dtype=torch.float32, device=f"cuda:{d}") for d, (lo, hi) in zip(D, spans)]
    ctx.matmul_sharded(fb.matmul_site(M, N, K), As, Bs, Cs, [hi - lo for lo, hi in spans], root=0, mode=mode)
    got = np.concatenate([t.cpu().numpy() for t in Cs])
    want = o.matmul(A, B, M, N, K, threads=8)
    if mode == fb.STRICT:
        assert np.array_equal(got.view(np.uint32), want.view(np.uint32))
    else:
        A2, B2 = A.reshape(M, K).astype(np.float64), B.reshape(K, N).astype(np.float64)
        scale = np.sqrt((A2 ** 2).sum(1))[:, None] * np.sqrt((B2 ** 2).sum(0))[None, :]
        # the stated 3xTF32 bound
        exact = A2 @ B2
        assert np.max(np.abs(got.reshape(M, N) - exact) / scale) <= 2e-6


# ---- one process per GPU -----------------------------------------------------------------

def _rank_worker(rank, world, port, q):
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        obj = [fb.nccl_unique_id() if rank == 0 else None]
        dist.broadcast_object_list(obj, src=0)
        ctx = fb.Context((rank,), rank=rank, nranks=world, nccl_id=obj[0])
        n = (1 << 21) + 7
        x = o.gen(n, 6, 0, o.U01)
        lo, hi = fb.shard_range(n, world, rank)
        out = torch.empty(1, dtype=torch.float32, device=f"cuda:{rank}")
        ctx.fold_sum_sharded([on(rank, x[lo:hi])], [out], seed=0.0)
        s = float(out.cpu().item())
        # repeated calls through the peer exchange: the same value every time
        xr = on(rank, x[lo:hi])
        again = set()
        for _ in range(9):
            ctx.fold_sum_sharded([xr], [out], seed=0.0)
            again.add(float(out.cpu().item()))
        ok_repeat = again == {s}
        M, N, K = 300, 200, 150
        A, B = o.gen(M * K, 7, 0), o.gen(K * N, 7, M * K)
        mlo, mhi = fb.shard_range(M, world, rank)
        Bd = on(rank, B) if rank == 0 else torch.full((K * N,), float("nan"), device=f"cuda:{rank}")
        C = torch.empty((mhi - mlo) * N, dtype=torch.float32, device=f"cuda:{rank}")
        ctx.matmul_sharded(fb.matmul_site(M, N, K), [on(rank, A[mlo * K:mhi * K])], [Bd], [C], [mhi - mlo])
        want = o.matmul(A, B, M, N, K, row0=mlo, row1=mhi).reshape(M, N)[mlo:mhi].ravel()
        ok_mm = np.array_equal(C.cpu().numpy().view(np.uint32), want.view(np.uint32))
        # the host-array entry: this rank's A and C blocks, B's slices gathered over NVLink
        K2 = 640
        A2, B2 = o.gen(M * K2, 8, 0), o.gen(K2 * N, 8, M * K2)
        Ch = np.full((mhi - mlo) * N, np.nan, np.float32)
        ctx.matmul_host_sharded(fb.matmul_site(M, N, K2), [A2[mlo * K2:mhi * K2].copy()], [B2], [Ch], [mhi - mlo])
        ctx.synchronize()
        want2 = o.matmul(A2, B2, M, N, K2, row0=mlo, row1=mhi).reshape(M, N)[mlo:mhi].ravel()
        ok_mm = ok_mm and np.array_equal(Ch.view(np.uint32), want2.view(np.uint32))
        ok_sum = abs(s - o.sum_f64(0.0, x)) <= 1e-6 * o.sum_abs_f64(x)
        ctx.close()
        q.put((rank, s, ok_sum and ok_repeat, ok_mm))
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(NDEV < 2, reason="needs two GPUs")
def test_one_process_per_gpu():
    import torch.multiprocessing as mp
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    ctxm = mp.get_context("spawn")
    q = ctxm.Queue()
    world = 2
    procs = [ctxm.Process(target=_rank_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = [q.get(timeout=300) for _ in range(world)]
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    assert len({r[1] for r in res}) == 1
    assert all(r[2] and r[3] for r in res), res


def _skip_worker(rank, world, port, q):
    # the exchange's wait is bounded: a rank that never makes the call leaves
    # the other rank with MAPAL_ERR_TIMEOUT after MAPAL_GPU_PEER_WAIT_MS, not a hang
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), MAPAL_GPU_PEER_WAIT_MS="1000",
                      NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        obj = [fb.nccl_unique_id() if rank == 0 else None]
        dist.broadcast_object_list(obj, src=0)
        ctx = fb.Context((rank,), rank=rank, nranks=world, nccl_id=obj[0])
        x = torch.ones(1000, device=f"cuda:{rank}")
        out = torch.empty(1, device=f"cuda:{rank}")
        ctx.fold_sum_sharded([x], [out])  # both ranks: setup and one exchange
        first = float(out.cpu().item())
        status = None
        if rank == 0:  # rank 1 skips the second call
            try:
                ctx.fold_sum_sharded([x], [out])
            except fb.MapalInfraError as e:
                status = e.status
        dist.barrier()
        q.put((rank, first, ctx.sum_combine(), status))
        ctx.close()
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(NDEV < 2, reason="needs two GPUs")
def test_peer_exchange_wait_is_bounded():
    import torch.multiprocessing as mp
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    ctxm = mp.get_context("spawn")
    q = ctxm.Queue()
    procs = [ctxm.Process(target=_skip_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = sorted(q.get(timeout=300) for _ in range(2))
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    assert [r[1] for r in res] == [2000.0, 2000.0]
    assert [r[2] for r in res] == [1, 1]  # the peer combine was in use
    assert res[0][3] == fb.ERR_TIMEOUT and res[1][3] is None
