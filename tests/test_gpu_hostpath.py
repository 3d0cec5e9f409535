"""mapal_gpu_matmul_f32_host: the matmul site on host arrays, transfers overlapped
with the multiply in row blocks. Same bar as the device-pointer entry: strict
mode bit-exact with the oracle, 3xTF32 mode equal to the device entry's bits."""
import numpy as np
import pytest
import torch

import flow_b200 as fb
import oracle as o
from _gpu import dev, empty_f32, first_diff, host, same_bits

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def ctx():
    c = fb.Context((0,))
    yield c
    c.close()


def _site(M, N, K, lda=None, ldb=None, abase=0, bbase=0, seed=0.0):
    s = fb.matmul_site(M, N, K, lda, ldb)
    s.a.base, s.b.base, s.seed = abase, bbase, seed
    s.a.len += abase
    s.b.len += bbase
    return s


def _inputs(s, seed=11):
    A = o.gen(int(s.a.len), seed, 0)
    B = o.gen(int(s.b.len), seed, 1 << 24)
    return A, B


@pytest.mark.parametrize("M,N,K", [(1, 1, 1), (77, 130, 33), (300, 257, 64), (1000, 260, 77),
                                   (1024, 1024, 256), (2049, 96, 40),
                                   # deep K: the strict path uploads and multiplies in k-range phases
                                   (777, 300, 600), (1030, 513, 1000), (520, 64, 4096),
                                   # 128 x 112 tiles, the later k-ranges continuing from C
                                   (512, 2500, 700)])
@pytest.mark.parametrize("pinned", [True, False])
def test_strict_host_bit_exact(ctx, M, N, K, pinned):
    s = _site(M, N, K)
    A, B = _inputs(s)
    want = o.matmul(A, B, M, N, K)
    if pinned:
        Ah = torch.from_numpy(A).pin_memory()
        Bh = torch.from_numpy(B).pin_memory()
        Ch = torch.full((M * N,), float("nan"), dtype=torch.float32).pin_memory()
        ctx.matmul_host(s, Ah, Bh, Ch)
        got = Ch.numpy()
    else:
        got = np.full(M * N, np.nan, np.float32)
        ctx.matmul_host(s, A, B, got)
    assert same_bits(got, want), first_diff(got, want)


@pytest.mark.parametrize("K", [50, 700])
def test_strict_host_padded_and_offset(ctx, K):
    M, N = 600, 200
    s = _site(M, N, K, lda=K + 3, ldb=N + 5, abase=7, bbase=2, seed=0.5)
    A, B = _inputs(s, seed=4)
    rc, want = o.tile_site(o.TileSite.from_buffer_copy(bytes(s)), A, B)  # same record layout
    assert rc == 0
    got = np.full(M * N, np.nan, np.float32)
    ctx.matmul_host(s, A, B, got)
    assert same_bits(got, want), first_diff(got, want)


def test_tf32x3_host_matches_device_entry(ctx):
    M, N, K = 512, 384, 640
    s = _site(M, N, K)
    A, B = _inputs(s, seed=9)
    Cd = empty_f32(M * N)
    ctx.matmul(s, dev(A), dev(B), Cd, fb.TF32X3)
    got = np.full(M * N, np.nan, np.float32)
    ctx.matmul_host(s, A, B, got, fb.TF32X3)
    assert same_bits(got, host(Cd))


def test_host_empty_fold_is_seed(ctx):
    s = _site(5, 7, 0, seed=2.5)
    got = np.full(35, np.nan, np.float32)
    ctx.matmul_host(s, np.zeros(1, np.float32), np.zeros(1, np.float32), got)
    assert np.all(got == 2.5)


def test_host_async_and_reuse(ctx):
    # async mode: the call returns after enqueueing; synchronising the context
    # covers the copies back. Alternating sizes regrows the staging buffer.
    ctx.set_sync(False)
    try:
        for M, N, K in [(700, 300, 90), (1500, 600, 120), (700, 300, 90)]:
            s = _site(M, N, K)
            A, B = _inputs(s, seed=M)
            Ah = torch.from_numpy(A).pin_memory()
            Bh = torch.from_numpy(B).pin_memory()
            Ch = torch.full((M * N,), float("nan"), dtype=torch.float32).pin_memory()
            ctx.matmul_host(s, Ah, Bh, Ch)
            ctx.synchronize()
            assert same_bits(Ch.numpy(), o.matmul(A, B, M, N, K))
    finally:
        ctx.set_sync(True)


def test_host_rejects_bad_records(ctx):
    s = _site(10, 10, 10)
    s.a.len -= 1  # the last A element lies outside the array: the index_oob trap
    A = np.zeros(int(s.a.len), np.float32)
    B = np.zeros(int(s.b.len), np.float32)
    C = np.zeros(100, np.float32)
    with pytest.raises(fb.MapalTrap):
        ctx.matmul_host(s, A, B, C)
    with pytest.raises(fb.Unsupported):
        ctx.matmul_host(fb.fir_site(10, 3), np.zeros(3, np.float32), np.zeros(12, np.float32),
                        np.zeros(10, np.float32))


NDEV = torch.cuda.device_count() if torch.cuda.is_available() else 0


@pytest.mark.skipif(NDEV < 2, reason="needs two GPUs")
@pytest.mark.parametrize("M,N,K,ldb,bbase", [(1000, 300, 1000, None, 0),    # B slices gathered over NVLink
                                             (700, 257, 777, 263, 5),       # padded, offset B; ragged slices
                                             (3, 129, 640, None, 0),        # ranks with no rows still serve B
                                             (500, 200, 100, None, 0)])     # shallow K: per-rank full upload
def test_strict_host_sharded_bit_exact(M, N, K, ldb, bbase):
    D = list(range(min(NDEV, 8)))
    ctx = fb.Context(D)
    try:
        s = _site(M, N, K, ldb=ldb, bbase=bbase, seed=0.25)
        A, B = _inputs(s, seed=21)
        rc, want = o.tile_site(o.TileSite.from_buffer_copy(bytes(s)), A, B)
        assert rc == 0
        spans = [fb.shard_range(M, len(D), i) for i in range(len(D))]
        Bh = torch.from_numpy(B).pin_memory()
        As = [torch.from_numpy(A[lo * K:hi * K].copy()).pin_memory() for lo, hi in spans]
        Cs = [torch.full(((hi - lo) * N,), float("nan"), dtype=torch.float32).pin_memory() for lo, hi in spans]
        for _ in range(2):  # the second call reuses the staging and the comm stream
            ctx.matmul_host_sharded(s, As, [Bh] * len(D), Cs, [hi - lo for lo, hi in spans])
            got = np.concatenate([c.numpy() for c in Cs])
            assert same_bits(got, want), first_diff(got, want)
    finally:
        ctx.close()
