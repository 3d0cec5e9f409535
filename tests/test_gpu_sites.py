"""Parity of every site kernel with the CPU oracle, through the C ABI, on a B200.

Bar: bit-exact for generators, moves, gathers, elementwise maps, FIR, conv2d
and strict matmul (the interpreter's separately rounded, in-order folds);
the sum fold is a fixed tree in f64 and must stay within 1e-6 * sum|x| of
the exact sum (and of the left fold, up to that fold's own error)."""
import json
import os

import numpy as np
import pytest
import torch

import flow_b200 as fb
import oracle as o
from _gpu import dev, empty_f32, first_diff, host, same_bits

pytestmark = pytest.mark.gpu

GOLD = json.load(open(os.path.join(os.path.dirname(__file__), "golden", "reference_outputs.json")))


@pytest.fixture(scope="module")
def ctx():
    c = fb.Context((0,))
    yield c
    c.close()


def int_a(n):
    return o.affine(n, 7, 13, 101, 50)


def int_b(n):
    return o.affine(n, 7, 57, 101, 50)


def int_w(n):
    return o.affine(n, 5, 3, 31, 15)


# ---- generators ------------------------------------------------------------------

@pytest.mark.parametrize("seed,offset,kind", [(0, 0, fb.U11), (1, 12345, fb.U01), (3, (1 << 31) - 100, fb.U11),
                                              (-5, 7, fb.U01)])
def test_gen_matches_oracle(ctx, seed, offset, kind):
    n = 100003
    out = empty_f32(n)
    ctx.gen(out, seed, offset, kind)
    assert same_bits(host(out), o.gen(n, seed, offset, kind))


@pytest.mark.parametrize("rng", [1 << 20, 1 << 28, 1000])
def test_gen_index_matches_oracle(ctx, rng):
    n = 65537
    out = torch.empty(n, dtype=torch.int32, device="cuda")
    ctx.gen_index(out, 3, 99, rng)
    assert np.array_equal(host(out), o.gen_index(n, 3, 99, rng))


def test_affine_iota_fill_widen(ctx):
    n = 1052676
    out = empty_f32(n)
    ctx.gen_affine(out, 7, 13, 101, 50)
    assert same_bits(host(out), int_a(n))
    iota = torch.empty(1000, dtype=torch.int32, device="cuda")
    ctx.iota(iota)
    assert np.array_equal(host(iota), np.arange(1000, dtype=np.int32))
    wid = empty_f32(1000)
    ctx.widen(dev(np.array([16777217, -3] * 500, np.int32)), wid)
    assert same_bits(host(wid), np.array([16777217, -3] * 500, np.int32).astype(np.float32))
    f = empty_f32(77)
    ctx.fill(f, -0.0)
    assert same_bits(host(f), np.full(77, -0.0, np.float32))


# ---- saxpy / zip ------------------------------------------------------------------------

@pytest.mark.parametrize("n", [1, 3, 4, 1000, (1 << 20) + 3])
def test_saxpy_random(ctx, n):
    x, y0 = o.gen(n, 1, 0), o.gen(n, 1, n)
    out = empty_f32(n)
    ctx.saxpy(2.5, dev(x), dev(y0), out)
    assert same_bits(host(out), o.saxpy(2.5, x, y0))


def test_saxpy_misaligned_and_inplace(ctx):
    n = 4099
    x, y0 = o.gen(n + 1, 1, 0), o.gen(n + 1, 1, 9999)
    dx, dy = dev(x), dev(y0)
    ctx.saxpy(-1.25, dx[1:], dy[1:], dy[1:])  # 4-byte offset views, y aliasing y0
    want = o.saxpy(-1.25, x[1:].copy(), y0[1:].copy())
    assert same_bits(host(dy)[1:], want) and host(dy)[0] == y0[0]


@pytest.mark.parametrize("n", [256, 1048576])
def test_saxpy_golden(ctx, n):
    out = empty_f32(n)
    ctx.saxpy(2.5, dev(int_a(n)), dev(int_w(n)), out)
    y = host(out)
    want = [c["values"] for c in GOLD["ladder2"] if c["shape"] == "saxpy" and c["size"] == n][0]
    assert ["%g" % y[0], "%g" % y[-1]] == want


@pytest.mark.parametrize("op", [fb.OP_ADD, fb.OP_SUB, fb.OP_MUL, fb.OP_DIV, fb.OP_MOD])
def test_zip_map_ops(ctx, op):
    n = 10007
    x = o.gen(n, 2, 0) * np.float32(100)
    y = o.gen(n, 2, n)
    y[::97] = 0.0  # division and fmod by zero give IEEE inf / NaN, no trap
    out = empty_f32(n)
    ctx.zip_map(op, dev(x), dev(y), out)
    assert same_bits(host(out), o.zip_map(op, x, y))


# ---- move sites ---------------------------------------------------------------------------

@pytest.mark.parametrize("side", [16, 1024])
def test_transpose_golden(ctx, side):
    a = int_a(side * side)
    out = empty_f32(side * side)
    site = fb.transpose_site(side, side)
    ctx.transpose(site, dev(a), out)
    rc, want = o.move_site(o.transpose_site(side, side), a)
    assert rc == 0 and same_bits(host(out), want)
    gold = [c["values"] for c in GOLD["ladder2"] if c["shape"] == "transpose" and c["size"] == side][0]
    assert ["%g" % host(out)[0], "%g" % host(out)[-1]] == gold


@pytest.mark.parametrize("R,C", [(37, 1000), (1000, 37), (1, 5), (4096, 4096), (33, 33)])
def test_transpose_shapes(ctx, R, C):
    a = o.gen(R * C, 1, 0)
    out = empty_f32(R * C)
    ctx.transpose(fb.transpose_site(R, C), dev(a), out)
    assert same_bits(host(out), a.reshape(R, C).T.ravel())


def test_move_site_generic_and_trap(ctx):
    a = o.gen(5000, 1, 0)
    s = fb.MoveSite(width=40, rows=30, cq=7, cr=3, len=5000)
    out = empty_f32(1200)
    ctx.transpose(s, dev(a), out)
    rc, want = o.move_site(o.MoveSite(40, 30, 7, 3, 5000), a)
    assert rc == 0 and same_bits(host(out), want)
    s.len = 7 * 29 + 3 * 39  # one short of the largest address
    with pytest.raises(fb.MapalTrap) as e:
        ctx.transpose(s, dev(a), out)
    assert e.value.kind == "index_oob" and e.value.exit_code == 101


# ---- gather -----------------------------------------------------------------------------------

@pytest.mark.parametrize("n", [1, 7, 1 << 20, (1 << 20) + 5])
def test_gather_random(ctx, n):
    x = o.gen(1 << 20, 1, 0)
    idx = o.gen_index(n, 1, 1 << 20, 1 << 20)
    out = empty_f32(n)
    ctx.gather(dev(x), dev(idx), out)
    rc, want = o.gather(x, idx)
    assert rc == 0 and same_bits(host(out), want)


def test_gather_golden(ctx):
    n = 1048576
    idx = ((np.arange(n, dtype=np.int64) * 1021 + 12347) % n).astype(np.int32)
    out = empty_f32(n)
    ctx.gather(dev(int_a(n)), dev(idx), out)
    y = host(out)
    gold = [c["values"] for c in GOLD["ladder2"] if c["shape"] == "gather" and c["size"] == n][0]
    assert ["%g" % y[0], "%g" % y[-1]] == gold


@pytest.mark.parametrize("bad", [-1, 1000, -(1 << 31)])
def test_gather_trap_then_recovers(ctx, bad):
    x = dev(o.gen(1000, 1, 0))
    idx = np.arange(64, dtype=np.int32)
    idx[37] = bad
    out = empty_f32(64)
    with pytest.raises(fb.MapalTrap) as e:
        ctx.gather(x, dev(idx), out)
    assert e.value.kind == "index_oob"
    idx[37] = 999  # the flag was cleared: the next call is clean
    ctx.gather(x, dev(idx), out)
    assert host(out)[37] == o.gen(1000, 1, 0)[999]


def test_async_trap_surfaces_at_synchronize(ctx):
    x = dev(o.gen(100, 1, 0))
    out = empty_f32(8)
    ctx.set_sync(False)
    try:
        ctx.gather(x, dev(np.array([0, 1, 2, 3, 4, 5, 6, 100], np.int32)), out)
        with pytest.raises(fb.MapalTrap):
            ctx.synchronize()
        ctx.synchronize()  # cleared
    finally:
        ctx.set_sync(True)


# ---- sum fold --------------------------------------------------------------------------------

@pytest.mark.parametrize("n", [0, 1, 5, 1000, 1 << 20, (1 << 20) + 7, 3 << 22])
def test_fold_sum_tolerance(ctx, n):
    x = o.gen(n, 1, 0, fb.U01)
    out = empty_f32(1)
    ctx.fold_sum(dev(x), out, seed=0.0)
    got = float(host(out)[0])
    exact = o.sum_f64(0.0, x)
    tol = 1e-6 * max(o.sum_abs_f64(x), 1e-30)
    assert abs(got - exact) <= tol
    fold = o.fold_sum(0.0, x)  # the interpreter's left fold, with its own rounding error
    assert abs(got - fold) <= abs(fold - exact) + tol
    ctx.fold_sum(dev(x), out, seed=0.0)
    assert float(host(out)[0]) == got  # deterministic run to run


@pytest.mark.parametrize("n", [256, 1048576])
def test_fold_sum_golden(ctx, n):
    out = empty_f32(1)
    ctx.fold_sum(dev(int_a(n)), out)
    gold = [c["values"] for c in GOLD["ladder2"] if c["shape"] == "reduce" and c["size"] == n][0]
    assert ["%g" % host(out)[0]] == gold


def test_fold_sum_seed_and_specials(ctx):
    x = np.array([1.0, 2.0, 3.0], np.float32)
    out = empty_f32(1)
    ctx.fold_sum(dev(x), out, seed=10.0)
    assert host(out)[0] == 16.0
    x = np.array([1.0, np.inf, -np.inf], np.float32)
    ctx.fold_sum(dev(x), out)
    assert np.isnan(host(out)[0])


@pytest.mark.parametrize("n", [0, 1, 3, 2047, 2048, 2049, 8195, 300007, (1 << 20) + 5])
@pytest.mark.parametrize("offset", [0, 1])
def test_fold_sum_strict_bit_exact(ctx, n, offset):
    # the interpreter's order, so fractional inputs give its exact last bits;
    # offset 1 makes the input pointer 4-byte but not 16-byte aligned
    x = o.gen(n + offset, 3, 0, fb.U11)
    xd = dev(x)[offset:]
    out = empty_f32(1)
    ctx.fold_sum_strict(xd, out, seed=0.75)
    assert same_bits(host(out), np.array([o.fold_sum(0.75, x[offset:])], np.float32))


@pytest.mark.parametrize("n", [0, 1, 1000, (1 << 20) + 3, 1 << 24])
def test_fold_sum_i32_wrapping_exact(ctx, n):
    rng = np.random.default_rng(n)
    x = rng.integers(-2**31, 2**31, size=n, dtype=np.int64).astype(np.int32)
    out = torch.empty(1, dtype=torch.int32, device="cuda")
    ctx.fold_sum_i32(dev(x), out, seed=-123)
    want = np.int64(-123) + x.astype(np.int64).sum()
    want = ((int(want) + 2**31) % 2**32) - 2**31
    assert int(host(out)[0]) == want


def test_fold_sum_strict_specials(ctx):
    out = empty_f32(1)
    ctx.fold_sum_strict(dev(np.array([1e30, -1e30, 1.0, np.float32(2.0**-30)], np.float32)), out)
    assert host(out)[0] == np.float32(1.0) + np.float32(2.0**-30)
    ctx.fold_sum_strict(dev(np.array([1.0, np.inf, -np.inf], np.float32)), out)
    assert np.isnan(host(out)[0])


# ---- FIR ---------------------------------------------------------------------------------------

@pytest.mark.parametrize("n", [256, 65536, 1048576])
def test_fir_golden(ctx, n):
    x, w = int_a(n + 63), int_w(64)
    out = empty_f32(n)
    ctx.fir(fb.fir_site(n, 64), dev(w), dev(x), out)
    assert same_bits(host(out), o.fir(w, x, n))
    gold = [c["values"] for c in GOLD["shapes"] if c["shape"] == "fir" and c["size"] == n][0]
    assert ["%.9g" % host(out)[0], "%.9g" % host(out)[-1]] == gold


@pytest.mark.parametrize("n,taps", [(1, 1), (100, 7), (1000, 8), (4097, 16), ((1 << 20) - 63, 64), (3000, 100),
                                    (10000, 1000), (3, 16), (2049, 32), (2047, 64), (6145, 64), (100003, 32)])
def test_fir_random(ctx, n, taps):
    x = o.gen(n + taps - 1, 1, 0)
    w = o.gen(taps, 1, n + taps - 1)
    out = empty_f32(n)
    ctx.fir(fb.fir_site(n, taps), dev(w), dev(x), out)
    want = o.fir(w, x, n)
    assert same_bits(host(out), want), first_diff(host(out), want)


def test_fir4_acceptance(ctx):
    g = GOLD["fir4"]
    s = fb.fir_site(1, 4)
    s.b.base, s.b.len = g["window_start"], len(g["signal"])
    out = empty_f32(1)
    ctx.fir(s, dev(np.array(g["coeffs"], np.float32)), dev(np.array(g["signal"], np.float32)), out)
    assert fb.render_f32(float(host(out)[0])) == g["output"]


# ---- conv2d ---------------------------------------------------------------------------------------

@pytest.mark.parametrize("side", [16, 20, 92, 512, 1024])
def test_conv2d_golden(ctx, side):
    stride = side + 2
    img, w = int_a(stride * stride), int_w(9)
    out = empty_f32(side * side)
    ctx.conv2d_3x3(fb.conv2d_site(side, side, stride, stride * stride), dev(w), dev(img), out)
    want = o.conv2d_3x3(w, img, stride, side, side)
    assert same_bits(host(out), want), first_diff(host(out), want)
    gold = [c["values"] for c in GOLD["shapes"] if c["shape"] == "conv2d" and c["size"] == side][0]
    assert ["%.9g" % host(out)[0], "%.9g" % host(out)[-1]] == gold


@pytest.mark.parametrize("H,W", [(1024, 1024), (3, 3), (5, 300), (300, 7), (130, 129)])
def test_conv2d_random_valid(ctx, H, W):
    img = o.gen(H * W, 1, 0)
    w = o.gen(9, 1, H * W)
    R, C = H - 2, W - 2
    out = empty_f32(R * C)
    ctx.conv2d_3x3(fb.conv2d_site(R, C, W, H * W), dev(w), dev(img), out)
    want = o.conv2d_3x3(w, img, W, R, C)
    assert same_bits(host(out), want), first_diff(host(out), want)


@pytest.mark.parametrize("H,W,base", [(4098, 4098, 0), (2051, 3001, 0), (2051, 3001, 3), (1800, 6000, 1)])
def test_conv2d_large_sites(ctx, H, W, base):
    # sites of four or more 16-row strips per SM take the persistent,
    # double-buffered kernel: square, ragged, and an image that starts off
    # the 16-byte boundary (its first rows are staged by the edge path)
    img = o.gen(base + H * W, 2, 0)
    w = o.gen(9, 2, base + H * W)
    R, C = H - 2, W - 2
    site = fb.conv2d_site(R, C, W, base + H * W)
    site.b.base = base
    out = empty_f32(R * C)
    ctx.conv2d_3x3(site, dev(w), dev(img), out)
    want = o.conv2d_3x3(w, img[base:].copy(), W, R, C)
    assert same_bits(host(out), want), first_diff(host(out), want)


# ---- matmul strict ----------------------------------------------------------------------------------

@pytest.mark.parametrize("case", GOLD["matmul_known_answers"], ids=lambda c: f"n{c['n']}")
def test_matmul_known_answers(ctx, case):
    n = case["n"]
    A, B = int_a(n * n), int_b(n * n)
    C = empty_f32(n * n)
    ctx.matmul(fb.matmul_site(n, n, n), dev(A), dev(B), C)
    c = host(C)
    assert (c[0], c[-1]) == (case["c0"], case["clast"])
    if n <= 512:
        assert same_bits(c, o.matmul(A, B, n, n, n, threads=8))


@pytest.mark.parametrize("M,N,K", [(5, 20, 7), (6, 32, 5), (33, 65, 70), (128, 128, 128), (1, 1, 1),
                                   (257, 129, 1000), (1024, 1024, 1024), (300, 4097, 19), (127, 128, 129),
                                   # row blocks of the sharded 4096^2 site (whole waves + 64x64 remainder)
                                   (512, 4096, 64), (2048, 4096, 40), (1000, 4000, 33),
                                   # 128 x 112 tiles (the plan for these row blocks), ragged rows,
                                   # columns and k, a row stride that is not a multiple of 4
                                   (500, 4000, 70), (1024, 4096, 130), (640, 3001, 70)])
def test_matmul_random(ctx, M, N, K):
    A = o.gen(M * K, 0, 0)
    B = o.gen(K * N, 0, M * K)
    C = empty_f32(M * N)
    ctx.matmul(fb.matmul_site(M, N, K), dev(A), dev(B), C)
    want = o.matmul(A, B, M, N, K, threads=8)
    assert same_bits(host(C), want), first_diff(host(C), want)


def test_matmul_4096_sampled_rows(ctx):
    n = 4096
    A = o.gen(n * n, 2, 0)
    B = o.gen(n * n, 2, n * n)
    C = empty_f32(n * n)
    ctx.matmul(fb.matmul_site(n, n, n), dev(A), dev(B), C)
    c = host(C).reshape(n, n)
    for r0 in (0, 1337, 4088):  # 8 full rows per sample block
        want = o.matmul(A, B, n, n, n, row0=r0, row1=r0 + 8, threads=8).reshape(n, n)[r0:r0 + 8]
        assert same_bits(c[r0:r0 + 8], want), first_diff(c[r0:r0 + 8], want)


def test_matmul_padded_rows_and_zero_signs(ctx):
    M, N, K, lda, ldb = 40, 24, 18, 21, 29
    A = o.gen(M * lda, 4, 0)
    B = o.gen(K * ldb, 4, 77777)
    A[:lda] = -0.0  # row 0: every product is -0; acc starts at +0 so the cell is +0
    s = fb.matmul_site(M, N, K, lda=lda, ldb=ldb)
    C = empty_f32(M * N)
    ctx.matmul(s, dev(A), dev(B), C)
    rc, want = o.tile_site(o.TileSite.from_buffer_copy(bytes(s)), A, B)
    assert rc == 0 and same_bits(host(C), want)
    assert np.all(host(C)[:N].view(np.uint32) == 0)


def test_matmul_n112_padded_rows_and_zero_signs(ctx):
    # 4 tile rows x 2500 columns: 92 tiles of 128 x 112 (one wave) against 80 of 128 x 128
    M, N, K, lda, ldb = 512, 2500, 37, 41, 2503
    A = o.gen(M * lda, 6, 0)
    B = o.gen(K * ldb, 6, 99991)
    A[:lda] = -0.0
    s = fb.matmul_site(M, N, K, lda=lda, ldb=ldb)
    s.seed = -0.0
    C = empty_f32(M * N)
    ctx.matmul(s, dev(A), dev(B), C)
    rc, want = o.tile_site(o.TileSite.from_buffer_copy(bytes(s)), A, B)
    assert rc == 0 and same_bits(host(C), want), first_diff(host(C), want)


def test_matmul_k0_is_seed(ctx):
    s = fb.matmul_site(3, 5, 0)
    s.seed = 2.5
    C = empty_f32(15)
    ctx.matmul(s, dev(np.zeros(1, np.float32)), dev(np.zeros(1, np.float32)), C)
    assert np.all(host(C) == 2.5)


def test_matmul_rejects_non_matmul_record_and_traps_oob(ctx):
    s = fb.matmul_site(4, 4, 4)
    s.b.clane = 2
    with pytest.raises(fb.Unsupported):
        ctx.matmul(s, dev(np.zeros(16, np.float32)), dev(np.zeros(40, np.float32)), empty_f32(16))
    s = fb.matmul_site(4, 4, 4)
    s.b.len = 15
    with pytest.raises(fb.MapalTrap):
        ctx.matmul(s, dev(np.zeros(16, np.float32)), dev(np.zeros(16, np.float32)), empty_f32(16))


# ---- any tile site -------------------------------------------------------------------------------------

def test_tile_site_generic_record(ctx):
    s = fb.TileSite()
    s.rows, s.c, s.k = 17, 23, 11
    s.a.base, s.a.ci, s.a.ck, s.a.clane = 3, 5, 2, 1
    s.b.base, s.b.ci, s.b.ck, s.b.clane = 1, 0, 7, 3
    s.b.ksplit.div, s.b.ksplit.cq, s.b.ksplit.cr = 4, 2, 5
    s.seed = -1.5
    s.mul_a_first, s.add_acc_first = 0, 0
    s.a.len, s.b.len = 5000, 5000
    a, b = o.gen(5000, 6, 0), o.gen(5000, 6, 5000)
    out = empty_f32(17 * 23)
    ctx.tile_site(s, dev(a), dev(b), out)
    rc, want = o.tile_site(o.TileSite.from_buffer_copy(bytes(s)), a, b)
    assert rc == 0 and same_bits(host(out), want)


def test_tile_site_dispatches_shapes(ctx):
    n = 100
    x, w = o.gen(n + 63, 1, 0), o.gen(64, 1, 500)
    out = empty_f32(n)
    ctx.tile_site(fb.fir_site(n, 64), dev(w), dev(x), out)
    assert same_bits(host(out), o.fir(w, x, n))


def test_launch_count_moves(ctx):
    before = fb.launch_count()
    C = empty_f32(64 * 64)
    ctx.matmul(fb.matmul_site(64, 64, 64), dev(o.gen(4096, 1, 0)), dev(o.gen(4096, 1, 4096)), C)
    assert fb.launch_count() > before


def test_profile(ctx):
    p = ctx.profile()
    assert p.cc_major == 10 and p.sm_count >= 100 and p.tmem_bytes_per_sm == 256 * 1024
    assert p.l2_bytes > 64 << 20 and p.smem_per_block_optin >= 200 * 1024
