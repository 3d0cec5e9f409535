"""A second, independent restatement in numpy of the seeded stream and of the
small sites on uniform-random inputs, checked against the C oracle. No
reference output pins random f32 inputs (the reference only ever used
integer-valued ones), so this guards the oracle's own arithmetic order."""
import numpy as np
import pytest

import oracle as o

M32 = np.int64(1 << 32)


def wrap(v):
    v = np.asarray(v, dtype=np.int64) % M32
    return np.where(v >= (1 << 31), v - M32, v).astype(np.int64)


def tdiv(a, b):  # Rust i32 `/`: truncation toward zero
    q = np.abs(a) // abs(b)
    return np.where((a < 0) != (b < 0), -q, q)


def trem(a, b):  # Rust i32 `%`: sign of the dividend
    return a - tdiv(a, b) * b


def np_hash(seed, i):
    i = np.asarray(i, dtype=np.int64)
    h = wrap(wrap(i * 1103515245) + wrap(np.int64(seed) * 1640531527 + 12345))
    for _ in range(3):
        h = wrap(wrap(h * h) + tdiv(h, 65536) + 1013904223)
    return h


def np_u11(seed, i):
    q = tdiv(np_hash(seed, i), 128)
    r = trem(trem(q, 1 << 24) + (1 << 24), 1 << 24)
    return (r.astype(np.float32) / np.float32(8388608.0)) - np.float32(1.0)


def np_u01(seed, i):
    q = tdiv(np_hash(seed, i), 128)
    r = trem(trem(q, 1 << 24) + (1 << 24), 1 << 24)
    return r.astype(np.float32) / np.float32(16777216.0)


@pytest.mark.parametrize("seed", [0, 1, 2, 3, 4, -7])
def test_stream_matches_numpy(seed):
    i = np.arange(0, 1 << 16)
    assert np.array_equal(o.gen(i.size, seed, 0, o.U11), np_u11(seed, i))
    assert np.array_equal(o.gen(i.size, seed, 0, o.U01), np_u01(seed, i))
    # offsets continue the same stream
    assert np.array_equal(o.gen(1000, seed, 12345, o.U11), np_u11(seed, np.arange(12345, 13345)))
    # stream positions past 2^31 wrap as i32 indices
    big = np.arange((1 << 31) - 3, (1 << 31) + 3)
    assert np.array_equal(o.gen(6, seed, int(big[0]), o.U11), np_u11(seed, wrap(big)))


def test_stream_statistics():
    u = o.gen(1 << 20, 1, 0, o.U11).astype(np.float64)
    assert u.min() >= -1.0 and u.max() < 1.0
    assert abs(u.mean()) < 3e-3 and abs(u.var() - 1 / 3) < 3e-3
    lag1 = np.corrcoef(u[:-1], u[1:])[0, 1]
    assert abs(lag1) < 3e-3
    idx = o.gen_index(1 << 20, 1, 0, 1 << 20)
    assert idx.min() >= 0 and idx.max() < (1 << 20)
    big = o.gen_index(1 << 16, 3, 0, 1 << 28)
    assert big.min() >= 0 and big.max() < (1 << 28) and big.max() > (1 << 27)


def np_matmul_strict(A, B):
    M, K = A.shape
    N = B.shape[1]
    C = np.zeros((M, N), np.float32)
    for k in range(K):  # acc = acc + a*b, k ascending, every op rounded in f32
        C = (C + (A[:, k:k + 1] * B[k:k + 1, :]).astype(np.float32)).astype(np.float32)
    return C


@pytest.mark.parametrize("shape", [(5, 20, 7), (6, 32, 5), (33, 65, 70), (64, 64, 64)])
def test_matmul_random_matches_numpy(shape):
    M, N, K = shape
    A = o.gen(M * K, 0, 0, o.U11)
    B = o.gen(K * N, 0, M * K, o.U11)
    C = o.matmul(A, B, M, N, K)
    assert np.array_equal(C.reshape(M, N), np_matmul_strict(A.reshape(M, K), B.reshape(K, N)))


def test_fir_conv_random_match_numpy():
    n, taps = 1000, 64
    x = o.gen(n + taps - 1, 1, 0, o.U11)
    w = o.gen(taps, 1, n + taps - 1, o.U11)
    acc = np.zeros(n, np.float32)
    for k in range(taps):
        acc = (acc + (w[k] * x[k:k + n]).astype(np.float32)).astype(np.float32)
    assert np.array_equal(o.fir(w, x, n), acc)
    R = C = 30
    img = o.gen((R + 2) * (C + 2), 1, 0, o.U11).reshape(R + 2, C + 2)
    w9 = o.gen(9, 1, 5000, o.U11)
    acc = np.zeros((R, C), np.float32)
    for k in range(9):
        acc = (acc + (w9[k] * img[k // 3:k // 3 + R, k % 3:k % 3 + C]).astype(np.float32)).astype(np.float32)
    assert np.array_equal(o.conv2d_3x3(w9, img.ravel().copy(), C + 2, R, C), acc.ravel())


def test_saxpy_sum_random_match_numpy():
    x = o.gen(4096, 1, 0, o.U11)
    y = o.gen(4096, 1, 4096, o.U11)
    assert np.array_equal(o.saxpy(2.5, x, y), (np.float32(2.5) * x).astype(np.float32) + y)
    acc = np.float32(0.0)
    for v in x[:2000]:
        acc = np.float32(acc + v)
    assert o.fold_sum(0.0, x[:2000]) == acc


def test_traps():
    x = np.arange(8, dtype=np.float32)
    rc, _ = o.gather(x, np.array([0, 8], np.int32))
    assert rc == 2
    rc, _ = o.gather(x, np.array([-1], np.int32))
    assert rc == 2
    s = o.matmul_site(2, 2, 2)
    s.a.len = 3  # A shorter than the site reads
    rc, _ = o.tile_site(s, np.zeros(4, np.float32), np.zeros(4, np.float32))
    assert rc == 2
