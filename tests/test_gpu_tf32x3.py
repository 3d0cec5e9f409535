"""The opt-in 3xTF32 tensor-core matmul (tcgen05) against the oracle.

Tolerance (stated in the ABI header): for every cell, with K <= 4096,
    |C - A.B| <= TOL * ||A[i, :]|| * ||B[:, j]||,   TOL = 2e-6,
A.B being the exact (f64) product. Why this bound: the split x = hi + lo
(hi, lo TF32) makes each product exact to about 2^-21 relative; what remains
is the tensor pipe's f32 accumulation, whose error grows with the number of
additions into one accumulator (two alternating accumulators halve it).
Measured on a B200: at most 7e-7 at K = 4096 and 3e-7 at K <= 1024, against
1.3e-7 - 2.6e-7 for the strict f32 fold. A 3xTF32 that lost one cross
product (2xTF32) errs by 1.4e-5 or more on these inputs and 1xTF32 by
1.8e-5 or more: both fail the bound (test_tf32x3_tolerance_rejects_fewer_products,
a numpy emulation on the same inputs). Integer-valued inputs (the
reference's own generators) are exact."""
import json
import os

import numpy as np
import pytest
import torch

import flow_b200 as fb
import oracle as o
from _gpu import dev, empty_f32, host

pytestmark = pytest.mark.gpu

GOLD = json.load(open(os.path.join(os.path.dirname(__file__), "golden", "reference_outputs.json")))
TOL = 2e-6
SHAPES = [(128, 256, 16), (256, 256, 256), (200, 300, 100), (129, 257, 33), (64, 64, 30), (1, 1, 1),
          (1024, 1024, 1024), (300, 700, 4096),
          # K a multiple of 4 (A read in place by the fused kernel) below one 16-deep k-block
          (130, 270, 4), (64, 64, 8), (257, 129, 12), (100, 33, 20)]


@pytest.fixture(scope="module")
def ctx():
    c = fb.Context((0,))
    yield c
    c.close()


def rel_err(C, want, A, B, M, N, K, rows=None):
    """max |C - want| / (||A_i|| ||B_j||) over the cells of C."""
    A2 = A.reshape(M, K).astype(np.float64)
    B2 = B.reshape(K, N).astype(np.float64)
    rn = np.sqrt((A2 * A2).sum(1))
    cn = np.sqrt((B2 * B2).sum(0))
    if rows is not None:
        rn = rn[rows]
    scale = np.maximum(rn[:, None] * cn[None, :], 1e-30)
    return float(np.max(np.abs(C.astype(np.float64) - want.astype(np.float64)) / scale))


def exact(A, B, M, N, K):
    return A.reshape(M, K).astype(np.float64) @ B.reshape(K, N).astype(np.float64)


@pytest.mark.parametrize("M,N,K", SHAPES)
def test_tf32x3_random(ctx, M, N, K):
    A = o.gen(M * K, 0, 0)
    B = o.gen(K * N, 0, M * K)
    C = empty_f32(M * N)
    ctx.matmul(fb.matmul_site(M, N, K), dev(A), dev(B), C, mode=fb.TF32X3)
    got = host(C).reshape(M, N)
    assert np.all(np.isfinite(got))
    ref = exact(A, B, M, N, K)
    err = rel_err(got, ref, A, B, M, N, K)
    # the strict fold's own error on the same inputs, for scale
    strict = o.matmul(A, B, M, N, K, threads=8).reshape(M, N)
    err_strict = rel_err(strict, ref, A, B, M, N, K)
    print(f"3xTF32 {M}x{N}x{K}: max normalised error {err:.3g} (strict f32 fold {err_strict:.3g})")
    assert err <= TOL
    # within a small multiple of the strict fold's error (floor: one split
    # product alone may err by 2^-21 relative)
    assert err <= 4.0 * max(err_strict, 2.5e-7)


def test_tf32x3_4096_sampled_rows(ctx):
    n = 4096
    A = o.gen(n * n, 2, 0)
    B = o.gen(n * n, 2, n * n)
    C = empty_f32(n * n)
    ctx.matmul(fb.matmul_site(n, n, n), dev(A), dev(B), C, mode=fb.TF32X3)
    c = host(C).reshape(n, n)
    B2 = B.reshape(n, n).astype(np.float64)
    for r0 in (0, 2049, 4088):
        want = A.reshape(n, n)[r0:r0 + 8].astype(np.float64) @ B2
        err = rel_err(c[r0:r0 + 8], want, A, B, n, n, n, rows=slice(r0, r0 + 8))
        print(f"3xTF32 4096^3 rows {r0}..{r0 + 7}: max normalised error {err:.3g}")
        assert err <= TOL


@pytest.mark.parametrize("case", [c for c in GOLD["matmul_known_answers"] if c["n"] in (16, 256, 1024)],
                         ids=lambda c: f"n{c['n']}")
def test_tf32x3_integer_inputs_exact(ctx, case):
    n = case["n"]
    A = o.affine(n * n, 7, 13, 101, 50)
    B = o.affine(n * n, 7, 57, 101, 50)
    C = empty_f32(n * n)
    ctx.matmul(fb.matmul_site(n, n, n), dev(A), dev(B), C, mode=fb.TF32X3)
    c = host(C)
    assert (c[0], c[-1]) == (case["c0"], case["clast"])
    assert np.array_equal(c, o.matmul(A, B, n, n, n, threads=8))


def test_tf32x3_seed_and_padded_strides(ctx):
    M, N, K, lda, ldb = 100, 130, 70, 73, 131
    A = o.gen(M * lda, 5, 0)
    B = o.gen(K * ldb, 5, 99999)
    s = fb.matmul_site(M, N, K, lda=lda, ldb=ldb)
    s.seed = 3.0
    C = empty_f32(M * N)
    ctx.matmul(s, dev(A), dev(B), C, mode=fb.TF32X3)
    rc, want = o.tile_site(o.TileSite.from_buffer_copy(bytes(s)), A, B)
    assert rc == 0
    Ad = A.reshape(M, lda)[:, :K].ravel().copy()
    Bd = B.reshape(K, ldb)[:, :N].ravel().copy()
    # the seed is added after the product: compare C - seed with A.B
    assert rel_err(host(C).reshape(M, N).astype(np.float64) - 3.0, exact(Ad, Bd, M, N, K),
                   Ad, Bd, M, N, K) <= TOL
    assert rc == 0 and want.size == M * N


def test_tf32x3_repeatable(ctx):
    M = N = K = 512
    A, B = dev(o.gen(M * K, 1, 0)), dev(o.gen(K * N, 1, M * K))
    C1, C2 = empty_f32(M * N), empty_f32(M * N)
    ctx.matmul(fb.matmul_site(M, N, K), A, B, C1, mode=fb.TF32X3)
    ctx.matmul(fb.matmul_site(M, N, K), A, B, C2, mode=fb.TF32X3)
    assert torch.equal(C1, C2)


@pytest.mark.parametrize("lda_pad", [0, 3])
def test_tf32x3_non_finite_inputs(ctx, lda_pad):
    # NaN propagates to every cell it touches, including a NaN whose payload
    # lies only in the low 13 mantissa bits (the tensor pipe would read it as
    # infinity after truncation); a cell touching an infinity is not finite.
    # lda_pad = 3 takes the pre-split path (rows TMA cannot address in place).
    M, N, K = 130, 260, 40
    lda = K + lda_pad
    A = o.gen(M * lda, 7, 0).reshape(M, lda)
    B = o.gen(K * N, 7, M * lda).reshape(K, N)
    A[3, 5] = np.float32(np.inf)
    A[70, 11] = np.uint32(0x7F800001).view(np.float32)  # NaN, payload in the low bits only
    B[9, 200] = np.float32(np.nan)
    s = fb.matmul_site(M, N, K, lda=lda)
    C = empty_f32(M * N)
    ctx.matmul(s, dev(A.ravel()), dev(B.ravel()), C, mode=fb.TF32X3)
    c = host(C).reshape(M, N)
    assert np.all(np.isnan(c[70, :]))
    assert np.all(np.isnan(c[:, 200]))
    assert not np.any(np.isfinite(c[3, :]))
    finite_rows = [r for r in range(M) if r not in (3, 70)]
    cols = [j for j in range(N) if j != 200]
    got = c[np.ix_(finite_rows, cols)]
    Ad = A[finite_rows, :K]
    Bd = B[:, cols]
    assert rel_err(got, Ad.astype(np.float64) @ Bd.astype(np.float64), Ad.ravel(), Bd.ravel(),
                   len(finite_rows), len(cols), K) <= TOL
