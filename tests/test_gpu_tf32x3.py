"""The opt-in 3xTF32 tensor-core matmul (tcgen05) against the oracle.

Tolerance (stated in the ABI header): for every cell
    |C - C_oracle| <= 1e-5 * ||A[i, :]|| * ||B[:, j]||
The split drops only Alo*Blo (about 2^-22 relative per product), so the
observed error is orders of magnitude below the bound; integer-valued inputs
(the reference's own generators) are exact."""
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
TOL = 1e-5


@pytest.fixture(scope="module")
def ctx():
    c = fb.Context((0,))
    yield c
    c.close()


def rel_err(C, want, A, B, M, N, K, rows=None):
    A2 = A.reshape(M, K).astype(np.float64)
    B2 = B.reshape(K, N).astype(np.float64)
    rn = np.sqrt((A2 * A2).sum(1))
    cn = np.sqrt((B2 * B2).sum(0))
    if rows is not None:
        rn = rn[rows]
    scale = np.maximum(rn[:, None] * cn[None, :], 1e-30)
    return float(np.max(np.abs(C.astype(np.float64) - want.astype(np.float64)) / scale))


@pytest.mark.parametrize("M,N,K", [(128, 256, 16), (256, 256, 256), (200, 300, 100), (129, 257, 33),
                                   (64, 64, 30), (1, 1, 1), (1024, 1024, 1024), (300, 700, 4096)])
def test_tf32x3_random(ctx, M, N, K):
    A = o.gen(M * K, 0, 0)
    B = o.gen(K * N, 0, M * K)
    C = empty_f32(M * N)
    ctx.matmul(fb.matmul_site(M, N, K), dev(A), dev(B), C, mode=fb.TF32X3)
    got = host(C).reshape(M, N)
    want = o.matmul(A, B, M, N, K, threads=8).reshape(M, N)
    assert np.all(np.isfinite(got))
    assert rel_err(got, want, A, B, M, N, K) <= TOL


def test_tf32x3_4096_sampled_rows(ctx):
    n = 4096
    A = o.gen(n * n, 2, 0)
    B = o.gen(n * n, 2, n * n)
    C = empty_f32(n * n)
    ctx.matmul(fb.matmul_site(n, n, n), dev(A), dev(B), C, mode=fb.TF32X3)
    c = host(C).reshape(n, n)
    for r0 in (0, 2049, 4088):
        want = o.matmul(A, B, n, n, n, row0=r0, row1=r0 + 8, threads=8).reshape(n, n)[r0:r0 + 8]
        assert rel_err(c[r0:r0 + 8], want, A, B, n, n, n, rows=slice(r0, r0 + 8)) <= TOL


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
    assert rel_err(host(C).reshape(M, N) - 3.0, want.reshape(M, N) - 3.0, Ad, Bd, M, N, K) <= TOL


def test_tf32x3_repeatable(ctx):
    M = N = K = 512
    A, B = dev(o.gen(M * K, 1, 0)), dev(o.gen(K * N, 1, M * K))
    C1, C2 = empty_f32(M * N), empty_f32(M * N)
    ctx.matmul(fb.matmul_site(M, N, K), A, B, C1, mode=fb.TF32X3)
    ctx.matmul(fb.matmul_site(M, N, K), A, B, C2, mode=fb.TF32X3)
    assert torch.equal(C1, C2)
