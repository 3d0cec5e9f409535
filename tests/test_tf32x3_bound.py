"""The 3xTF32 tolerance has teeth: on the inputs of the GPU tests
(tests/test_gpu_tf32x3.py), a split product that dropped one of its cross
terms (2xTF32) or both (1xTF32) errs beyond the stated bound even when every
product is exact and the accumulation is f64 — so a kernel that silently lost
a product cannot pass those tests. Pure numpy, no GPU."""
import numpy as np
import pytest

import oracle as o

TOL = 2e-6  # the bound of tests/test_gpu_tf32x3.py and include/mapal_gpu.h
SHAPES = [(128, 256, 16), (256, 256, 256), (200, 300, 100), (129, 257, 33), (64, 64, 30), (1, 1, 1),
          (1024, 1024, 1024), (300, 700, 4096), (130, 270, 4), (64, 64, 8), (257, 129, 12), (100, 33, 20)]


def rna_tf32(x: np.ndarray) -> np.ndarray:
    """f32 -> TF32 (10 explicit mantissa bits), round to nearest, ties away
    from zero (cvt.rna.tf32.f32), on finite inputs."""
    u = np.asarray(x, np.float32).view(np.uint32).astype(np.uint64)
    return (((u + 0x1000) & 0xFFFFE000).astype(np.uint32)).view(np.float32)


def split(x: np.ndarray):
    hi = rna_tf32(x)
    lo = rna_tf32((np.asarray(x, np.float32) - hi).astype(np.float32))
    return hi.astype(np.float64), lo.astype(np.float64)


def norm_err(C, ref, A2, B2) -> float:
    scale = np.sqrt((A2 * A2).sum(1))[:, None] * np.sqrt((B2 * B2).sum(0))[None, :]
    return float(np.max(np.abs(C - ref) / scale))


def test_rna_tf32_rounding():
    x = np.array([1.0, 1 + 2.0 ** -11, 1 + 2.0 ** -12, -(1 + 2.0 ** -11), 1 + 3 * 2.0 ** -11], np.float32)
    assert rna_tf32(x).tolist() == [1.0, 1 + 2.0 ** -10, 1.0, -(1 + 2.0 ** -10), 1 + 2.0 ** -9]


@pytest.mark.parametrize("M,N,K", SHAPES)
def test_tf32x3_tolerance_rejects_fewer_products(M, N, K):
    A = o.gen(M * K, 0, 0).reshape(M, K)
    B = o.gen(K * N, 0, M * K).reshape(K, N)
    A2, B2 = A.astype(np.float64), B.astype(np.float64)
    ref = A2 @ B2
    ahi, alo = split(A)
    bhi, blo = split(B)
    three = norm_err(ahi @ bhi + ahi @ blo + alo @ bhi, ref, A2, B2)
    two_a = norm_err(ahi @ bhi + ahi @ blo, ref, A2, B2)
    two_b = norm_err(ahi @ bhi + alo @ bhi, ref, A2, B2)
    one = norm_err(ahi @ bhi, ref, A2, B2)
    # the split itself is far inside the bound; every reduced form is outside it
    assert three < TOL / 10
    assert min(two_a, two_b, one) > 5 * TOL, (two_a, two_b, one)
