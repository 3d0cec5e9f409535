"""The checks bench.py puts in its JSON line, pinned on the CPU: the float32
restatement of the interpreter's matmul fold that certifies `strict_row_check`
(and the 16384 line's `row_check`) agrees with the oracle bit for bit and
rejects a one-ulp difference; the 3xTF32 error column is the normalised
error the tests use."""
import os
import sys

import numpy as np
import torch

import oracle as o

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
import bench  # noqa: E402


def _case(M, N, K, seed):
    A = o.gen(M * K, seed, 0)
    B = o.gen(K * N, seed, M * K)
    C = o.matmul(A, B, M, N, K, threads=4)
    return torch.from_numpy(A), torch.from_numpy(B), torch.from_numpy(C.copy())


def test_strict_rows_check_agrees_with_the_oracle():
    M, N, K = 37, 53, 300
    A, B, C = _case(M, N, K, 3)
    assert bench.strict_rows_check(torch, A, B, C, M, N, K, [0, 18, 36])
    assert bench.strict_rows_check(torch, A, B, C, M, N, K, [5], cols=[0, 7, 52])


def test_strict_rows_check_rejects_one_ulp():
    M, N, K = 16, 24, 64
    A, B, C = _case(M, N, K, 4)
    bad = C.clone().view(torch.int32)
    bad[5 * N + 7] += 1  # the next float up in one checked cell
    assert not bench.strict_rows_check(torch, A, B, bad.view(torch.float32), M, N, K, [5])
    # a row that was not checked may differ
    assert bench.strict_rows_check(torch, A, B, bad.view(torch.float32), M, N, K, [4, 6])


def test_tf32x3_rows_error_is_the_normalised_error():
    M, N, K = 8, 12, 40
    A, B, _ = _case(M, N, K, 5)
    exact = A.double().view(M, K) @ B.double().view(K, N)
    C = exact.float().clone()
    C[2, 3] += 1e-3
    a2 = A.double().view(M, K)
    b2 = B.double().view(K, N)
    scale = float(a2[2].norm() * b2[:, 3].norm())
    err = bench.tf32x3_rows_error(torch, A, B, C.view(-1), M, N, K, [2])
    assert abs(err - abs(float(C[2, 3].double() - exact[2, 3])) / scale) < 1e-9
