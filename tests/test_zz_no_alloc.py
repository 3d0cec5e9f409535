"""The sum fold that allocates nothing (mapal_gpu_fold_sum_f32_noalloc),
called through the C ABI and checked against the context-based entry point
(mapal_gpu_fold_sum_f32) on two calls in a row.

It exists for callers that cannot allocate device memory: a host runtime that
serves all device memory from one arena it sized up front, a process at its
HBM limit, or a latency-bound loop that cannot take cudaMalloc's implicit
synchronisation. Its scratch is a fixed array in the library's device data,
shared by every call, so the second call also checks that nothing of the
first call's scratch leaks into it.

Named test_zz_* so that pytest collects it after every other test file."""
import ctypes

import numpy as np
import pytest
import torch

import flow_b200 as fb
import oracle as o

pytestmark = pytest.mark.gpu

TOL = 1e-6  # the sum-fold tolerance of the parity tests: 1e-6 * sum|x|


def noalloc_sum(x: torch.Tensor, seed: float) -> float:
    out = torch.full((1,), float("nan"), dtype=torch.float32, device="cuda")
    stream = torch.cuda.current_stream().cuda_stream
    rc = fb.lib().mapal_gpu_fold_sum_f32_noalloc(seed, ctypes.c_void_p(x.data_ptr()), x.numel(),
                                                 ctypes.c_void_p(out.data_ptr()), ctypes.c_void_p(stream))
    assert rc == 0, fb.lib().mapal_gpu_last_error()
    torch.cuda.synchronize()
    return float(out.item())


def ctx_sum(ctx: fb.Context, x: torch.Tensor, seed: float) -> float:
    out = torch.full((1,), float("nan"), dtype=torch.float32, device="cuda")
    ctx.fold_sum(x, out, seed=seed)
    torch.cuda.synchronize()
    return float(out.item())


def test_noalloc_sum_matches_context_entry_point_twice():
    torch.cuda.init()
    cases = [((1 << 20) + 7, 1, 0.0), (3000, 2, 2.5)]  # two calls in a row, different sizes
    with fb.Context((0,)) as ctx:
        for n, seed, fold_seed in cases:
            xh = o.gen(n, seed, 0, o.U01)
            x = torch.from_numpy(xh).cuda()
            got = noalloc_sum(x, fold_seed)
            want = ctx_sum(ctx, x, fold_seed)
            scale = o.sum_abs_f64(xh) + abs(fold_seed)
            assert abs(got - want) <= TOL * scale, (n, got, want)
            assert abs(got - o.sum_f64(fold_seed, xh)) <= TOL * scale


def test_noalloc_rejects_null_output():
    x = torch.zeros(4, dtype=torch.float32, device="cuda")
    rc = fb.lib().mapal_gpu_fold_sum_f32_noalloc(0.0, ctypes.c_void_p(x.data_ptr()), 4, None, None)
    assert rc == fb.ERR_INVALID
