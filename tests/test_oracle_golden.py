"""Pin the CPU oracle to the reference's own outputs (tests/golden/reference_outputs.json,
made by tests/golden/make_golden.py from the reference's known answers and its
C++ baseline programs)."""
import json
import os

import numpy as np
import pytest

import oracle as o

GOLD = json.load(open(os.path.join(os.path.dirname(__file__), "golden", "reference_outputs.json")))


def int_a(n):  # (t*7 + 13) % 101 - 50, the benches' A / x generator
    return o.affine(n, 7, 13, 101, 50)


def int_b(n):  # (t*7 + 57) % 101 - 50, the matmul B generator
    return o.affine(n, 7, 57, 101, 50)


def int_w(n):  # (t*5 + 3) % 31 - 15, the benches' y0 / w generator
    return o.affine(n, 5, 3, 31, 15)


@pytest.mark.parametrize("case", GOLD["matmul_known_answers"], ids=lambda c: f"n{c['n']}")
def test_matmul_known_answers(case):
    n = case["n"]
    A, B = int_a(n * n), int_b(n * n)
    assert o.matmul_cell(A, B, n, n, 0, 0) == case["c0"]
    assert o.matmul_cell(A, B, n, n, n - 1, n - 1) == case["clast"]


@pytest.mark.parametrize("case", GOLD["cpp_mt"], ids=lambda c: f"n{c['n']}")
def test_matmul_matches_cpp_mt(case):
    n = case["n"]
    C = o.matmul(int_a(n * n), int_b(n * n), n, n, n)
    assert C[0] == case["c0"] and C[-1] == case["clast"]
    # the general TileSite evaluator agrees with the specialised matmul
    rc, C2 = o.tile_site(o.matmul_site(n, n, n), int_a(n * n), int_b(n * n))
    assert rc == 0 and np.array_equal(C, C2)


def _ladder(shape, size):
    for c in GOLD["ladder2"]:
        if c["shape"] == shape and c["size"] == size:
            return c["values"]
    raise KeyError((shape, size))


@pytest.mark.parametrize("n", [256, 1048576])
def test_saxpy_matches_ladder2(n):
    y = o.saxpy(2.5, int_a(n), int_w(n))
    assert ["%g" % y[0], "%g" % y[-1]] == _ladder("saxpy", n)


@pytest.mark.parametrize("n", [256, 1048576])
def test_reduce_matches_ladder2(n):
    assert ["%g" % o.fold_sum(0.0, int_a(n))] == _ladder("reduce", n)


@pytest.mark.parametrize("side", [16, 1024])
def test_transpose_matches_ladder2(side):
    rc, b = o.move_site(o.transpose_site(side, side), int_a(side * side))
    assert rc == 0
    assert ["%g" % b[0], "%g" % b[-1]] == _ladder("transpose", side)


@pytest.mark.parametrize("n", [256, 1048576])
def test_gather_matches_ladder2(n):
    idx = ((np.arange(n, dtype=np.int64) * 1021 + 12347) % n).astype(np.int32)
    rc, y = o.gather(int_a(n), idx)
    assert rc == 0
    assert ["%g" % y[0], "%g" % y[-1]] == _ladder("gather", n)


@pytest.mark.parametrize("case", GOLD["shapes"], ids=lambda c: f"{c['shape']}{c['size']}")
def test_fir_conv_match_shapes_baseline(case):
    n = case["size"]
    if case["shape"] == "fir":
        x, w = int_a(n + 63), int_w(64)
        y = o.fir(w, x, n)
        rc, y2 = o.tile_site(o.fir_site(n, 64), w, x)
        assert rc == 0 and np.array_equal(y, y2)
    else:
        stride = n + 2
        img, w = int_a(stride * stride), int_w(9)
        y = o.conv2d_3x3(w, img, stride, n, n)
        rc, y2 = o.tile_site(o.conv2d_site(n, n, stride, stride * stride), w, img)
        assert rc == 0 and np.array_equal(y, y2)
    assert ["%.9g" % y[0], "%.9g" % y[-1]] == case["values"]


def test_fir4_acceptance():
    g = GOLD["fir4"]
    sig = np.array(g["signal"], np.float32)
    coeffs = np.array(g["coeffs"], np.float32)
    s = o.fir_site(1, 4)
    s.b.base = g["window_start"]
    s.b.len = sig.size
    rc, out = o.tile_site(s, coeffs, sig)
    assert rc == 0 and o.render_f32(out[0]) == g["output"]


def test_float_print_pin():
    g = GOLD["float_print_pin"]
    f32 = np.float32
    vals = [o.render_f64(0.1 + 0.2), o.render_f32(f32(1.0) / f32(3.0)), o.render_f64(float("inf")),
            o.render_f64(float("-inf")), o.render_f64(float("nan")), o.render_f64(np.fmod(7.5, 2.0)),
            o.render_f64(np.fmod(-7.5, 2.0))]
    assert vals == g["lines"]


def test_matmul4_loop_example():
    a = np.array([-37, -30, -23, -16, -9, -2, 5, 12, 19, 26, 33, 40, 47, -47, -40, -33], np.float32)
    b = np.array([7, 14, 21, 28, 35, 42, 49, -45, -38, -31, -24, -17, -10, -3, 4, 11], np.float32)
    C = o.matmul(a, b, 4, 4, 4)
    assert (C[0], C[15]) == (-275.0, 3748.0)
