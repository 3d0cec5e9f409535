"""The C ABI without a GPU: the library loads, exports every function that
include/*.h declares, its records match the oracle's layouts, and the
re-exported mapal-rt symbols behave as the reference's (stdout bytes, trap
message, exit 101)."""
import ctypes
import os
import re
import subprocess
import sys

import numpy as np
import pytest

import flow_b200 as fb
import oracle as o
from flow_b200 import _native

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADERS = [os.path.join(ROOT, "include", h) for h in ("mapal_gpu.h", "mapal_rt.h")]


def declared_functions():
    names = []
    for h in HEADERS:
        text = open(h).read()
        text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
        names += re.findall(r"\b(mapal_\w+)\s*\(", text)
    return sorted(set(names))


def test_exports_every_declared_symbol():
    lib = fb.lib()
    declared = declared_functions()
    assert len(declared) >= 40
    missing = [n for n in declared if not hasattr(lib, n)]
    assert not missing, missing
    # and the Python binding covers exactly the declared set
    assert sorted(_native.SIGNATURES) == declared


def test_abi_version():
    assert fb.lib().mapal_gpu_abi_version() == 1


def test_record_layouts_match_oracle():
    for prod, ref in [(fb.TileSite, o.TileSite), (fb.TileRead, o.TileRead), (fb.MoveSite, o.MoveSite),
                      (fb.KSplit, o.KSplit)]:
        assert ctypes.sizeof(prod) == ctypes.sizeof(ref)
        for (n1, _), (n2, _) in zip(prod._fields_, ref._fields_):
            assert n1 == n2 and getattr(prod, n1).offset == getattr(ref, n2).offset
    assert ctypes.sizeof(fb.TileSite) == 3 * 8 + 2 * 64 + 8


def test_builders_match_oracle_builders():
    for a, b in [(fb.matmul_site(7, 9, 11), o.matmul_site(7, 9, 11)), (fb.fir_site(100, 64), o.fir_site(100, 64)),
                 (fb.conv2d_site(16, 16, 18, 324), o.conv2d_site(16, 16, 18, 324))]:
        assert bytes(a) == bytes(b)


@pytest.mark.parametrize("n,nr", [(0, 1), (10, 3), (1 << 30, 8), (7, 8), (1000003, 4)])
def test_shard_range(n, nr):
    spans = [fb.shard_range(n, nr, r) for r in range(nr)]
    assert spans[0][0] == 0 and spans[-1][1] == n
    for (lo, hi), (lo2, _) in zip(spans, spans[1:]):
        assert hi == lo2
    sizes = [hi - lo for lo, hi in spans]
    assert max(sizes) - min(sizes) <= 1


def test_shard_range_rejects_bad_rank():
    with pytest.raises(fb.MapalInfraError):
        fb.shard_range(10, 2, 2)


def test_no_device_is_an_infra_error():
    if fb.device_count() > 0:
        pytest.skip("a GPU is visible")
    with pytest.raises(fb.MapalInfraError) as e:
        fb.Context(devices=(0,), torch_stream=False)
    assert e.value.exit_code == 102


def test_render_matches_oracle_on_random_floats():
    rng = np.random.default_rng(5)
    bits = rng.integers(0, 1 << 32, 20000, dtype=np.uint64).astype(np.uint32)
    vals = bits.view(np.float32)
    special = np.array([0.0, -0.0, 1.0, 0.1, 1e20, 1e-7, 3.4028235e38, 1.17549435e-38, 1e-45,
                        4080.0, 5.375, 16777217.0, float("inf"), float("-inf"), float("nan")], np.float32)
    for v in list(vals) + list(special):
        assert fb.render_f32(float(v)) == o.render_f32(float(v)), v
    for v in list(rng.standard_normal(2000) * 10.0 ** rng.integers(-30, 30, 2000)) + [0.1 + 0.2, 1e300, 5e-324]:
        assert fb.render_f64(float(v)) == o.render_f64(float(v)), v


def test_render_matches_numpy_shortest_positional():
    rng = np.random.default_rng(9)
    vals = rng.integers(0, 1 << 32, 5000, dtype=np.uint64).astype(np.uint32).view(np.float32)
    for v in vals:
        if not np.isfinite(v):
            continue
        ref = np.format_float_positional(v, unique=True, trim="-")
        assert fb.render_f32(float(v)) == ref, v


PRINT_PROG = r"""
import ctypes, sys
sys.path.insert(0, %r)
import flow_b200 as fb
L = fb.lib()
L.mapal_print_f64(0.1 + 0.2, True)
L.mapal_print_f32(ctypes.c_float(1.0).value / 3.0, True)
L.mapal_print_f64(float("inf"), True)
L.mapal_print_f64(float("-inf"), True)
L.mapal_print_f64(float("nan"), True)
L.mapal_print_f64(1.5, True)
L.mapal_print_f64(-1.5, True)
L.mapal_print_i32(-275, True)
L.mapal_print_i64(-(1 << 40), False)
L.mapal_print_str(b" ok", 3, True)
L.mapal_print_bool(True, True)
L.mapal_print_u8(255, True)
L.mapal_print_f32(4080.0, True)
L.mapal_print_f32(-0.0, True)
"""


def test_prints_match_reference_pin():
    import json
    gold = json.load(open(os.path.join(ROOT, "tests", "golden", "reference_outputs.json")))
    out = subprocess.run([sys.executable, "-c", PRINT_PROG % ROOT], capture_output=True, text=True,
                         check=True).stdout
    lines = out.splitlines()
    # f32 1/3 is computed in f64 by Python then rounded: 0.33333334 either way
    assert lines[:7] == gold["float_print_pin"]["lines"]
    assert lines[7:] == ["-275", "-1099511627776 ok", "true", "255", "4080", "-0"]


@pytest.mark.parametrize("kind,msg", [(0, "div_zero"), (1, "index_oob"), (7, "unknown")])
def test_trap_exits_101(kind, msg):
    prog = f"import sys; sys.path.insert(0, {ROOT!r}); import flow_b200 as fb; " \
           f"fb.lib().mapal_print_i32(1, True); fb.lib().mapal_trap({kind})"
    r = subprocess.run([sys.executable, "-c", prog], capture_output=True, text=True)
    assert r.returncode == 101
    assert r.stdout == "1\n"
    assert r.stderr.strip().endswith(f"mapal trap: {msg}")


def test_time_ms_monotonic():
    L = fb.lib()
    a = L.mapal_time_ms()
    b = L.mapal_time_ms()
    assert 0.0 <= a <= b
