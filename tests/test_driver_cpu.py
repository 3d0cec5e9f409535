"""The program driver without a GPU: the oracle's program evaluator pinned to the
reference's known answers, and the driver's site plan for each program.

`mapal-run --plan` reads a program and prints the ABI calls it would make
(no device needed); programs outside the subset exit 2.
"""
import glob
import json
import os
import subprocess

import pytest

import mapal_programs as P
from oracle.mapal_eval import TIME_MARK, expected, matches

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
DRIVER = os.path.join(ROOT, "flow_b200", "mapal-run")
PROGRAMS = sorted(glob.glob(os.path.join(HERE, "programs", "*.mapal")))
GOLD = json.load(open(os.path.join(HERE, "golden", "reference_outputs.json")))


def _gold(table, shape, size):
    for c in GOLD[table]:
        if c["shape"] == shape and c["size"] == size:
            return c["values"]
    raise KeyError((shape, size))


# ---- the evaluator against the reference's known answers ---------------------------

@pytest.mark.parametrize("case", [c for c in GOLD["matmul_known_answers"] if c["n"] <= 256],
                         ids=lambda c: f"n{c['n']}")
def test_eval_matmul_known_answers(case):
    out, rc = expected(P.matmul(case["n"]))
    assert rc == 0 and out == f"{case['c0']}\n{case['clast']}\n"


@pytest.mark.parametrize("shape,size,prog", [
    ("saxpy", 256, P.saxpy), ("saxpy", 1048576, P.saxpy), ("reduce", 256, P.reduce),
    ("reduce", 1048576, P.reduce), ("transpose", 16, P.transpose), ("transpose", 1024, P.transpose),
    ("gather", 256, P.gather), ("gather", 1048576, P.gather)])
def test_eval_matches_ladder2(shape, size, prog):
    out, rc = expected(prog(size))
    assert rc == 0 and out.split("\n")[:-1] == _gold("ladder2", shape, size)


@pytest.mark.parametrize("shape,size", [("fir", 256), ("fir", 65536), ("conv2d", 16), ("conv2d", 20),
                                        ("conv2d", 92), ("conv2d", 512)])
def test_eval_matches_shapes_baseline(shape, size):
    out, rc = expected(P.fir(size) if shape == "fir" else P.conv2d(size))
    assert rc == 0 and out.split("\n")[:-1] == _gold("shapes", shape, size)


def test_eval_float_print_pin():
    out, rc = expected(P.FLOAT_PRINT)
    assert rc == 0 and out.split("\n")[:-1] == GOLD["float_print_pin"]["lines"]


def test_eval_traps_and_order():
    # the print before the trapping site appears, nothing after it
    src = 'fn main() {\n 10 -> iota -> d;\n "a" -> println;\n d -> map { i -> 5 / (i - 3) } -> q;\n' \
          ' "b" -> println;\n}\n'
    assert expected(src) == ("a\n", 101)
    src = "fn main() {\n 4 -> iota -> d;\n d -> map { i -> i + 1 } -> e;\n d -> map { i -> d[i] } -> ok;\n" \
          " e -> map { j -> ok[j] } -> bad;\n}\n"
    assert expected(src)[1] == 101


def test_time_mark_matching():
    assert matches("ms=1.25\n", "ms=" + TIME_MARK + "\n")
    assert matches("ms=3\n", "ms=" + TIME_MARK + "\n")
    assert not matches("ms=1.25\nx\n", "ms=" + TIME_MARK + "\n")


# ---- the driver's site plan ---------------------------------------------------------

def _plan(src: str, tmp_path, *flags: str) -> subprocess.CompletedProcess:
    f = tmp_path / "p.mapal"
    f.write_text(src)
    return subprocess.run([DRIVER, "--plan", *flags, str(f)], capture_output=True, text=True, timeout=60)


@pytest.fixture(scope="module", autouse=True)
def _driver_built():
    if not os.path.exists(DRIVER):
        pytest.fail(f"{DRIVER} is missing: python -m flow_b200.build")


@pytest.mark.parametrize("prog,site", [
    (P.matmul(64), "tile_site rows=64 c=64 k=64 a{base=0 ci=64 ck=1 clane=0 ks=0/0/0} "
                   "b{base=0 ci=0 ck=64 clane=1 ks=0/0/0}"),
    (P.fir(1000, 17), "tile_site rows=1 c=1000 k=17 a{base=0 ci=0 ck=1 clane=0 ks=0/0/0} "
                      "b{base=0 ci=0 ck=1 clane=1 ks=0/0/0}"),
    (P.conv2d(30), "tile_site rows=30 c=30 k=9 a{base=0 ci=0 ck=1 clane=0 ks=0/0/0} "
                   "b{base=0 ci=32 ck=0 clane=1 ks=3/32/1}"),
    (P.saxpy(1000), "saxpy n=1000"),
    (P.reduce(1000), "fold_sum_f32_strict n=1000"),
    (P.transpose(40), "move_site width=40 rows=40 cq=1 cr=40"),
    (P.gather(1000), "gather n=1000 n_x=1000"),
])
def test_plan_recognises_sites(prog, site, tmp_path):
    # the recogniser alone: with fusion on, a site whose input is a deferred
    # map becomes one general map body that recomputes the input instead
    r = _plan(prog, tmp_path, "--no-fuse")
    assert r.returncode == 0, r.stderr
    assert site in r.stdout.split("\n")


def test_plan_gather_recomputes_its_index_array(tmp_path):
    lines = _plan(P.gather(1000), tmp_path).stdout.split("\n")
    assert lines[1:3] == ["map_expr n=1000 ops=8 arrays=0 deferred", "map_expr n=1000 ops=9 arrays=1 fused=1"]


@pytest.mark.parametrize("path", PROGRAMS, ids=os.path.basename)
def test_plan_every_program(path):
    r = subprocess.run([DRIVER, "--plan", path], capture_output=True, text=True, timeout=60)
    assert r.returncode == 0, r.stderr
    # a program with bulk statements makes ABI calls
    calls = [ln for ln in r.stdout.split("\n") if ln and not ln.startswith(("print", "read element"))]
    assert bool(calls) == ("-> map" in open(path).read())


FUSE_SRC = ("fn main() {\n 100 -> iota -> d;\n d -> map { i -> i * i % 7 -> widen_f32 } -> f;\n"
            " f -> map { x -> x / 3.0 - x % 2.0 } -> g;\n g[5] -> println;\n}\n")


def test_plan_general_body_uses_map_expr(tmp_path):
    r = _plan(FUSE_SRC, tmp_path, "--no-fuse")
    assert r.returncode == 0, r.stderr
    assert r.stdout.split("\n")[:2] == ["map_expr n=100 ops=7 arrays=0",  # i, i, *, 7, %, widen, store
                                        "map_expr n=100 ops=8 arrays=1"]


def test_plan_fuses_producer_into_consumer(tmp_path):
    # f's body (trap-free: % by a nonzero literal) is recomputed at both of g's
    # uses of x; f is never written, g is written when its element is read
    r = _plan(FUSE_SRC, tmp_path)
    assert r.returncode == 0, r.stderr
    assert r.stdout.split("\n")[:4] == ["map_expr n=100 ops=7 arrays=0 deferred",
                                        "map_expr n=100 ops=18 arrays=0 fused=2 deferred",
                                        "map_expr n=100 ops=18 arrays=0", "read element 5"]


def test_plan_fusion_gates(tmp_path):
    lines = _plan(open(os.path.join(HERE, "programs", "fused_chain.mapal")).read(), tmp_path).stdout.split("\n")
    # a three-stage chain becomes one program
    assert "map_expr n=70001 ops=43 arrays=0 fused=3 deferred" in lines
    # a clock read writes the live deferred map first
    assert lines.index("map_expr n=70001 ops=6 arrays=0") < lines.index("map_expr n=70001 ops=4 arrays=1 deferred")
    # too deep / too long once fused: the consumer reads the producer's array
    assert "map_expr n=70001 ops=18 arrays=1 deferred" in lines
    assert "map_expr n=70001 ops=16 arrays=1 deferred" in lines
    # bodies that can trap are launched where they stand, never deferred
    trap = _plan("fn main() {\n 10 -> iota -> d;\n d -> map { i -> 100 / (i - 3) } -> q;\n"
                 " d -> map { i -> q[9 - i] } -> r;\n}\n", tmp_path).stdout.split("\n")
    assert trap[:2] == ["map_expr n=10 ops=6 arrays=0", "map_expr n=10 ops=5 arrays=1"]


def test_plan_dead_unconsumed_map_still_runs(tmp_path):
    r = _plan("fn main() {\n 64 -> iota -> d;\n d -> map { i -> i + 1 } -> unused;\n \"x\" -> println;\n}\n",
              tmp_path)
    assert r.stdout.split("\n")[:3] == ["map_expr n=64 ops=4 arrays=0 deferred", "map_expr n=64 ops=4 arrays=0",
                                        "println"]


def test_plan_lifts_counted_loops(tmp_path):
    # the loop form of the product becomes the matmul tile site (lift.rs R-LF / R-LM)
    for prog in (P.matmul_loops(16), P.matmul_loops(4, literals=True)):
        r = _plan(prog, tmp_path)
        assert r.returncode == 0, r.stderr
        n = 16 if "16 -> iota" in prog or "[f32; 256]" in prog else 4
        assert f"lift product: counted loop over {n * n} -> map" in r.stdout
        assert (f"tile_site rows={n} c={n} k={n} a{{base=0 ci={n} ck=1 clane=0 ks=0/0/0}} "
                f"b{{base=0 ci=0 ck={n} clane=1 ks=0/0/0}}") in r.stdout.split("\n")


@pytest.mark.parametrize("src,why", [
    ("fn helper() { 1 -> println; }\nfn main() { 1 -> println; }\n", "expected"),
    ("fn f(x: i32) -> i32 {\n mut k: i32 <- 0;\n mut s: i32 <- 0;\n loop {\n (k < 4) -> {\n -true-> {\n"
     " s + x -> s;\n k + 2 -> k;\n -> loop;\n }\n -false-> s -> ret;\n }\n }\n}\n"
     "fn main() {\n 4 -> iota -> d;\n d -> f -> e;\n}\n", "counted map loop"),
    ("fn main() {\n mut k: i32 <- 0;\n}\n", "expected"),
    ("fn main() {\n 10 -> iota -> d;\n d -> map { i -> i -> widen_f64 } -> e;\n}\n", "map body stage"),
    ("fn main() {\n 10 -> iota -> d;\n d -> map { i -> (1, d) -> fold { a, v -> a * v } } -> e;\n}\n",
     "fold"),
])
def test_plan_refuses_outside_subset(src, why, tmp_path):
    r = _plan(src, tmp_path)
    assert r.returncode == 2
    assert "unsupported" in r.stderr and why in r.stderr


def test_plan_partitions_matmul_across_gpus(tmp_path):
    f = tmp_path / "mm.mapal"
    f.write_text(P.matmul(64))
    r = subprocess.run([DRIVER, "--plan", "--gpus", "3", str(f)], capture_output=True, text=True, timeout=60)
    assert r.returncode == 0, r.stderr
    assert "matmul_f32_sharded gpus=3 rows=22,21,21" in r.stdout
    # every other site stays on the first device
    assert "gen_affine n=4096 mul=7 add=13 mod=101 sub=50" in r.stdout


def test_plan_tf32x3_mode(tmp_path):
    f = tmp_path / "mm.mapal"
    f.write_text(P.matmul(32))
    r = subprocess.run([DRIVER, "--plan", "--tf32x3", str(f)], capture_output=True, text=True, timeout=60)
    assert r.returncode == 0 and "matmul mode tf32x3" in r.stdout


def test_plan_nt_matmul_relayouts_then_matmul():
    path = os.path.join(HERE, "programs", "matmul_nt_48x40x36.mapal")
    r = subprocess.run([DRIVER, "--plan", path], capture_output=True, text=True, timeout=60)
    assert r.returncode == 0, r.stderr
    lines = r.stdout.split("\n")
    assert "move_site width=40 rows=36 cq=1 cr=36 (B^T -> K x N)" in lines
    assert ("tile_site rows=48 c=40 k=36 a{base=0 ci=36 ck=1 clane=0 ks=0/0/0} "
            "b{base=0 ci=0 ck=40 clane=1 ks=0/0/0}") in lines
