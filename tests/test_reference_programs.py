"""The reference's own bench programs (benches/shapes/*.mapal, the f32 matmul
cap and counted-loop sources of benches/matmul, and the examples inside the
bench subset), kept byte for byte under tests/golden/mapal/ by
tests/golden/make_golden.py. Without a GPU: every one is inside the driver's
subset and plans to the site class the reference's recognizer gives it
(crates/mapal-ir/src/algo.rs:815-1079), and the expected outputs stored beside
them agree with the reference's C++ baseline legs and with the evaluator."""
import json
import os
import subprocess

import pytest

from oracle.mapal_eval import expected

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
DRIVER = os.path.join(ROOT, "flow_b200", "mapal-run")
GOLD = json.load(open(os.path.join(HERE, "golden", "reference_outputs.json")))
CASES = GOLD["reference_programs"]
MAPAL_DIR = os.path.join(HERE, "golden", "mapal")

# The site each bench program's timed statement must plan to: the
# specialised kernel of its class, never the general map body.
TIMED_SITE = {
    "saxpy": "saxpy n=", "transpose": "move_site ", "gather": "gather n=",
    "reduce": "fold_sum_f32_strict n=", "fir": "tile_site rows=1 ", "conv2d": "tile_site ",
    "attn": "tile_site ", "matmul": "tile_site ",
}


def _plan(path: str, *flags: str) -> subprocess.CompletedProcess:
    return subprocess.run([DRIVER, "--plan", *flags, path], capture_output=True, text=True, timeout=60)


@pytest.fixture(scope="module", autouse=True)
def _driver_built():
    if not os.path.exists(DRIVER):
        pytest.fail(f"{DRIVER} is missing: python -m flow_b200.build")


def test_fixture_set_is_complete():
    files = sorted(f"{d}/{f}" for d in os.listdir(MAPAL_DIR) for f in os.listdir(os.path.join(MAPAL_DIR, d)))
    assert files == sorted(c["file"] for c in CASES)
    # every benches/shapes source and every f32 cap matmul is present
    assert sum(c["file"].startswith("shapes/") for c in CASES) == 22
    assert sum(c["file"].endswith("_cap_f32.mapal") for c in CASES) == 8


@pytest.mark.parametrize("case", CASES, ids=lambda c: c["file"])
def test_reference_program_plans(case):
    path = os.path.join(MAPAL_DIR, case["file"])
    r = _plan(path)
    assert r.returncode == 0, r.stderr
    name = os.path.basename(case["file"])
    cls = next((k for k in TIMED_SITE if name.startswith(k)), None)
    if cls is not None:
        # the recognizer alone (with fusion on, an untimed gather may take its
        # index map into one general body instead)
        r = _plan(path, "--no-fuse")
        assert any(ln.startswith(TIMED_SITE[cls]) for ln in r.stdout.split("\n")), r.stdout


def _probe_values(case) -> list[float]:
    lines = [ln for ln in case["expected"].split("\n") if ln and not ln.startswith("iter ms=")]
    return [float(v) for v in lines]


@pytest.mark.parametrize("table,shape,size,file", [
    ("ladder2", "saxpy", 256, "shapes/saxpy_256.mapal"),
    ("ladder2", "saxpy", 1048576, "shapes/saxpy_1048576.mapal"),
    ("ladder2", "reduce", 256, "shapes/reduce_256.mapal"),
    ("ladder2", "reduce", 1048576, "shapes/reduce_1048576.mapal"),
    ("ladder2", "transpose", 16, "shapes/transpose_16.mapal"),
    ("ladder2", "transpose", 1024, "shapes/transpose_1024.mapal"),
    ("ladder2", "gather", 1048576, "shapes/gather_1048576.mapal"),
    ("shapes", "fir", 65536, "shapes/fir_65536.mapal"),
    ("shapes", "fir", 1048576, "shapes/fir_1048576.mapal"),
    ("shapes", "conv2d", 16, "shapes/conv2d_16.mapal"),
    ("shapes", "conv2d", 512, "shapes/conv2d_512.mapal"),
    ("shapes", "conv2d", 1024, "shapes/conv2d_1024.mapal"),
])
def test_expected_agrees_with_reference_cpp_legs(table, shape, size, file):
    # the reference's C++ baseline programs print the same probe values (the
    # Mapal source may print more: transpose_16 adds b[1]). gather_256 and
    # fir_256 are not paired: their index map / tap count differ from the C++ legs'.
    case = next(c for c in CASES if c["file"] == file)
    ref = next(c for c in GOLD[table] if c["shape"] == shape and c["size"] == size)
    want = [float(v) for v in ref["values"]]
    assert _probe_values(case)[:len(want)] == want


@pytest.mark.parametrize("case", [c for c in CASES if c["file"].startswith("matmul/") or
                                  c["file"].startswith("examples/matmul")], ids=lambda c: c["file"])
def test_matmul_expected_is_the_published_answer(case):
    import re
    n = int(re.search(r"matmul(\d+)", case["file"]).group(1))
    known = {c["n"]: (c["c0"], c["clast"]) for c in GOLD["matmul_known_answers"]}
    if n not in known:  # N=32 is published for the loop form only
        known[32] = (-1219, 4392)
    assert tuple(_probe_values(case)) == known[n]


@pytest.mark.parametrize("case", [c for c in CASES if c["expected_from"] == "oracle evaluator"
                                  and "1048576" not in c["file"] and "1024" not in c["file"]
                                  and "2048" not in c["file"] and "1536" not in c["file"]],
                         ids=lambda c: c["file"])
def test_expected_is_the_evaluators(case):
    # small programs: the stored expectation is what the evaluator prints now
    src = open(os.path.join(MAPAL_DIR, case["file"])).read()
    assert expected(src) == (case["expected"], case["rc"])


def test_fixtures_are_the_reference_sources():
    ref = os.environ.get("MAPAL_REFERENCE", os.path.join(os.path.dirname(ROOT), "reference"))
    if not os.path.isdir(os.path.join(ref, "benches")):
        pytest.skip("reference tree not present")
    for c in CASES:
        with open(os.path.join(ref, c["source"]), "rb") as a, open(os.path.join(MAPAL_DIR, c["file"]), "rb") as b:
            assert a.read() == b.read(), c["file"]
