"""The program driver on the GPU: `mapal-run prog.mapal` against the oracle's
program evaluator — the same stdout byte for byte and the same exit code
(0, or 101 after a trap), the protocol of the reference's CUDA differential
tests (crates/backends/cuda/tests/differential.rs:242-276)."""
import glob
import os
import subprocess

import pytest

import mapal_programs as P
from oracle.mapal_eval import expected, matches

pytestmark = pytest.mark.gpu

HERE = os.path.dirname(os.path.abspath(__file__))
DRIVER = os.path.join(os.path.dirname(HERE), "flow_b200", "mapal-run")
PROGRAMS = sorted(glob.glob(os.path.join(HERE, "programs", "*.mapal")))


def _run(path: str, *flags: str) -> subprocess.CompletedProcess:
    return subprocess.run([DRIVER, *flags, path], capture_output=True, text=True, timeout=300)


def _check(path: str, src: str, *flags: str):
    want, want_rc = expected(src)
    r = _run(path, *flags)
    assert r.returncode == want_rc, (r.returncode, r.stdout, r.stderr)
    assert matches(r.stdout, want), (r.stdout, want)
    if want_rc == 101:
        assert r.stderr.startswith("mapal trap: ")


@pytest.mark.parametrize("path", PROGRAMS, ids=os.path.basename)
def test_program(path):
    _check(path, open(path).read())


@pytest.mark.parametrize("path", PROGRAMS, ids=os.path.basename)
def test_program_unfused(path):
    # every map site writes its array: the same stdout as the fused run
    _check(path, open(path).read(), "--no-fuse")


@pytest.mark.parametrize("name,src", [
    ("saxpy_2e20", P.saxpy(1 << 20)), ("reduce_2e20", P.reduce(1 << 20)),
    ("transpose_1024", P.transpose(1024)), ("gather_2e20", P.gather(1 << 20)),
    ("fir_2e20", P.fir(1 << 20)), ("conv2d_1024", P.conv2d(1024)), ("matmul_256", P.matmul(256)),
    ("float_print", P.FLOAT_PRINT)])
def test_bench_shape(name, src, tmp_path):
    f = tmp_path / f"{name}.mapal"
    f.write_text(src)
    _check(str(f), src)


def test_matmul_4096_known_answer(tmp_path):
    # the headline shape end to end: c[0] and c[N*N-1] of the integer-generator
    # product are the reference's published known answers
    f = tmp_path / "matmul_4096.mapal"
    f.write_text(P.matmul(4096))
    r = _run(str(f))
    assert r.returncode == 0, r.stderr
    assert r.stdout == "74348\n-302529\n"


@pytest.mark.parametrize("n,literals", [(4, True), (16, False), (64, False), (256, False)])
def test_loop_form_matmul_known_answers(n, literals, tmp_path):
    # the counted-loop form, lifted to the tile site, prints the reference's
    # published answers for the same inputs
    import json
    gold = json.load(open(os.path.join(HERE, "golden", "reference_outputs.json")))["matmul_known_answers"]
    case = [c for c in gold if c["n"] == n][0]
    f = tmp_path / f"matmul_loops_{n}.mapal"
    f.write_text(P.matmul_loops(n, literals))
    r = _run(str(f))
    assert r.returncode == 0, r.stderr
    assert r.stdout == f"{case['c0']}\n{case['clast']}\n"


@pytest.mark.parametrize("name,src", [("matmul_256", P.matmul(256)), ("matmul_frac_96", None),
                                      ("loops_64", P.matmul_loops(64))])
def test_matmul_partitioned_across_gpus(name, src, tmp_path):
    # --gpus 2: row blocks of A and C per device, B broadcast; the same bytes
    import torch
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    if src is None:
        src = open(os.path.join(HERE, "programs", "matmul_frac_96.mapal")).read()
    f = tmp_path / f"{name}.mapal"
    f.write_text(src)
    one = subprocess.run([DRIVER, str(f)], capture_output=True, text=True, timeout=300)
    two = subprocess.run([DRIVER, "--gpus", "2", str(f)], capture_output=True, text=True, timeout=300)
    assert one.returncode == 0 and two.returncode == 0, (one.stderr, two.stderr)
    assert two.stdout == one.stdout


def test_tf32x3_mode_on_integer_inputs(tmp_path):
    # the benches' integer generators give products and sums exact in the
    # 3xTF32 split, so the tensor-core mode prints the same known answers
    f = tmp_path / "matmul_256.mapal"
    f.write_text(P.matmul(256))
    r = subprocess.run([DRIVER, "--tf32x3", str(f)], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stderr
    assert r.stdout == "-3694\n10946\n"
