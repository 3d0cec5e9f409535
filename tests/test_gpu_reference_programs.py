"""The reference's own bench programs through the GPU driver, unmodified:
`mapal-run <file>` for every source under tests/golden/mapal/ (every
benches/shapes program, the f32 cap and counted-loop matmuls of
benches/matmul, and the examples inside the bench subset). Stdout must equal
the expected text line for line — the interpreter's output from the oracle
evaluator, or the published known answer of results.csv for the products the
evaluator cannot run here — with each `iter ms=` line carrying a positive
number, and the exit code must match (the protocol of
crates/backends/cuda/tests/differential.rs:242-276)."""
import json
import os
import re
import subprocess

import pytest

from oracle.mapal_eval import matches

pytestmark = pytest.mark.gpu

HERE = os.path.dirname(os.path.abspath(__file__))
DRIVER = os.path.join(os.path.dirname(HERE), "flow_b200", "mapal-run")
CASES = json.load(open(os.path.join(HERE, "golden", "reference_outputs.json")))["reference_programs"]
MAPAL_DIR = os.path.join(HERE, "golden", "mapal")


def _run(path: str, *flags: str) -> subprocess.CompletedProcess:
    return subprocess.run([DRIVER, *flags, path], capture_output=True, text=True, timeout=300)


@pytest.mark.parametrize("case", CASES, ids=lambda c: c["file"])
def test_reference_program_on_gpu(case):
    r = _run(os.path.join(MAPAL_DIR, case["file"]))
    assert r.returncode == case["rc"], (r.returncode, r.stdout, r.stderr)
    assert matches(r.stdout, case["expected"]), (r.stdout, case["expected"])
    for ms in re.findall(r"^iter ms=(.*)$", r.stdout, re.M):
        assert float(ms) > 0.0, r.stdout


@pytest.mark.parametrize("case", [c for c in CASES if c["file"].startswith("shapes/")],
                         ids=lambda c: c["file"])
def test_reference_program_unfused(case):
    # every map statement writes its array: the same output
    r = _run(os.path.join(MAPAL_DIR, case["file"]), "--no-fuse")
    assert r.returncode == case["rc"], (r.returncode, r.stdout, r.stderr)
    assert matches(r.stdout, case["expected"]), (r.stdout, case["expected"])
