"""Generate tests/golden/reference_outputs.json from the reference itself.

Run in a container that has the reference tree (default /root/reference, or
$MAPAL_REFERENCE) after `make -C oracle ref`:

    python tests/golden/make_golden.py

Sources, all the reference's own:
  * benches/matmul/results.csv — c[0] / c[N*N-1] known answers of the matmul
    cap programs (the f32 rows of the flow-cuda-cap-kernel leg);
  * examples/matmul4_loop.mapal header — its documented output (-275, 3748);
  * crates/mapal-interp/tests/acceptance.rs — fir4 == 5.375;
  * crates/backends/cuda/tests/differential.rs — the float print parity pin;
  * the reference's C++ baseline programs (benches/matmul/cpp_mt.cpp,
    benches/shapes/ladder2_baseline.cpp, benches/shapes/shapes_baseline.cpp),
    compiled unmodified from the reference tree into oracle/_ref/ and run
    here: their printed probe values for the shapes the GPU kernels cover.
The fixture is committed; GPU test runs never read the reference tree.
"""
from __future__ import annotations

import csv
import json
import os
import re
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
REF = os.environ.get("MAPAL_REFERENCE", "/root/reference")
REF_BIN = os.path.join(ROOT, "oracle", "_ref")


def run(args: list[str]) -> list[str]:
    env = dict(os.environ, THREADS="1")
    out = subprocess.run(args, check=True, capture_output=True, text=True, env=env).stdout
    return [l for l in out.splitlines() if l and not l.startswith("iter ms=")]


def matmul_known_answers() -> list[dict]:
    rows = []
    with open(os.path.join(REF, "benches/matmul/results.csv")) as f:
        for rec in csv.reader(f):
            if len(rec) < 5 or rec[0] != "flow-cuda-cap-kernel-f32":
                continue
            m = re.match(r"out=(-?\d+)/(-?\d+)", rec[4])
            rows.append({"n": int(rec[1]), "c0": int(m.group(1)), "clast": int(m.group(2)),
                         "source": "benches/matmul/results.csv"})
    return rows


def matmul4_loop() -> dict:
    text = open(os.path.join(REF, "examples/matmul4_loop.mapal")).read()
    m = re.search(r"prints (-?\d+) then (-?\d+)", text)
    return {"n": 4, "c0": int(m.group(1)), "clast": int(m.group(2)),
            "source": "examples/matmul4_loop.mapal header"}


def fir4() -> dict:
    text = open(os.path.join(REF, "crates/mapal-interp/tests/acceptance.rs")).read()
    m = re.search(r'run\(&ir, BUDGET\)\.output, "([0-9.]+)\\n"\);\s*\}\s*', text[text.index("fn golden_fir"):])
    return {"signal": [1.0, 2.0, 3.0, 4.0, 5.0, 6.0, 7.0, 8.0],
            "coeffs": [0.5, 0.25, 0.125, 0.0625], "window_start": 4,
            "output": m.group(1), "source": "crates/mapal-interp/tests/acceptance.rs golden_fir"}


def float_print_pin() -> dict:
    text = open(os.path.join(REF, "crates/backends/cuda/tests/differential.rs")).read()
    body = text[text.index("fn differential_float_print_parity"):]
    m = re.search(r'rr\.output, "([^"]+)",\s*"oracle contract"', body)
    lines = m.group(1).replace("\\n", "\n").splitlines()
    # The program's values, in print order (f64, f32, f64, f64, f64, f64, f64).
    return {"lines": lines,
            "values": ["f64:0.1+0.2", "f32:1/3", "f64:1/0", "f64:-1/0", "f64:0/0",
                       "f64:fmod(7.5,2)", "f64:fmod(-7.5,2)"],
            "source": "crates/backends/cuda/tests/differential.rs differential_float_print_parity"}


def cpp_mt() -> list[dict]:
    out = []
    for n in (4, 16, 64, 128, 256):
        line = run([os.path.join(REF_BIN, "cpp_mt"), str(n), "1", "f32"])[0]
        m = re.search(r"c0=(-?[\d.]+) clast=(-?[\d.]+)", line)
        out.append({"n": n, "c0": float(m.group(1)), "clast": float(m.group(2)),
                    "source": "benches/matmul/cpp_mt.cpp"})
    return out


def ladder2() -> list[dict]:
    cases = [("saxpy", 256), ("saxpy", 1048576), ("reduce", 256), ("reduce", 1048576),
             ("transpose", 16), ("transpose", 1024), ("gather", 256), ("gather", 1048576)]
    out = []
    for shape, n in cases:
        vals = run([os.path.join(REF_BIN, "ladder2_baseline"), shape, "1t", "1", str(n)])
        out.append({"shape": shape, "size": n, "printf": "%g", "values": vals,
                    "source": "benches/shapes/ladder2_baseline.cpp"})
    return out


def shapes() -> list[dict]:
    cases = [("fir", 256), ("fir", 65536), ("fir", 1048576), ("conv2d", 16), ("conv2d", 20),
             ("conv2d", 92), ("conv2d", 512), ("conv2d", 1024)]
    out = []
    for shape, n in cases:
        vals = run([os.path.join(REF_BIN, "shapes_baseline"), shape, "1t", "1", str(n)])
        out.append({"shape": shape, "size": n, "printf": "%.9g", "values": vals,
                    "source": "benches/shapes/shapes_baseline.cpp"})
    return out


def main() -> int:
    if not os.path.isdir(os.path.join(REF, "benches")):
        print(f"reference tree not found at {REF}", file=sys.stderr)
        return 2
    data = {
        "matmul_known_answers": [matmul4_loop()] + matmul_known_answers(),
        "fir4": fir4(),
        "float_print_pin": float_print_pin(),
        "cpp_mt": cpp_mt(),
        "ladder2": ladder2(),
        "shapes": shapes(),
    }
    path = os.path.join(HERE, "reference_outputs.json")
    with open(path, "w") as f:
        json.dump(data, f, indent=1)
        f.write("\n")
    print(f"wrote {path}")
    return 0


if __name__ == "__main__":
    sys.exit(main())
