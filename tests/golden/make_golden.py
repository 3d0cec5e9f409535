"""Generate tests/golden/reference_outputs.json from the reference itself.

Run where the reference tree is at hand ($MAPAL_REFERENCE, else a checkout
named `reference` beside this repository) after `make -C oracle ref`:

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
# The reference tree: $MAPAL_REFERENCE, else a checkout named `reference` beside
# this repository.
REF = os.environ.get("MAPAL_REFERENCE", os.path.join(os.path.dirname(ROOT), "reference"))
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


# The reference's own bench programs that the GPU driver must run unmodified:
# every benches/shapes source, the f32 cap matmuls, the counted-loop matmuls and
# the examples inside the bench subset. They are copied byte for byte into
# tests/golden/mapal/<dir>/ (test inputs, never product code).
PROGRAM_GLOBS = [("shapes", "benches/shapes", lambda f: f.endswith(".mapal")),
                 ("matmul", "benches/matmul", lambda f: re.fullmatch(r"matmul\d+(_cap_f32)?\.mapal", f)),
                 ("examples", "examples", lambda f: f in ("matmul4_loop.mapal", "matmul4096.mapal",
                                                          "vector_add.mapal", "zip_demo.mapal"))]
# Programs whose interpreter run is too long for the oracle evaluator here (or
# that it does not parse: counted loops): their expected output is the
# published known answer of the same product (results.csv; the loop and cap
# forms compute every cell in the same k order).
KNOWN_ANSWER_LEG = {"cap": "flow-cuda-cap-f32", "loop": "flow-cuda"}


def _known_answer(leg: str, n: int) -> tuple[int, int] | None:
    with open(os.path.join(REF, "benches/matmul/results.csv")) as f:
        for rec in csv.reader(f):
            if len(rec) >= 5 and rec[0] == leg and int(rec[1]) == n:
                m = re.match(r"out=(-?\d+)/(-?\d+)", rec[4])
                return int(m.group(1)), int(m.group(2))
    return None


def reference_programs() -> list[dict]:
    sys.path.insert(0, ROOT)
    from oracle.mapal_eval import Unsupported, expected

    out_dir = os.path.join(HERE, "mapal")
    cases = []
    for sub, rel, keep in PROGRAM_GLOBS:
        os.makedirs(os.path.join(out_dir, sub), exist_ok=True)
        for name in sorted(os.listdir(os.path.join(REF, rel))):
            if not keep(name):
                continue
            src = open(os.path.join(REF, rel, name), "rb").read()
            with open(os.path.join(out_dir, sub, name), "wb") as f:
                f.write(src)
            text = src.decode()
            m = re.fullmatch(r"matmul(\d+)(_cap_f32)?\.mapal", name)
            n = int(m.group(1)) if m else None
            case = {"file": f"{sub}/{name}", "source": f"{rel}/{name}"}
            if m and (n >= 2048 or not m.group(2)):
                c0_clast = _known_answer(KNOWN_ANSWER_LEG["cap"], n) or \
                    _known_answer(KNOWN_ANSWER_LEG["loop"], n)
                case.update({"expected": f"{c0_clast[0]}\n{c0_clast[1]}\n", "rc": 0,
                             "expected_from": f"benches/matmul/results.csv N={n}"})
                if "time" in text:
                    case["expected"] += "iter ms=\x00time\x00\n"
            else:
                try:
                    want, rc = expected(text)
                    case.update({"expected": want, "rc": rc, "expected_from": "oracle evaluator"})
                except Unsupported:
                    km = re.search(r"matmul(\d+)", name)
                    ka = _known_answer(KNOWN_ANSWER_LEG["loop"], int(km.group(1))) if km else None
                    if ka is None:
                        raise
                    case.update({"expected": f"{ka[0]}\n{ka[1]}\n", "rc": 0,
                                 "expected_from": f"benches/matmul/results.csv N={km.group(1)}"})
            cases.append(case)
    return cases


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
        "reference_programs": reference_programs(),
    }
    path = os.path.join(HERE, "reference_outputs.json")
    with open(path, "w") as f:
        json.dump(data, f, indent=1)
        f.write("\n")
    print(f"wrote {path}")
    return 0


if __name__ == "__main__":
    sys.exit(main())
