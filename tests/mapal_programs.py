"""Mapal source text for the bench shapes, at any size, written for these tests.

The inputs are the integer generators the reference's benches and C++
baselines use, so the printed values are pinned by the known answers in
tests/golden/reference_outputs.json:
  A / x:  (t*7 + 13) % 101 - 50      B:  (t*7 + 57) % 101 - 50
  y0 / w: (t*5 + 3) % 31 - 15        gather index: (t*1021 + 12347) % n
Each program prints the first and the last output element.
"""
from __future__ import annotations

GEN_A = "(t * 7 + 13) % 101 - 50 -> widen_f32"
GEN_B = "(t * 7 + 57) % 101 - 50 -> widen_f32"
GEN_W = "(t * 5 + 3) % 31 - 15 -> widen_f32"


def matmul(n: int) -> str:
    nn = n * n
    return f"""// {n} x {n} product, each cell a strict fold over k
fn main() {{
    {nn} -> iota -> cells;
    cells -> map {{ t -> {GEN_A} }} -> a;
    cells -> map {{ t -> {GEN_B} }} -> b;
    {n} -> iota -> ks;
    cells -> map {{ t -> (0.0, ks) -> fold {{ acc, k -> acc + a[(t / {n}) * {n} + k] * b[k * {n} + t % {n}] }} }} -> c;
    c[0] -> println;
    c[{nn - 1}] -> println;
}}
"""


def saxpy(n: int) -> str:
    return f"""fn main() {{
    {n} -> iota -> dom;
    dom -> map {{ t -> {GEN_A} }} -> x;
    dom -> map {{ t -> {GEN_W} }} -> y0;
    (x, y0) -> zip -> map {{ p -> 2.5 * p.0 + p.1 }} -> y;
    y[0] -> println;
    y[{n - 1}] -> println;
}}
"""


def reduce(n: int) -> str:
    return f"""fn main() {{
    {n} -> iota -> dom;
    dom -> map {{ t -> {GEN_A} }} -> x;
    (0.0, x) -> fold {{ acc, v -> acc + v }} -> s;
    s -> println;
}}
"""


def transpose(side: int) -> str:
    nn = side * side
    return f"""fn main() {{
    {nn} -> iota -> dom;
    dom -> map {{ t -> {GEN_A} }} -> a;
    dom -> map {{ t -> a[(t % {side}) * {side} + t / {side}] }} -> b;
    b[0] -> println;
    b[{nn - 1}] -> println;
}}
"""


def gather(n: int) -> str:
    return f"""fn main() {{
    {n} -> iota -> dom;
    dom -> map {{ t -> {GEN_A} }} -> x;
    dom -> map {{ t -> (t * 1021 + 12347) % {n} }} -> idx;
    idx -> map {{ j -> x[j] }} -> y;
    y[0] -> println;
    y[{n - 1}] -> println;
}}
"""


def fir(n: int, taps: int = 64) -> str:
    return f"""fn main() {{
    {n + taps - 1} -> iota -> xi;
    xi -> map {{ t -> {GEN_A} }} -> x;
    {taps} -> iota -> ks;
    ks -> map {{ t -> {GEN_W} }} -> w;
    {n} -> iota -> outs;
    outs -> map {{ t -> (0.0, ks) -> fold {{ acc, k -> acc + w[k] * x[t + k] }} }} -> y;
    y[0] -> println;
    y[{n - 1}] -> println;
}}
"""


def conv2d(n: int) -> str:
    s = n + 2
    return f"""fn main() {{
    {s * s} -> iota -> px;
    px -> map {{ t -> {GEN_A} }} -> img;
    9 -> iota -> ks;
    ks -> map {{ t -> {GEN_W} }} -> w;
    {n * n} -> iota -> outs;
    outs -> map {{ t -> (0.0, ks) -> fold {{ acc, k -> acc + w[k] * img[(t / {n} + k / 3) * {s} + t % {n} + k % 3] }} }} -> o;
    o[0] -> println;
    o[{n * n - 1}] -> println;
}}
"""


FLOAT_PRINT = """fn main() {
    0.1 + 0.2 -> println;
    1 -> widen_f32 -> one;
    one / 3.0 -> println;
    1.0 / 0.0 -> println;
    -1.0 / 0.0 -> println;
    0.0 / 0.0 -> println;
    7.5 % 2.0 -> println;
    -7.5 % 2.0 -> println;
}
"""


def matmul_loops(n: int, literals: bool = False) -> str:
    """The same product in the counted-loop form: a dot-product helper with a
    (counter, accumulator) loop and a product helper whose loop writes every
    element of its result once, which the driver lifts into fold / map."""
    nn = n * n
    if literals:
        gen = lambda mul, add: ", ".join(f"{((t * mul + add) % 101) - 50}.0" for t in range(nn))
        inputs = f"""    [{gen(7, 13)}] -> a;
    [{gen(7, 57)}] -> b;"""
    else:
        inputs = f"""    {nn} -> iota -> cells;
    cells -> map {{ t -> {GEN_A} }} -> a;
    cells -> map {{ t -> {GEN_B} }} -> b;"""
    return f"""fn dot(x: [f32; {nn}], y: [f32; {nn}], row: i32, col: i32) -> f32 {{
    mut s: i32 <- 0;
    mut total: f32 <- 0.0;
    loop {{
        (s < {n}) -> {{
            -true-> {{
                total + x[row * {n} + s] * y[s * {n} + col] -> total;
                s + 1 -> s;
                -> loop;
            }}
            -false-> total -> ret;
        }}
    }}
}}

fn product(x: [f32; {nn}], y: [f32; {nn}]) -> [f32; {nn}] {{
    mut out: [f32; {nn}] <- x;
    mut cell: i32 <- 0;
    loop {{
        (cell < {nn}) -> {{
            -true-> {{
                cell / {n} -> r;
                cell % {n} -> c;
                (x, y, r, c) -> dot -> v;
                out[cell] <- v;
                cell + 1 -> cell;
                -> loop;
            }}
            -false-> out -> ret;
        }}
    }}
}}

fn main() {{
{inputs}
    (a, b) -> product -> prod;
    prod[0] -> println;
    prod[{nn - 1}] -> println;
}}
"""
