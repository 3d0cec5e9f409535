"""The general map body (mapal_gpu_map_expr) against the oracle's evaluation
of the same stack program: bit-exact values, and the trap classes of the
interpreter (index_oob for a read outside its array, div_zero for integer
/ or % by zero)."""
import numpy as np
import pytest
import torch

import flow_b200 as fb
import oracle as o
from _gpu import dev, empty_f32, host, same_bits

pytestmark = pytest.mark.gpu

P = fb.program


@pytest.fixture(scope="module")
def ctx():
    c = fb.Context((0,))
    yield c
    c.close()


def run_both(ctx, prog, arrays, n, out_i32=False):
    out = torch.empty(n, dtype=torch.int32 if out_i32 else torch.float32, device="cuda")
    ctx.map_expr(prog, [dev(a) for a in arrays], out, n)
    rc, want = o.map_expr(prog, arrays, n, np.int32 if out_i32 else np.float32)
    assert rc == 0
    return host(out), want


def test_generator_body(ctx):
    # t -> (t * 7 + 13) % 101 - 50 -> widen_f32   (benches/shapes/saxpy_1048576.mapal:8)
    prog = P(("T_I32",), ("CONST_I32", 7), ("MUL_I32",), ("CONST_I32", 13), ("ADD_I32",), ("CONST_I32", 101),
             ("REM_I32",), ("CONST_I32", 50), ("SUB_I32",), ("WIDEN_I32_F32",), ("STORE_F32",))
    got, want = run_both(ctx, prog, [], 1 << 20)
    assert same_bits(got, want) and same_bits(want, o.affine(1 << 20, 7, 13, 101, 50))


def test_zip_body_strict(ctx):
    # (x, y) -> zip -> map { p -> (p.0 * p.1 - 2.5) / p.0 }
    n = 100003
    x, y = o.gen(n, 1, 0), o.gen(n, 1, n)
    prog = P(("IN_F32", 0), ("IN_F32", 1), ("MUL_F32",), ("CONST_F32", 2.5), ("SUB_F32",), ("IN_F32", 0),
             ("DIV_F32",), ("STORE_F32",))
    got, want = run_both(ctx, prog, [x, y], n)
    assert same_bits(got, want)


def test_indexed_reads_and_int_ops(ctx):
    # t -> a[(t % 64) * 64 + t / 64] * 3.0 - a[t]
    n = 4096
    a = o.gen(n, 2, 0)
    prog = P(("T_I32",), ("CONST_I32", 64), ("REM_I32",), ("CONST_I32", 64), ("MUL_I32",), ("T_I32",),
             ("CONST_I32", 64), ("DIV_I32",), ("ADD_I32",), ("LOAD_F32", 0), ("CONST_F32", 3.0), ("MUL_F32",),
             ("T_I32",), ("LOAD_F32", 0), ("SUB_F32",), ("STORE_F32",))
    got, want = run_both(ctx, prog, [a], n)
    assert same_bits(got, want)


def test_int_result_and_negatives(ctx):
    # t -> -(t * 1021 + 12347) % 1000 / -3 (wrapping, truncating, dividend-signed)
    prog = P(("T_I32",), ("CONST_I32", 1021), ("MUL_I32",), ("CONST_I32", 12347), ("ADD_I32",), ("NEG_I32",),
             ("CONST_I32", 1000), ("REM_I32",), ("CONST_I32", -3), ("DIV_I32",), ("STORE_I32",))
    got, want = run_both(ctx, prog, [], 1 << 16, out_i32=True)
    assert np.array_equal(got, want)


def test_fmod_and_float_specials(ctx):
    n = 5000
    x = o.gen(n, 3, 0) * np.float32(10)
    y = o.gen(n, 3, n)
    y[::7] = 0.0
    prog = P(("IN_F32", 0), ("IN_F32", 1), ("REM_F32",), ("NEG_F32",), ("STORE_F32",))
    got, want = run_both(ctx, prog, [x, y], n)
    assert same_bits(got, want)


def test_traps(ctx):
    a = np.arange(10, dtype=np.float32)
    oob = P(("T_I32",), ("CONST_I32", 2), ("MUL_I32",), ("LOAD_F32", 0), ("STORE_F32",))
    with pytest.raises(fb.MapalTrap) as e:
        ctx.map_expr(oob, [dev(a)], empty_f32(8))
    assert e.value.kind == "index_oob"
    assert o.map_expr(oob, [a], 8)[0] == fb.TRAP_INDEX_OOB
    div0 = P(("CONST_I32", 5), ("T_I32",), ("DIV_I32",), ("STORE_I32",))
    with pytest.raises(fb.MapalTrap) as e:
        ctx.map_expr(div0, [], torch.empty(4, dtype=torch.int32, device="cuda"))
    assert e.value.kind == "div_zero"


def test_malformed_programs_rejected(ctx):
    for bad in [P(("T_I32",), ("STORE_F32",)),                       # type mismatch
                P(("CONST_F32", 1.0), ("CONST_I32", 1), ("ADD_F32",), ("STORE_F32",)),
                P(("T_I32",), ("WIDEN_I32_F32",)),                   # no store
                P(("IN_F32", 3), ("STORE_F32",))]:                   # slot beyond the table
        with pytest.raises(fb.MapalInfraError):
            ctx.map_expr(bad, [], empty_f32(4))


@pytest.mark.parametrize("n", [1, 3, 1023, 1025, 4097, 100001])
def test_ragged_domains_and_deep_stack(ctx, n):
    # ((t+1)*(t+2) + (t+3)*(t+4)) * ((t+5) - (t+6)*(t+7)) -> widen, with every
    # product's operands pushed first: the stack reaches depth 5, so values
    # below the top go through the spill slots; n exercises partial chunks.
    prog = P(("T_I32",), ("CONST_I32", 1), ("ADD_I32",), ("T_I32",), ("CONST_I32", 2), ("ADD_I32",),
             ("MUL_I32",), ("T_I32",), ("CONST_I32", 3), ("ADD_I32",), ("T_I32",), ("CONST_I32", 4),
             ("ADD_I32",), ("MUL_I32",), ("ADD_I32",), ("T_I32",), ("CONST_I32", 5), ("ADD_I32",),
             ("T_I32",), ("CONST_I32", 6), ("ADD_I32",), ("T_I32",), ("CONST_I32", 7), ("ADD_I32",),
             ("MUL_I32",), ("SUB_I32",), ("MUL_I32",), ("WIDEN_I32_F32",), ("STORE_F32",))
    got, want = run_both(ctx, prog, [], n)
    assert same_bits(got, want)


def test_constant_operands_in_both_positions(ctx):
    # 2.5 / x - (1.5 * 0.75) and 7 - t % 5: a constant as the left operand
    # stays a stack value; one right after another operand folds into the op
    n = 3001
    x = o.gen(n, 5, 0)
    prog = P(("CONST_F32", 2.5), ("IN_F32", 0), ("DIV_F32",), ("CONST_F32", 1.5), ("CONST_F32", 0.75),
             ("MUL_F32",), ("SUB_F32",), ("STORE_F32",))
    got, want = run_both(ctx, prog, [x], n)
    assert same_bits(got, want)
    prog = P(("CONST_I32", 7), ("T_I32",), ("CONST_I32", 5), ("REM_I32",), ("SUB_I32",), ("STORE_I32",))
    got, want = run_both(ctx, prog, [], n, out_i32=True)
    assert np.array_equal(got, want)


def test_trap_in_a_few_elements_of_many(ctx):
    # only elements t = 999999 and beyond read past the array: index_oob
    n = 1 << 20
    a = o.gen(999999, 6, 0)
    prog = P(("T_I32",), ("LOAD_F32", 0), ("STORE_F32",))
    with pytest.raises(fb.MapalTrap) as e:
        ctx.map_expr(prog, [dev(a)], empty_f32(n))
    assert e.value.kind == "index_oob"
    ok = empty_f32(999999)
    ctx.map_expr(prog, [dev(a)], ok)
    assert same_bits(host(ok), a)
