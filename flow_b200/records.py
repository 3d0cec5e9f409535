"""The site records that cross the C ABI (include/mapal_gpu.h), as ctypes
structures, and builders for the shapes the reference recognizes.

Field meaning follows the reference's records:
TileRead / TileKSplit / TileSite (crates/mapal-ir/src/algo.rs:221-345) and
MoveSite (algo.rs:309-333). `len` fields are this ABI's addition: the read
array's length, which the reference knows from the array type.
"""
from __future__ import annotations

import ctypes


class KSplit(ctypes.Structure):
    """k = kq*div + kr decomposition of a fold axis (TileKSplit, algo.rs:245-257)."""
    _fields_ = [("div", ctypes.c_uint64), ("cq", ctypes.c_uint64), ("cr", ctypes.c_uint64)]


class TileRead(ctypes.Structure):
    """addr = base + ci*i + clane*lane + ck*k + cq*(k/div) + cr*(k%div) (algo.rs:227-240)."""
    _fields_ = [
        ("base", ctypes.c_uint64),
        ("ci", ctypes.c_uint64),
        ("ck", ctypes.c_uint64),
        ("clane", ctypes.c_uint64),
        ("ksplit", KSplit),
        ("len", ctypes.c_uint64),
    ]


class TileSite(ctypes.Structure):
    """A recognized map-of-fold site (algo.rs:335-345)."""
    _fields_ = [
        ("rows", ctypes.c_uint64),
        ("c", ctypes.c_uint64),
        ("k", ctypes.c_uint64),
        ("a", TileRead),
        ("b", TileRead),
        ("seed", ctypes.c_float),
        ("mul_a_first", ctypes.c_uint8),
        ("add_acc_first", ctypes.c_uint8),
        ("reserved", ctypes.c_uint8 * 2),
    ]


class MoveSite(ctypes.Structure):
    """A fold-less move site: out[t] = in[cq*(t/width) + cr*(t%width)] (algo.rs:309-333)."""
    _fields_ = [
        ("width", ctypes.c_uint64),
        ("rows", ctypes.c_uint64),
        ("cq", ctypes.c_uint64),
        ("cr", ctypes.c_uint64),
        ("len", ctypes.c_uint64),
    ]


class ExprOp(ctypes.Structure):
    """One op of a general map body (MAPAL_X_* in include/mapal_gpu.h)."""
    _fields_ = [("code", ctypes.c_uint16), ("slot", ctypes.c_uint16), ("i", ctypes.c_int32),
                ("f", ctypes.c_float)]


# MAPAL_X_* op codes
X = dict(T_I32=0, CONST_I32=1, CONST_F32=2, IN_I32=3, IN_F32=4, LOAD_I32=5, LOAD_F32=6, ADD_I32=10,
         SUB_I32=11, MUL_I32=12, DIV_I32=13, REM_I32=14, NEG_I32=15, ADD_F32=20, SUB_F32=21, MUL_F32=22,
         DIV_F32=23, REM_F32=24, NEG_F32=25, WIDEN_I32_F32=30, STORE_I32=40, STORE_F32=41)


def program(*ops) -> ctypes.Array:
    """Build an ExprOp array from (name[, slot | imm]) tuples, e.g.
    program(("T_I32",), ("CONST_I32", 7), ("MUL_I32",), ("WIDEN_I32_F32",), ("STORE_F32",))."""
    arr = (ExprOp * len(ops))()
    for k, op in enumerate(ops):
        name = op[0]
        arr[k].code = X[name]
        if len(op) > 1:
            if name in ("IN_I32", "IN_F32", "LOAD_I32", "LOAD_F32"):
                arr[k].slot = op[1]
            elif name == "CONST_F32":
                arr[k].f = op[1]
            else:
                arr[k].i = op[1]
    return arr


class GpuProfile(ctypes.Structure):
    """Machine facts (the sm_100a counterpart of profile.rs:99-156 Machine::Gpu)."""
    _fields_ = [
        ("device", ctypes.c_int32),
        ("cc_major", ctypes.c_int32),
        ("cc_minor", ctypes.c_int32),
        ("sm_count", ctypes.c_int32),
        ("warp_size", ctypes.c_int32),
        ("max_threads_per_block", ctypes.c_int32),
        ("max_threads_per_sm", ctypes.c_int32),
        ("regs_per_sm", ctypes.c_int32),
        ("smem_per_sm", ctypes.c_int64),
        ("smem_per_block_optin", ctypes.c_int64),
        ("l2_bytes", ctypes.c_int64),
        ("tmem_bytes_per_sm", ctypes.c_int64),
        ("hbm_bytes", ctypes.c_int64),
        ("sm_clock_khz", ctypes.c_int32),
        ("mem_clock_khz", ctypes.c_int32),
        ("mem_bus_bits", ctypes.c_int32),
        ("cluster_launch", ctypes.c_int32),
        ("name", ctypes.c_char * 96),
    ]


def matmul_site(M: int, N: int, K: int, lda: int | None = None, ldb: int | None = None) -> TileSite:
    """The matmul cap form's record: rows=M, c=N, k=K, a{ci=lda, ck=1}, b{ck=ldb, clane=1},
    seed 0.0 (tile_sites_pin record of benches/matmul/matmul*_cap_f32.mapal)."""
    lda = K if lda is None else lda
    ldb = N if ldb is None else ldb
    s = TileSite()
    s.rows, s.c, s.k = M, N, K
    s.a.ci, s.a.ck, s.a.len = lda, 1, (M - 1) * lda + K if M else 0
    s.b.ck, s.b.clane, s.b.len = ldb, 1, (K - 1) * ldb + N if K else 0
    s.seed = 0.0
    s.mul_a_first, s.add_acc_first = 1, 1
    return s


def fir_site(n_out: int, taps: int) -> TileSite:
    """The FIR window record: rows=1, c=n_out, k=taps, a=w{ck=1}, b=x{ck=1, clane=1}
    (tile_sites_pin record of benches/shapes/fir_1048576.mapal)."""
    s = TileSite()
    s.rows, s.c, s.k = 1, n_out, taps
    s.a.ck, s.a.len = 1, taps
    s.b.ck, s.b.clane, s.b.len = 1, 1, n_out + taps - 1
    s.mul_a_first, s.add_acc_first = 1, 1
    return s


def conv2d_site(out_rows: int, out_cols: int, stride: int, img_len: int) -> TileSite:
    """The 3x3 conv record: rows, c, k=9, a=w{ck=1}, b=img{ci=stride, clane=1,
    ksplit div3 cq=stride cr1} (tile_sites_pin record of benches/shapes/conv2d_1024.mapal)."""
    s = TileSite()
    s.rows, s.c, s.k = out_rows, out_cols, 9
    s.a.ck, s.a.len = 1, 9
    s.b.ci, s.b.clane, s.b.len = stride, 1, img_len
    s.b.ksplit.div, s.b.ksplit.cq, s.b.ksplit.cr = 3, stride, 1
    s.mul_a_first, s.add_acc_first = 1, 1
    return s


def transpose_site(R: int, C: int) -> MoveSite:
    """out = transpose(in) for in R x C row-major: width=R, rows=C, cq=1, cr=C
    (the MoveSite of benches/shapes/transpose_1024.mapal with R = C = 1024)."""
    s = MoveSite()
    s.width, s.rows, s.cq, s.cr, s.len = R, C, 1, C, R * C
    return s
