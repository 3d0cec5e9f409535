"""ctypes view of the CPU oracle (oracle/mapal_oracle.c).

TEST INFRASTRUCTURE ONLY: the reference results that tests/, the smoke check
and the bench's CPU-baseline leg compare against. The product (flow_b200 and
libmapal_gpu) never imports this package.
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "_build", "liboracle.so")
_REF_DIR = os.path.join(_HERE, "_ref")

_lib = None


def build() -> None:
    """Compile liboracle.so (and, when the reference tree is present, the
    reference's own C++ baselines into oracle/_ref)."""
    subprocess.run(["make", "-s", "-C", _HERE], check=True)
    # $MAPAL_REFERENCE, else a checkout named `reference` beside this repository
    ref = os.environ.get("MAPAL_REFERENCE", os.path.join(os.path.dirname(os.path.dirname(_HERE)), "reference"))
    if os.path.isdir(os.path.join(ref, "benches")):
        subprocess.run(["make", "-s", "-C", _HERE, "ref", f"REF={ref}"], check=True)


def ref_binary(name: str) -> str:
    """Path of a reference baseline built by `make -C oracle ref`."""
    return os.path.join(_REF_DIR, name)


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        if not os.path.exists(_LIB_PATH):
            build()
        _lib = ctypes.CDLL(_LIB_PATH)
        _declare(_lib)
    return _lib


# The record layouts of include/mapal_gpu.h, shared with the product binding.
class KSplit(ctypes.Structure):
    _fields_ = [("div", ctypes.c_uint64), ("cq", ctypes.c_uint64), ("cr", ctypes.c_uint64)]


class TileRead(ctypes.Structure):
    _fields_ = [
        ("base", ctypes.c_uint64),
        ("ci", ctypes.c_uint64),
        ("ck", ctypes.c_uint64),
        ("clane", ctypes.c_uint64),
        ("ksplit", KSplit),
        ("len", ctypes.c_uint64),
    ]


class TileSite(ctypes.Structure):
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
    _fields_ = [
        ("width", ctypes.c_uint64),
        ("rows", ctypes.c_uint64),
        ("cq", ctypes.c_uint64),
        ("cr", ctypes.c_uint64),
        ("len", ctypes.c_uint64),
    ]


_fp = ctypes.POINTER(ctypes.c_float)
_ip = ctypes.POINTER(ctypes.c_int32)
_i64 = ctypes.c_int64
_i32 = ctypes.c_int32


def _declare(L: ctypes.CDLL) -> None:
    L.or_gen_hash.argtypes = [_i32, _i32]
    L.or_gen_hash.restype = _i32
    L.or_gen_u11.argtypes = [_i32, _i32]
    L.or_gen_u11.restype = ctypes.c_float
    L.or_gen_u01.argtypes = [_i32, _i32]
    L.or_gen_u01.restype = ctypes.c_float
    L.or_gen_index.argtypes = [_i32, _i32, _i32]
    L.or_gen_index.restype = _i32
    L.or_fill_gen.argtypes = [_fp, _i64, _i32, _i64, ctypes.c_int]
    L.or_fill_index.argtypes = [_ip, _i64, _i32, _i64, _i32]
    L.or_fill_affine.argtypes = [_fp, _i64, _i64, _i32, _i32, _i32, _i32]
    L.or_saxpy.argtypes = [ctypes.c_float, _fp, _fp, _fp, _i64]
    L.or_zip_map.argtypes = [ctypes.c_int, _fp, _fp, _fp, _i64]
    L.or_move_site.argtypes = [ctypes.POINTER(MoveSite), _fp, _fp]
    L.or_gather.argtypes = [_fp, _i64, _ip, _fp, _i64]
    L.or_fold_sum.argtypes = [ctypes.c_float, _fp, _i64]
    L.or_fold_sum.restype = ctypes.c_float
    L.or_sum_f64.argtypes = [ctypes.c_float, _fp, _i64]
    L.or_sum_f64.restype = ctypes.c_double
    L.or_sum_abs_f64.argtypes = [_fp, _i64]
    L.or_sum_abs_f64.restype = ctypes.c_double
    L.or_tile_site.argtypes = [ctypes.POINTER(TileSite), _fp, _fp, _fp]
    L.or_matmul_rows.argtypes = [_fp, _fp, _fp, _i64, _i64, _i64, _i64, _i64, ctypes.c_int]
    L.or_matmul_cell.argtypes = [_fp, _fp, _i64, _i64, _i64, _i64]
    L.or_matmul_cell.restype = ctypes.c_float
    L.or_fir.argtypes = [_fp, _i64, _fp, _fp, _i64]
    L.or_conv2d_3x3.argtypes = [_fp, _fp, _i64, _fp, _i64, _i64]
    L.or_render_f32.argtypes = [ctypes.c_float, ctypes.c_char_p, ctypes.c_int]
    L.or_render_f64.argtypes = [ctypes.c_double, ctypes.c_char_p, ctypes.c_int]


def _f(a: np.ndarray):
    assert a.dtype == np.float32 and a.flags.c_contiguous
    return a.ctypes.data_as(_fp)


def _i(a: np.ndarray):
    assert a.dtype == np.int32 and a.flags.c_contiguous
    return a.ctypes.data_as(_ip)


# ---- generators -------------------------------------------------------------

U11, U01 = 0, 1


def gen(n: int, seed: int, offset: int = 0, kind: int = U11) -> np.ndarray:
    out = np.empty(n, np.float32)
    lib().or_fill_gen(_f(out), n, seed, offset, kind)
    return out


def gen_index(n: int, seed: int, offset: int, rng: int) -> np.ndarray:
    out = np.empty(n, np.int32)
    lib().or_fill_index(_i(out), n, seed, offset, rng)
    return out


def affine(n: int, mul: int, add: int, mod: int, sub: int, start: int = 0) -> np.ndarray:
    out = np.empty(n, np.float32)
    lib().or_fill_affine(_f(out), n, start, mul, add, mod, sub)
    return out


# ---- sites ----------------------------------------------------------------------


def saxpy(a: float, x: np.ndarray, y0: np.ndarray) -> np.ndarray:
    y = np.empty_like(x)
    lib().or_saxpy(a, _f(x), _f(y0), _f(y), x.size)
    return y


def zip_map(op: int, x: np.ndarray, y: np.ndarray) -> np.ndarray:
    out = np.empty_like(x)
    rc = lib().or_zip_map(op, _f(x), _f(y), _f(out), x.size)
    assert rc == 0
    return out


def move_site(site: MoveSite, a: np.ndarray):
    out = np.empty(site.rows * site.width, np.float32)
    rc = lib().or_move_site(ctypes.byref(site), _f(a), _f(out))
    return rc, out


def gather(x: np.ndarray, idx: np.ndarray):
    out = np.empty(idx.size, np.float32)
    rc = lib().or_gather(_f(x), x.size, _i(idx), _f(out), idx.size)
    return rc, out


def fold_sum(seed: float, x: np.ndarray) -> float:
    return float(np.float32(lib().or_fold_sum(seed, _f(x), x.size)))


def sum_f64(seed: float, x: np.ndarray) -> float:
    return lib().or_sum_f64(seed, _f(x), x.size)


def sum_abs_f64(x: np.ndarray) -> float:
    return lib().or_sum_abs_f64(_f(x), x.size)


def tile_site(site: TileSite, a: np.ndarray, b: np.ndarray):
    out = np.empty(site.rows * site.c, np.float32)
    rc = lib().or_tile_site(ctypes.byref(site), _f(a), _f(b), _f(out))
    return rc, out


def matmul(A: np.ndarray, B: np.ndarray, M: int, N: int, K: int, row0: int = 0,
           row1: int | None = None, threads: int = 1) -> np.ndarray:
    row1 = M if row1 is None else row1
    C = np.zeros(M * N, np.float32)
    lib().or_matmul_rows(_f(A), _f(B), _f(C), M, N, K, row0, row1, threads)
    return C


def matmul_cell(A: np.ndarray, B: np.ndarray, N: int, K: int, i: int, j: int) -> float:
    return float(np.float32(lib().or_matmul_cell(_f(A), _f(B), N, K, i, j)))


def fir(w: np.ndarray, x: np.ndarray, n_out: int) -> np.ndarray:
    y = np.empty(n_out, np.float32)
    lib().or_fir(_f(w), w.size, _f(x), _f(y), n_out)
    return y


def conv2d_3x3(w: np.ndarray, img: np.ndarray, stride: int, out_rows: int,
               out_cols: int) -> np.ndarray:
    out = np.empty(out_rows * out_cols, np.float32)
    lib().or_conv2d_3x3(_f(w), _f(img), stride, _f(out), out_rows, out_cols)
    return out


def render_f32(v: float) -> str:
    buf = ctypes.create_string_buffer(64)
    n = lib().or_render_f32(v, buf, 64)
    assert n >= 0
    return buf.value.decode()


def render_f64(v: float) -> str:
    buf = ctypes.create_string_buffer(400)
    n = lib().or_render_f64(v, buf, 400)
    assert n >= 0
    return buf.value.decode()


# ---- record builders (the reference's recognised site records) -------------------


def matmul_site(M: int, N: int, K: int) -> TileSite:
    """TileSite of the matmul cap form: rows=M, c=N, k=K, a{ci=K, ck=1},
    b{ck=N, clane=1}, seed 0.0 (tile_sites_pin record for matmul*_cap_f32)."""
    s = TileSite()
    s.rows, s.c, s.k = M, N, K
    s.a.ci, s.a.ck, s.a.len = K, 1, M * K
    s.b.ck, s.b.clane, s.b.len = N, 1, K * N
    s.seed = 0.0
    s.mul_a_first = 1
    s.add_acc_first = 1
    return s


def fir_site(n_out: int, taps: int) -> TileSite:
    """TileSite of the FIR window: rows=1, c=n_out, a=w{ck=1}, b=x{ck=1, clane=1}."""
    s = TileSite()
    s.rows, s.c, s.k = 1, n_out, taps
    s.a.ck, s.a.len = 1, taps
    s.b.ck, s.b.clane, s.b.len = 1, 1, n_out + taps - 1
    s.mul_a_first = 1
    s.add_acc_first = 1
    return s


def conv2d_site(out_rows: int, out_cols: int, stride: int, img_len: int) -> TileSite:
    """TileSite of the 3x3 conv: a=w{ck=1}, b=img{ci=stride, clane=1,
    ksplit div3 cq=stride cr=1} (tile_sites_pin record for conv2d_1024)."""
    s = TileSite()
    s.rows, s.c, s.k = out_rows, out_cols, 9
    s.a.ck, s.a.len = 1, 9
    s.b.ci, s.b.clane, s.b.len = stride, 1, img_len
    s.b.ksplit.div, s.b.ksplit.cq, s.b.ksplit.cr = 3, stride, 1
    s.mul_a_first = 1
    s.add_acc_first = 1
    return s


def transpose_site(R: int, C: int) -> MoveSite:
    """MoveSite of out = transpose(in), in R x C row-major: width=R, rows=C, cq=1, cr=C."""
    s = MoveSite()
    s.width, s.rows, s.cq, s.cr, s.len = R, C, 1, C, R * C
    return s


class ExprOp(ctypes.Structure):
    """MAPAL_X_* op (include/mapal_gpu.h)."""
    _fields_ = [("code", ctypes.c_uint16), ("slot", ctypes.c_uint16), ("i", ctypes.c_int32),
                ("f", ctypes.c_float)]


def map_expr(prog, arrays: list, n: int, out_dtype=np.float32):
    """Evaluate a map-body program over [0, n): (rc, out)."""
    L = lib()
    L.or_map_expr.argtypes = [ctypes.POINTER(ExprOp), ctypes.c_uint32, ctypes.POINTER(ctypes.c_void_p),
                              ctypes.POINTER(ctypes.c_uint64), ctypes.c_uint32, ctypes.c_void_p, ctypes.c_uint64]
    ops = (ExprOp * len(prog))()
    for k, p in enumerate(prog):
        ops[k].code, ops[k].slot, ops[k].i, ops[k].f = p.code, p.slot, p.i, p.f
    ptrs = (ctypes.c_void_p * max(1, len(arrays)))(*[a.ctypes.data for a in arrays])
    lens = (ctypes.c_uint64 * max(1, len(arrays)))(*[a.size for a in arrays])
    out = np.zeros(n, out_dtype)
    rc = L.or_map_expr(ops, len(prog), ptrs, lens, len(arrays), out.ctypes.data, n)
    return rc, out
