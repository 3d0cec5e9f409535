"""ctypes binding of libmapal_gpu.so (include/mapal_gpu.h, include/mapal_rt.h).

The library is built in-tree (python -m flow_b200.build). Loading fails
loudly when it is missing: there is no CPU fallback for any site.
"""
from __future__ import annotations

import ctypes
import os

from .records import ExprOp, GpuProfile, MoveSite, TileSite

LIB_PATH = os.path.join(os.path.dirname(os.path.abspath(__file__)), "libmapal_gpu.so")

_c = ctypes
_vp = _c.c_void_p
_u64 = _c.c_uint64
_i64 = _c.c_int64
_i32 = _c.c_int32
_int = _c.c_int
_f32 = _c.c_float
_pp = _c.POINTER(_c.c_void_p)
_pu64 = _c.POINTER(_c.c_uint64)

# name -> (restype, argtypes), one entry per function of include/*.h
SIGNATURES: dict[str, tuple] = {
    "mapal_gpu_abi_version": (_int, []),
    "mapal_gpu_last_error": (_c.c_char_p, []),
    "mapal_gpu_launch_count": (_u64, []),
    "mapal_gpu_device_count": (_int, [_c.POINTER(_int)]),
    "mapal_gpu_ctx_create": (_int, [_c.c_uint32, _pp]),
    "mapal_gpu_nccl_unique_id": (_int, [_c.c_char_p]),
    "mapal_gpu_ctx_create_rank": (_int, [_int, _int, _int, _c.c_char_p, _pp]),
    "mapal_gpu_ctx_destroy": (_int, [_vp]),
    "mapal_gpu_ctx_local_devices": (_int, [_vp, _c.POINTER(_int)]),
    "mapal_gpu_ctx_world": (_int, [_vp, _c.POINTER(_int), _c.POINTER(_int)]),
    "mapal_gpu_ctx_sum_combine": (_int, [_vp, _c.POINTER(_int)]),
    "mapal_gpu_profile": (_int, [_vp, _int, _c.POINTER(GpuProfile)]),
    "mapal_gpu_get_stream": (_int, [_vp, _int, _pp]),
    "mapal_gpu_set_stream": (_int, [_vp, _int, _vp]),
    "mapal_gpu_set_sync": (_int, [_vp, _int]),
    "mapal_gpu_synchronize": (_int, [_vp]),
    "mapal_gpu_iota_i32": (_int, [_vp, _vp, _u64]),
    "mapal_gpu_fill_f32": (_int, [_vp, _vp, _f32, _u64]),
    "mapal_gpu_widen_i32_f32": (_int, [_vp, _vp, _vp, _u64]),
    "mapal_gpu_gen_affine_f32": (_int, [_vp, _vp, _u64, _i64, _i32, _i32, _i32, _i32]),
    "mapal_gpu_gen_f32": (_int, [_vp, _vp, _u64, _i32, _i64, _int]),
    "mapal_gpu_gen_index_i32": (_int, [_vp, _vp, _u64, _i32, _i64, _i32]),
    "mapal_gpu_map_saxpy": (_int, [_vp, _f32, _vp, _vp, _vp, _u64]),
    "mapal_gpu_zip_map_f32": (_int, [_vp, _int, _vp, _vp, _vp, _u64]),
    "mapal_gpu_map_expr": (_int, [_vp, _c.POINTER(ExprOp), _c.c_uint32, _pp, _pu64, _c.c_uint32, _vp, _u64]),
    "mapal_gpu_transpose": (_int, [_vp, _c.POINTER(MoveSite), _vp, _vp]),
    "mapal_gpu_gather": (_int, [_vp, _vp, _u64, _vp, _vp, _u64]),
    "mapal_gpu_fold_sum_f32": (_int, [_vp, _f32, _vp, _u64, _vp]),
    "mapal_gpu_fold_sum_f32_strict": (_int, [_vp, _f32, _vp, _u64, _vp]),
    "mapal_gpu_fold_sum_i32": (_int, [_vp, _i32, _vp, _u64, _vp]),
    "mapal_gpu_fold_sum_f32_noalloc": (_int, [_f32, _vp, _u64, _vp, _vp]),
    "mapal_gpu_fir_f32": (_int, [_vp, _c.POINTER(TileSite), _vp, _vp, _vp]),
    "mapal_gpu_conv2d_3x3_f32": (_int, [_vp, _c.POINTER(TileSite), _vp, _vp, _vp]),
    "mapal_gpu_matmul_f32": (_int, [_vp, _c.POINTER(TileSite), _vp, _vp, _vp, _int]),
    "mapal_gpu_matmul_f32_host": (_int, [_vp, _c.POINTER(TileSite), _vp, _vp, _vp, _int]),
    "mapal_gpu_matmul_f32_host_sharded": (_int, [_vp, _c.POINTER(TileSite), _vp, _vp, _vp, _vp, _int]),
    "mapal_gpu_tile_site_f32": (_int, [_vp, _c.POINTER(TileSite), _vp, _vp, _vp, _int]),
    "mapal_gpu_shard_range": (_int, [_u64, _int, _int, _pu64, _pu64]),
    "mapal_gpu_saxpy_sharded": (_int, [_vp, _f32, _pp, _pp, _pp, _pu64]),
    "mapal_gpu_fold_sum_f32_sharded": (_int, [_vp, _f32, _pp, _pu64, _pp]),
    "mapal_gpu_broadcast_f32": (_int, [_vp, _pp, _u64, _int]),
    "mapal_gpu_gather_sharded": (_int, [_vp, _pp, _u64, _pp, _pp, _pu64]),
    "mapal_gpu_matmul_f32_sharded": (_int, [_vp, _c.POINTER(TileSite), _pp, _pp, _pp, _pu64, _int, _int]),
    "mapal_gpu_probe_mma_peak": (_int, [_vp, _int, _c.c_uint32, _c.POINTER(_c.c_double)]),
    "mapal_gpu_probe_launch_floor": (_int, [_vp, _int, _vp, _u64, _vp]),
    # mapal-rt re-exports (include/mapal_rt.h)
    "mapal_print_i32": (None, [_i32, _c.c_bool]),
    "mapal_print_i64": (None, [_i64, _c.c_bool]),
    "mapal_print_u8": (None, [_c.c_uint8, _c.c_bool]),
    "mapal_print_bool": (None, [_c.c_bool, _c.c_bool]),
    "mapal_print_f32": (None, [_f32, _c.c_bool]),
    "mapal_print_f64": (None, [_c.c_double, _c.c_bool]),
    "mapal_print_str": (None, [_c.c_char_p, _c.c_size_t, _c.c_bool]),
    "mapal_trap": (None, [_c.c_uint32]),
    "mapal_time_ms": (_c.c_double, []),
    "mapal_render_f32": (_int, [_f32, _c.c_char_p, _c.c_size_t]),
    "mapal_render_f64": (_int, [_c.c_double, _c.c_char_p, _c.c_size_t]),
}

_lib: ctypes.CDLL | None = None


def load() -> ctypes.CDLL:
    """Load the in-tree library (raises if it has not been built)."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(
                f"{LIB_PATH} is missing: build it with `python -m flow_b200.build` "
                "(libmapal_gpu has no CPU fallback)")
        lib = ctypes.CDLL(LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        _lib = lib
    return _lib
