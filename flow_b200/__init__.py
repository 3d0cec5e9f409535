"""flow_b200 — Python host side of libmapal_gpu, the B200 (sm_100a) runtime
for Mapal's bulk array sites.

The reference's boundary for this path is its CUDA backend: `emit(ir)` turns
each recognized bulk site of a sealed CategoryIr into a kernel plus launch
glue (crates/backends/cuda/src/lib.rs:72-111), and the emitted program
reports a trap with exit code 101 and an infrastructure failure with 102
(module.rs:61-95). Here the kernels are fixed sm_100a kernels behind a C ABI
(include/mapal_gpu.h); this package calls them with the same site records
(TileSite, MoveSite) and maps the ABI's status codes onto exceptions with the
same classes: `MapalTrap` (exit 101: div_zero / index_oob), `Unsupported`
(EmitError::Unsupported) and `MapalInfraError` (exit 102).

Buffers are caller-owned device memory; torch CUDA tensors are accepted as
plain device buffers (torch is plumbing here, never the compute path).
There is no CPU fallback: every call runs a kernel of libmapal_gpu.so.
"""
from __future__ import annotations

import ctypes
from typing import Sequence

from . import _native
from .records import (ExprOp, GpuProfile, KSplit, MoveSite, TileRead, TileSite, conv2d_site, fir_site,
                      matmul_site, program, transpose_site)

__all__ = [
    "Context", "MapalTrap", "MapalInfraError", "Unsupported", "TileSite", "TileRead", "KSplit",
    "MoveSite", "GpuProfile", "matmul_site", "fir_site", "conv2d_site", "transpose_site",
    "STRICT", "TF32X3", "U11", "U01", "OP_ADD", "OP_SUB", "OP_MUL", "OP_DIV", "OP_MOD",
    "shard_range", "render_f32", "render_f64", "lib",
]

STRICT, TF32X3 = 0, 1
U11, U01 = 0, 1
OP_ADD, OP_SUB, OP_MUL, OP_DIV, OP_MOD = range(5)

OK, TRAP_DIV_ZERO, TRAP_INDEX_OOB = 0, 1, 2
ERR_INVALID, ERR_UNSUPPORTED, ERR_CUDA, ERR_NCCL, ERR_NOMEM, ERR_TIMEOUT = -1, -2, -3, -4, -5, -6


class MapalInfraError(RuntimeError):
    """An infrastructure failure: the reference's exit-102 class (module.rs:66-71)."""
    exit_code = 102

    def __init__(self, status: int, message: str):
        super().__init__(f"[status {status}] {message}")
        self.status = status


class Unsupported(MapalInfraError):
    """A site record this library has no kernel for (EmitError::Unsupported)."""


class MapalTrap(Exception):
    """A defined trap: the reference's exit-101 class (mapal_trap, mapal-rt/src/lib.rs:71-81)."""
    exit_code = 101

    def __init__(self, kind: str):
        super().__init__(f"mapal trap: {kind}")
        self.kind = kind


def lib() -> ctypes.CDLL:
    return _native.load()


def _check(rc: int) -> int:
    if rc == OK:
        return rc
    if rc == TRAP_DIV_ZERO:
        raise MapalTrap("div_zero")
    if rc == TRAP_INDEX_OOB:
        raise MapalTrap("index_oob")
    msg = (lib().mapal_gpu_last_error() or b"").decode(errors="replace")
    if rc == ERR_UNSUPPORTED:
        raise Unsupported(rc, msg)
    raise MapalInfraError(rc, msg)


def _ptr(t) -> int:
    """Address of a buffer: a torch tensor, a numpy array (host), an int address, or None."""
    if t is None:
        return 0
    if isinstance(t, int):
        return t
    if hasattr(t, "data_ptr"):
        return t.data_ptr()
    return t.ctypes.data


def _arr(ptrs: Sequence) -> ctypes.Array:
    return (ctypes.c_void_p * len(ptrs))(*[_ptr(p) for p in ptrs])


def _u64s(vals: Sequence[int]) -> ctypes.Array:
    return (ctypes.c_uint64 * len(vals))(*vals)


def shard_range(n: int, nranks: int, r: int) -> tuple[int, int]:
    """[lo, hi) of n units owned by rank r: contiguous, equal up to one unit."""
    lo, hi = ctypes.c_uint64(), ctypes.c_uint64()
    _check(lib().mapal_gpu_shard_range(n, nranks, r, ctypes.byref(lo), ctypes.byref(hi)))
    return lo.value, hi.value


def render_f32(v: float) -> str:
    """Rust `Display` of an f32 (what mapal_print_f32 writes)."""
    buf = ctypes.create_string_buffer(64)
    n = lib().mapal_render_f32(v, buf, 64)
    if n < 0:
        raise MapalInfraError(ERR_INVALID, "render failed")
    return buf.value.decode()


def render_f64(v: float) -> str:
    buf = ctypes.create_string_buffer(400)
    n = lib().mapal_render_f64(v, buf, 400)
    if n < 0:
        raise MapalInfraError(ERR_INVALID, "render failed")
    return buf.value.decode()


def launch_count() -> int:
    """Kernel launches libmapal_gpu has issued in this process so far."""
    return int(lib().mapal_gpu_launch_count())


def nccl_unique_id() -> bytes:
    buf = ctypes.create_string_buffer(128)
    _check(lib().mapal_gpu_nccl_unique_id(buf))
    return buf.raw


class Context:
    """A libmapal_gpu context: streams, trap flags, scratch and (for more than
    one device) NCCL communicators.

    Context(devices=(0,))                       one process, these devices
    Context(devices=(d,), rank=r, nranks=n, nccl_id=id)
                                                one rank of a multi-process job

    With torch_stream=True the library enqueues on torch's current stream of
    each device, so its kernels are ordered with torch work on the same stream.
    """

    def __init__(self, devices: Sequence[int] = (0,), *, rank: int | None = None,
                 nranks: int | None = None, nccl_id: bytes | None = None,
                 torch_stream: bool = True, sync: bool = True):
        L = lib()
        self._h = ctypes.c_void_p()
        self.devices = list(devices)
        if rank is None:
            mask = 0
            for d in self.devices:
                mask |= 1 << d
            _check(L.mapal_gpu_ctx_create(mask, ctypes.byref(self._h)))
        else:
            if len(self.devices) != 1:
                raise ValueError("a rank context drives exactly one device")
            _check(L.mapal_gpu_ctx_create_rank(self.devices[0], nranks, rank, nccl_id,
                                               ctypes.byref(self._h)))
        if torch_stream:
            import torch
            for i, d in enumerate(self.devices):
                s = torch.cuda.current_stream(d)
                _check(L.mapal_gpu_set_stream(self._h, i, ctypes.c_void_p(s.cuda_stream)))
        self.set_sync(sync)

    # ---- lifecycle -------------------------------------------------------------
    def close(self) -> None:
        if self._h:
            lib().mapal_gpu_ctx_destroy(self._h)
            self._h = ctypes.c_void_p()

    def __enter__(self) -> "Context":
        return self

    def __exit__(self, *exc) -> None:
        self.close()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    @property
    def handle(self) -> ctypes.c_void_p:
        return self._h

    def profile(self, local: int = 0) -> GpuProfile:
        p = GpuProfile()
        _check(lib().mapal_gpu_profile(self._h, local, ctypes.byref(p)))
        return p

    def world(self) -> tuple[int, int]:
        n, r = ctypes.c_int(), ctypes.c_int()
        _check(lib().mapal_gpu_ctx_world(self._h, ctypes.byref(n), ctypes.byref(r)))
        return n.value, r.value

    def sum_combine(self) -> int:
        """1: sharded sums combine over peer memory; -1: NCCL all-reduce; 0: not yet decided."""
        m = ctypes.c_int()
        _check(lib().mapal_gpu_ctx_sum_combine(self._h, ctypes.byref(m)))
        return m.value

    def stream(self, local: int = 0) -> int:
        s = ctypes.c_void_p()
        _check(lib().mapal_gpu_get_stream(self._h, local, ctypes.byref(s)))
        return s.value or 0

    def set_stream(self, stream: int | None, local: int = 0) -> None:
        _check(lib().mapal_gpu_set_stream(self._h, local, ctypes.c_void_p(stream or 0)))

    def set_sync(self, sync: bool) -> None:
        _check(lib().mapal_gpu_set_sync(self._h, 1 if sync else 0))

    def synchronize(self) -> None:
        _check(lib().mapal_gpu_synchronize(self._h))

    # ---- generators --------------------------------------------------------------
    def iota(self, out) -> None:
        _check(lib().mapal_gpu_iota_i32(self._h, _ptr(out), out.numel()))

    def fill(self, out, v: float) -> None:
        _check(lib().mapal_gpu_fill_f32(self._h, _ptr(out), v, out.numel()))

    def widen(self, inp, out) -> None:
        _check(lib().mapal_gpu_widen_i32_f32(self._h, _ptr(inp), _ptr(out), out.numel()))

    def gen_affine(self, out, mul: int, add: int, mod: int, sub: int, start: int = 0) -> None:
        _check(lib().mapal_gpu_gen_affine_f32(self._h, _ptr(out), out.numel(), start, mul, add, mod, sub))

    def gen(self, out, seed: int, offset: int = 0, kind: int = U11) -> None:
        _check(lib().mapal_gpu_gen_f32(self._h, _ptr(out), out.numel(), seed, offset, kind))

    def gen_index(self, out, seed: int, offset: int, rng: int) -> None:
        _check(lib().mapal_gpu_gen_index_i32(self._h, _ptr(out), out.numel(), seed, offset, rng))

    # ---- sites ----------------------------------------------------------------------
    def saxpy(self, a: float, x, y0, out) -> None:
        _check(lib().mapal_gpu_map_saxpy(self._h, a, _ptr(x), _ptr(y0), _ptr(out), out.numel()))

    def zip_map(self, op: int, x, y, out) -> None:
        _check(lib().mapal_gpu_zip_map_f32(self._h, op, _ptr(x), _ptr(y), _ptr(out), out.numel()))

    def map_expr(self, prog, arrays, out, n: int | None = None) -> None:
        """out[t] = prog evaluated at element t (see records.program)."""
        n = out.numel() if n is None else n
        lens = _u64s([a.numel() for a in arrays]) if arrays else None
        _check(lib().mapal_gpu_map_expr(self._h, prog, len(prog), _arr(arrays) if arrays else None, lens,
                                        len(arrays), _ptr(out), n))

    def transpose(self, site: MoveSite, inp, out) -> None:
        _check(lib().mapal_gpu_transpose(self._h, ctypes.byref(site), _ptr(inp), _ptr(out)))

    def gather(self, x, idx, out) -> None:
        _check(lib().mapal_gpu_gather(self._h, _ptr(x), x.numel(), _ptr(idx), _ptr(out), out.numel()))

    def fold_sum(self, x, out, seed: float = 0.0) -> None:
        """out (one device float) = seed + sum(x), tree order, f64 accumulation."""
        _check(lib().mapal_gpu_fold_sum_f32(self._h, seed, _ptr(x), x.numel(), _ptr(out)))

    def fold_sum_i32(self, x, out, seed: int = 0) -> None:
        """out (one device int32) = seed + sum(x) with wrapping i32 arithmetic (exact in any order)."""
        _check(lib().mapal_gpu_fold_sum_i32(self._h, seed, _ptr(x), x.numel(), _ptr(out)))

    def fold_sum_strict(self, x, out, seed: float = 0.0) -> None:
        """out (one device float) = the interpreter's left fold of x from seed, bit-exact."""
        _check(lib().mapal_gpu_fold_sum_f32_strict(self._h, seed, _ptr(x), x.numel(), _ptr(out)))

    def fir(self, site: TileSite, w, x, out) -> None:
        _check(lib().mapal_gpu_fir_f32(self._h, ctypes.byref(site), _ptr(w), _ptr(x), _ptr(out)))

    def conv2d_3x3(self, site: TileSite, w, img, out) -> None:
        _check(lib().mapal_gpu_conv2d_3x3_f32(self._h, ctypes.byref(site), _ptr(w), _ptr(img), _ptr(out)))

    def matmul(self, site: TileSite, A, B, C, mode: int = STRICT) -> None:
        _check(lib().mapal_gpu_matmul_f32(self._h, ctypes.byref(site), _ptr(A), _ptr(B), _ptr(C), mode))

    def matmul_host(self, site: TileSite, A, B, C, mode: int = STRICT) -> None:
        """The matmul site on HOST buffers (torch CPU tensors, pinned for overlap, or
        numpy arrays): copies in, multiply and copy out overlap in row blocks."""
        _check(lib().mapal_gpu_matmul_f32_host(self._h, ctypes.byref(site), _ptr(A), _ptr(B), _ptr(C), mode))

    def matmul_host_sharded(self, site: TileSite, As, Bs, Cs, rows: Sequence[int], mode: int = STRICT) -> None:
        """The host-array matmul over the context's ranks: As[d] / Cs[d] are the local
        device's row blocks in host memory, Bs[d] a host copy of the whole B."""
        _check(lib().mapal_gpu_matmul_f32_host_sharded(self._h, ctypes.byref(site), _arr(As), _arr(Bs), _arr(Cs),
                                                       _u64s(rows), mode))

    def tile_site(self, site: TileSite, a, b, out, mode: int = STRICT) -> None:
        _check(lib().mapal_gpu_tile_site_f32(self._h, ctypes.byref(site), _ptr(a), _ptr(b), _ptr(out), mode))

    # ---- sharded sites (one buffer per local device) --------------------------------
    def saxpy_sharded(self, a: float, xs, y0s, outs) -> None:
        n = _u64s([o.numel() for o in outs])
        _check(lib().mapal_gpu_saxpy_sharded(self._h, a, _arr(xs), _arr(y0s), _arr(outs), n))

    def fold_sum_sharded(self, xs, outs, seed: float = 0.0) -> None:
        n = _u64s([x.numel() for x in xs])
        _check(lib().mapal_gpu_fold_sum_f32_sharded(self._h, seed, _arr(xs), n, _arr(outs)))

    def broadcast(self, bufs, root: int = 0) -> None:
        _check(lib().mapal_gpu_broadcast_f32(self._h, _arr(bufs), bufs[0].numel(), root))

    def gather_sharded(self, xs, idxs, outs) -> None:
        n = _u64s([o.numel() for o in outs])
        _check(lib().mapal_gpu_gather_sharded(self._h, _arr(xs), xs[0].numel(), _arr(idxs), _arr(outs), n))

    def probe_mma_peak(self, kind: int = 0, iters: int = 4096) -> float:
        """Measured tensor-pipe rate in TFLOP/s of the 3xTF32 GEMM's MMA shape
        (kind 0: tf32; kind 1: the bf16 form of the same shape), operands
        resident in shared memory, one CTA per SM."""
        out = ctypes.c_double()
        _check(lib().mapal_gpu_probe_mma_peak(self._h, kind, iters, ctypes.byref(out)))
        return out.value

    def probe_launch_floor(self, kind: int, x=None, sink=None) -> None:
        """Enqueue the floor kernel: kind 0 an empty kernel, kind 1 a read of
        x with the sum fold's grid and loads but no combine."""
        n = x.numel() if x is not None else 0
        _check(lib().mapal_gpu_probe_launch_floor(self._h, kind, _ptr(x) if x is not None else None, n,
                                                  _ptr(sink) if sink is not None else None))

    def matmul_sharded(self, site: TileSite, As, Bs, Cs, rows: Sequence[int], root: int = 0,
                       mode: int = STRICT) -> None:
        _check(lib().mapal_gpu_matmul_f32_sharded(self._h, ctypes.byref(site), _arr(As), _arr(Bs),
                                                  _arr(Cs), _u64s(rows), root, mode))


def device_count() -> int:
    n = ctypes.c_int()
    _check(lib().mapal_gpu_device_count(ctypes.byref(n)))
    return n.value
