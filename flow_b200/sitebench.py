"""Micro-benchmark of one site class on one GPU (also the driver for ncu captures).

    python -m flow_b200.sitebench --site saxpy --n 1048576
    python -m flow_b200.sitebench --site matmul --n 4096 [--rows 512] [--mode tf32x3] --reps 3

Inputs are generated on the device from the seeded stream. Every launch
reads data that is not in L2: the inputs are replicated into as many buffer
sets as it takes to exceed twice the L2 size and the launches rotate through
them, between two CUDA events. The launches are timed twice: issued one by
one from Python (`ms_host_issued`; for sites of a few microseconds that is
the host's call rate) and captured into a CUDA graph and replayed (`ms`: the
GPU runs them back to back, as in a pipeline of sites). Sites whose inputs
exceed the L2 on their own use one set. Prints one JSON object per site.
"""
from __future__ import annotations

import argparse
import json
import math

import flow_b200 as fb

SITES = ("saxpy", "transpose", "gather", "sum", "sum_strict", "fir", "conv2d", "matmul", "map_expr", "tile_generic",
         "gen", "floor_empty", "floor_read", "floor_random")


def _alloc(torch, n, dtype=None):
    return torch.empty(n, dtype=dtype or torch.float32, device="cuda")


def make_site(ctx, torch, name: str, n: int, k: int | None = None, mode: int = fb.STRICT,
              rows: int | None = None):
    """Return (launch(set_index), bytes_per_launch, flops_per_launch, nsets_fn, extra)."""
    sets = []
    if name == "saxpy":
        def mk(i):
            x, y0, y = _alloc(torch, n), _alloc(torch, n), _alloc(torch, n)
            ctx.gen(x, 1, 0)
            ctx.gen(y0, 1, n)
            return (x, y0, y)
        per = 12 * n
        run = lambda s: ctx.saxpy(2.5, s[0], s[1], s[2])
        flops = 2 * n
    elif name == "transpose":
        side = int(math.isqrt(n))
        site = fb.transpose_site(side, side)

        def mk(i):
            a, b = _alloc(torch, side * side), _alloc(torch, side * side)
            ctx.gen(a, 1, 0)
            return (a, b)
        per = 8 * side * side
        run = lambda s: ctx.transpose(site, s[0], s[1])
        flops = 0
    elif name == "gather":
        def mk(i):
            x, idx, y = _alloc(torch, n), _alloc(torch, n, torch.int32), _alloc(torch, n)
            ctx.gen(x, 1, 0)
            ctx.gen_index(idx, 1, n, n)
            return (x, idx, y)
        per = 12 * n
        run = lambda s: ctx.gather(s[0], s[1], s[2])
        flops = 0
    elif name == "sum":
        def mk(i):
            x, out = _alloc(torch, n), _alloc(torch, 1)
            ctx.gen(x, 1, 0, fb.U01)
            return (x, out)
        per = 4 * n
        run = lambda s: ctx.fold_sum(s[0], s[1])
        flops = n
    elif name == "fir":
        taps = k or 64
        n_out = n - taps + 1
        site = fb.fir_site(n_out, taps)

        def mk(i):
            x, w, y = _alloc(torch, n), _alloc(torch, taps), _alloc(torch, n_out)
            ctx.gen(x, 1, 0)
            ctx.gen(w, 1, n)
            return (x, w, y)
        per = 4 * n + 4 * n_out + 4 * taps
        run = lambda s: ctx.fir(site, s[1], s[0], s[2])
        flops = 2 * taps * n_out
    elif name == "conv2d":
        side = int(math.isqrt(n))
        site = fb.conv2d_site(side - 2, side - 2, side, side * side)

        def mk(i):
            img, w, out = _alloc(torch, side * side), _alloc(torch, 9), _alloc(torch, (side - 2) ** 2)
            ctx.gen(img, 1, 0)
            ctx.gen(w, 1, side * side)
            return (img, w, out)
        per = 4 * side * side + 4 * (side - 2) ** 2 + 36
        run = lambda s: ctx.conv2d_3x3(site, s[1], s[0], s[2])
        flops = 18 * (side - 2) ** 2
    elif name == "matmul":
        # rows: an M x n block of the n x n site (one rank's row block of a
        # row-sharded site); default the whole site
        kk = k or n
        m = rows or n
        site = fb.matmul_site(m, n, kk)

        def mk(i):
            A, B, C = _alloc(torch, m * kk), _alloc(torch, kk * n), _alloc(torch, m * n)
            ctx.gen(A, 2, 0)
            ctx.gen(B, 2, m * kk)
            return (A, B, C)
        per = 4 * (m * kk + kk * n + m * n)
        run = lambda s: ctx.matmul(site, s[0], s[1], s[2], mode)
        flops = 2 * m * n * kk
    elif name == "map_expr":
        # the benches' generator body as a general map program:
        # t -> (t * 7 + 13) % 101 - 50 -> widen_f32
        from .records import program
        prog = program(("T_I32",), ("CONST_I32", 7), ("MUL_I32",), ("CONST_I32", 13), ("ADD_I32",),
                       ("CONST_I32", 101), ("REM_I32",), ("CONST_I32", 50), ("SUB_I32",), ("WIDEN_I32_F32",),
                       ("STORE_F32",))

        def mk(i):
            return (_alloc(torch, n),)
        per = 4 * n
        run = lambda s: ctx.map_expr(prog, [], s[0], n)
        flops = 0
    elif name == "sum_strict":
        # the interpreter-order fold (one dependent chain of f32 adds)
        def mk(i):
            x, out = _alloc(torch, n), _alloc(torch, 1)
            ctx.gen(x, 1, 0, fb.U01)
            return (x, out)
        per = 4 * n
        run = lambda s: ctx.fold_sum_strict(s[0], s[1])
        flops = n
    elif name == "tile_generic":
        # a TileSite no specialised kernel takes: C = A * B^T read in place
        # (b{ck=1, clane=K}), side x side x k, the rung-0 shape kernel
        from .records import TileSite
        side = int(math.isqrt(n))
        kk = k or 64
        site = TileSite()
        site.rows, site.c, site.k = side, side, kk
        site.a.ci, site.a.ck, site.a.len = kk, 1, side * kk
        site.b.ck, site.b.clane, site.b.len = 1, kk, side * kk
        site.mul_a_first, site.add_acc_first = 1, 1

        def mk(i):
            A, B, C = _alloc(torch, side * kk), _alloc(torch, side * kk), _alloc(torch, side * side)
            ctx.gen(A, 2, 0)
            ctx.gen(B, 2, side * kk)
            return (A, B, C)
        per = 4 * (2 * side * kk + side * side)
        run = lambda s: ctx.tile_site(site, s[0], s[1], s[2])
        flops = 2 * side * side * kk
    elif name == "gen":
        # the seeded uniform stream written to n floats
        def mk(i):
            return (_alloc(torch, n),)
        per = 4 * n
        run = lambda s: ctx.gen(s[0], 1, 0)
        flops = 0
    elif name == "floor_random":
        # n independent random 4-byte reads of x (the gather's bound)
        def mk(i):
            x, sink = _alloc(torch, n), _alloc(torch, 1)
            ctx.gen(x, 1, 0)
            return (x, sink)
        per = 4 * n
        run = lambda s: ctx.probe_launch_floor(2, s[0], s[1])
        flops = 0
    elif name == "floor_empty":
        # the launch floor: an empty kernel
        def mk(i):
            return ()
        per = 0
        run = lambda s: ctx.probe_launch_floor(0)
        flops = 0
    elif name == "floor_read":
        # the read floor: the sum fold's grid and loads over n floats, no combine
        def mk(i):
            x, sink = _alloc(torch, n), _alloc(torch, 1)
            ctx.gen(x, 1, 0, fb.U01)
            return (x, sink)
        per = 4 * n
        run = lambda s: ctx.probe_launch_floor(1, s[0], s[1])
        flops = 0
    else:
        raise ValueError(f"unknown site {name}")
    return mk, run, per, flops


def measure(ctx, torch, name: str, n: int, k: int | None = None, reps: int = 20, warmup: int = 3,
            mode: int = fb.STRICT, l2_bytes: int = 126 << 20, rotate: bool = True,
            graph: bool = True, rows: int | None = None) -> dict:
    mk, run, per, flops = make_site(ctx, torch, name, n, k, mode, rows)
    nsets = max(1, math.ceil(2 * l2_bytes / per)) if rotate and per else 1
    sets = [mk(i) for i in range(nsets)]
    ctx.synchronize()
    stream = torch.cuda.current_stream()
    for i in range(warmup):
        run(sets[i % nsets])
    ctx.synchronize()
    total = max(reps, nsets)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    # Host-issued: one library call per launch from Python. For sites of a few
    # microseconds the GPU then waits on the host between launches.
    e0.record(stream)
    for i in range(total):
        run(sets[i % nsets])
    e1.record(stream)
    ctx.synchronize()
    torch.cuda.synchronize()
    ms_host = e0.elapsed_time(e1) / total
    ms = ms_host
    if graph:
        # The same launches captured once into a CUDA graph and replayed: the
        # GPU sees them back to back, as from a program that issues sites
        # faster than they run.
        cap = torch.cuda.Stream()
        cap.wait_stream(stream)
        ctx.set_stream(cap.cuda_stream)
        g = torch.cuda.CUDAGraph()
        try:
            with torch.cuda.graph(g, stream=cap):
                for i in range(total):
                    run(sets[i % nsets])
        finally:
            ctx.set_stream(stream.cuda_stream)
        g.replay()
        torch.cuda.synchronize()
        e0.record(stream)
        g.replay()
        e1.record(stream)
        torch.cuda.synchronize()
        ms = e0.elapsed_time(e1) / total
        del g
    out = {"site": name, "n": n, **({"rows": rows} if rows else {}), "ms": ms, "bytes": per, "gbs": per / (ms * 1e-3) / 1e9 if per else None,
           "launches": total, "buffer_sets": nsets, "ms_host_issued": ms_host,
           "timing": "CUDA graph replay of the launches" if graph else "host-issued launches"}
    if flops:
        out["gflops"] = flops / (ms * 1e-3) / 1e9
    return out


def main() -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--site", choices=SITES + ("all",), default="all")
    ap.add_argument("--n", type=int, default=None, help="elements (side^2 for transpose/conv2d, side for matmul)")
    ap.add_argument("--k", type=int, default=None, help="taps (fir) or K (matmul)")
    ap.add_argument("--rows", type=int, default=None, help="matmul: rows of the block (default n)")
    ap.add_argument("--reps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--mode", choices=["strict", "tf32x3"], default="strict")
    ap.add_argument("--no-rotate", action="store_true")
    ap.add_argument("--no-graph", action="store_true", help="time host-issued launches only")
    args = ap.parse_args()
    import torch
    defaults = {"saxpy": 1 << 20, "transpose": 1024 * 1024, "gather": 1 << 20, "sum": 1 << 20,
                "fir": 1 << 20, "conv2d": 1024 * 1024, "matmul": 4096, "map_expr": 1 << 20, "floor_empty": 1,
                "floor_read": 1 << 20, "sum_strict": 1 << 20, "tile_generic": 1024 * 1024, "gen": 1 << 26,
                "floor_random": 1 << 26}
    sites = SITES if args.site == "all" else (args.site,)
    with fb.Context((0,), sync=False) as ctx:
        l2 = ctx.profile().l2_bytes
        mode = fb.TF32X3 if args.mode == "tf32x3" else fb.STRICT
        for s in sites:
            n = args.n or defaults[s]
            r = measure(ctx, torch, s, n, args.k, args.reps, args.warmup, mode, l2, not args.no_rotate,
                        not args.no_graph, args.rows if s == "matmul" else None)
            print(json.dumps(r), flush=True)
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
