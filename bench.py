#!/usr/bin/env python
"""bench.py — f32 matmul 4096^2 TFLOP/s (+ streaming-kernel HBM GB/s) on 1..8 B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--mode strict|tf32x3]
    python bench.py --impl reference ...     the reference's own CPU leg
    torchrun --nproc-per-node N bench.py --gpus N ...

One step = one pass of the matmul site C = A*B, M=N=K=4096, over resident
A, B drawn uniform[-1,1) from seed 2 (the seeded i32-hash stream, generated
on the device). With N GPUs the site is row-sharded: rank r owns rows
[lo, hi) of A and C, B is replicated by an NCCL broadcast from rank 0 inside
every step, so the total work is fixed (strong scaling). Time is taken with
CUDA events on the launching stream, max over ranks; L2 is flushed (a
256 MiB write) between timed steps. Rank 0 prints one JSON line.

The streaming suite (saxpy, transpose, gather, sum, FIR, conv2d at 2^20
scale, L2 flushed before every launch; and saxpy / sum / gather at 2^30,
2^30, 2^28 sharded over the ranks) is reported under "streaming".
"""
from __future__ import annotations

import argparse
import csv
import io
import json
import os
import re
import shutil
import statistics
import subprocess
import sys
import tempfile
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "f32 matmul 4096² TFLOP/s + streaming-kernel HBM GB/s at 1/2/4/8 B200"
N_MM = 4096
SEED_MM = 2
# The reference's published number for this metric: its rung-0 CUDA kernel,
# N=4096 f32, FMA off (bit-exact face), 57.2 ms on an RTX 4090.
PUBLISHED_REF_TFLOPS = 2.40
HBM_FALLBACK_GBS = 6650.0


# stdout carries exactly one JSON line: everything else any library writes to
# fd 1 (NCCL's version banner, for one) is sent to stderr, and the line goes
# to the original stdout.
_JSON_OUT = None


def quiet_stdout() -> None:
    global _JSON_OUT
    sys.stdout.flush()
    _JSON_OUT = os.fdopen(os.dup(1), "w")
    os.dup2(2, 1)


def emit_line(line: dict) -> None:
    out = _JSON_OUT or sys.stdout
    out.write(json.dumps(line) + "\n")
    out.flush()


def env_int(name: str, default: int) -> int:
    try:
        return int(os.environ.get(name, default))
    except ValueError:
        return default


def peaks() -> dict:
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return {"hbm_gbs": float(p["hbm_gbs"]), "sm_max_mhz": float(p.get("sm_max_mhz", 1965.0)),
                "bf16_tflops": float(p.get("bf16_tflops", 1590.0)), "source": "measured"}
    except Exception:
        return {"hbm_gbs": HBM_FALLBACK_GBS, "sm_max_mhz": 1965.0, "bf16_tflops": 1590.0,
                "source": "fallback"}


def host_cores() -> int:
    n = os.cpu_count() or 1
    try:
        q, per = open("/sys/fs/cgroup/cpu.max").read().split()
        if q != "max":
            n = min(n, max(1, -(-int(q) // int(per))))
    except Exception:
        pass
    return n


def smi_device(local: int) -> str:
    """nvidia-smi's name for CUDA device `local` (index or UUID)."""
    vis = os.environ.get("CUDA_VISIBLE_DEVICES")
    if vis:
        items = [v.strip() for v in vis.split(",") if v.strip()]
        if local < len(items):
            return items[local]
    return str(local)


# ---- clock sampling ----------------------------------------------------------------------

class Clocks:
    """nvidia-smi sampling every 200 ms while the timed region runs."""
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device: int):
        self.device = device
        self.proc = None
        self.path = None

    def start(self):
        if not shutil.which("nvidia-smi"):
            return
        fd, self.path = tempfile.mkstemp(suffix=".csv")
        os.close(fd)
        self.proc = subprocess.Popen(
            ["nvidia-smi", "-i", str(self.device), f"--query-gpu={self.FIELDS}", "--format=csv,noheader",
             "-lms", "200"], stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)

    def stop(self) -> dict | None:
        if not self.proc:
            return None
        time.sleep(0.25)
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        rows = list(csv.reader(io.StringIO(open(self.path).read())))
        os.unlink(self.path)
        sm, mx, reasons, power = [], 0.0, set(), []
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for r in rows:
            if len(r) < 9:
                continue
            try:
                sm.append(float(r[1].split()[0]))
                mx = max(mx, float(r[2].split()[0]))
                power.append(float(r[3].split()[0]))
            except ValueError:
                continue
            for name, v in zip(names, r[5:9]):
                if v.strip() == "Active":
                    reasons.add(name)
        if not sm:
            return None
        loaded = [s for s, p in zip(sm, power) if p > 250.0] or sm
        return {"sm_mhz": statistics.median(loaded), "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm), "power_w_max": max(power) if power else None}


# ---- the reference's CPU leg -----------------------------------------------------------------

def cpp_mt_path() -> str:
    return os.path.join(ROOT, "oracle", "_ref", "cpp_mt")


def run_cpp_mt(n: int, iters: int, threads: int, timeout: float = 300.0) -> dict:
    """Time benches/matmul/cpp_mt.cpp (the reference's threaded C++ matmul leg,
    compiled unmodified by oracle/Makefile) on this host's cores."""
    env = dict(os.environ, THREADS=str(threads))
    out = subprocess.run([cpp_mt_path(), str(n), str(iters), "f32"], capture_output=True, text=True,
                         env=env, timeout=timeout, check=True).stdout
    m = re.search(r"N=(\d+) ([\d.]+) ms ([\d.]+) GFLOP/s c0=(-?[\d.]+) clast=(-?[\d.]+) T=(\d+)", out)
    if not m:
        raise RuntimeError(f"unexpected cpp_mt output: {out!r}")
    ms = float(m.group(2))
    return {"ms": ms, "tflops": 2.0 * n ** 3 / (ms * 1e-3) / 1e12, "threads": int(m.group(6)),
            "c0": float(m.group(4)), "clast": float(m.group(5))}


def cpu_baseline(n: int = N_MM, iters: int = 1) -> dict:
    """The reference's threaded C++ matmul leg at size n on all host cores
    (one pass of the 4096^2 workload: 30-60 s on a 16-32 core host); the
    oracle port on a slice of rows if the reference leg was not built."""
    cores = host_cores()
    if os.path.exists(cpp_mt_path()):
        r = run_cpp_mt(n, iters, cores)
        return {"value": r["tflops"], "unit": "TFLOP/s", "cores": r["threads"], "kind": "reference",
                "sample": f"benches/matmul/cpp_mt.cpp f32 N={n}, {iters} iteration(s), min over "
                          f"iterations, integer-generator inputs (timing is data-independent)",
                "ms": r["ms"]}
    import numpy as np
    import oracle
    rows = 64
    A = oracle.gen(N_MM * N_MM, SEED_MM, 0)
    B = oracle.gen(N_MM * N_MM, SEED_MM, N_MM * N_MM)
    t0 = time.perf_counter()
    oracle.matmul(A, B, N_MM, N_MM, N_MM, 0, rows, threads=cores)
    dt = time.perf_counter() - t0
    return {"value": 2.0 * rows * N_MM * N_MM / dt / 1e12, "unit": "TFLOP/s", "cores": cores, "kind": "port",
            "sample": f"oracle strict matmul, {rows} of 4096 rows"}


def reference_arm(args) -> int:
    rank = env_int("RANK", 0)
    if rank != 0:
        return 0
    # One pass of the full 4096^2 workload (about a minute on 16 cores): the
    # reference's harness itself reports min over its iterations.
    iters = 1
    cb = cpu_baseline(N_MM, iters)
    line = {
        "impl": "reference", "metric": METRIC, "value": cb["value"], "unit": "TFLOP/s",
        "n_gpus": args.gpus, "steps": iters, "warmup": 0, "ms_per_step": cb.get("ms"),
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic", "config": {"workload": "f32 matmul M=N=K=4096 (reference C++ CPU leg)"},
        "cpu_baseline": cb, "e2e": {"value": cb["value"], "unit": "TFLOP/s", "h2d_bytes_per_step": 0,
                                    "d2h_bytes_per_step": 0},
    }
    emit_line(line)
    return 0



def ref_leg_path(name: str) -> str:
    return os.path.join(ROOT, "oracle", "_ref", name)


def streaming_cpu_legs(cores: int) -> dict:
    """The reference's own threaded C++ legs for the streaming suite
    (benches/shapes/ladder2_baseline.cpp: saxpy, reduce, transpose, gather;
    benches/shapes/shapes_baseline.cpp: FIR, conv2d), compiled unmodified into
    oracle/_ref/ and run as benches/shapes/shapes_ab.sh runs them: `mt` with
    THREADS = all host cores, the best of 20 iterations, data generation
    outside their timer. Sizes are the streaming configs: 2^20 elements,
    1024^2 transpose, 64-tap FIR over 2^20 samples (2^20 - 63 outputs), and
    conv2d on a 1024^2 image (side 1022 outputs)."""
    legs = [("saxpy_2^20", "ladder2_baseline", ["saxpy"], 1 << 20, 12 * (1 << 20)),
            ("transpose_1024^2", "ladder2_baseline", ["transpose"], 1024, 8 * 1024 * 1024),
            ("gather_2^20", "ladder2_baseline", ["gather"], 1 << 20, 12 * (1 << 20)),
            ("sum_2^20", "ladder2_baseline", ["reduce"], 1 << 20, 4 * (1 << 20)),
            ("fir_2^20x64", "shapes_baseline", ["fir"], (1 << 20) - 63, 4 * ((1 << 20) + (1 << 20) - 63)),
            ("conv2d_1024^2_3x3", "shapes_baseline", ["conv2d"], 1022, 4 * (1024 * 1024 + 1022 * 1022))]
    out = {}
    env = dict(os.environ, THREADS=str(cores))
    for key, binary, shape, size, nbytes in legs:
        path = ref_leg_path(binary)
        if not os.path.exists(path):
            out[key] = {"error": f"{binary} not built"}
            continue
        try:
            r = subprocess.run([path, shape[0], "mt", "20", str(size)], capture_output=True, text=True,
                               env=env, timeout=120, check=True).stdout
            ms = min(float(v) for v in re.findall(r"iter ms=([\d.]+)", r))
            out[key] = {"value": nbytes / (ms * 1e-3) / 1e9, "unit": "GB/s", "ms": ms, "cores": cores,
                        "kind": "reference",
                        "sample": f"benches/shapes/{binary}.cpp {shape[0]} mt, size {size}, best of 20"}
        except Exception as e:  # the bench line stands without it
            out[key] = {"error": str(e)[:200]}
    return out


def strict_rows_check(torch, A, B, C, m: int, n: int, k: int, rows, cols=None) -> bool:
    """Bit-exact check of output cells against a float32 restatement of the
    interpreter's fold for a matmul cell (crates/mapal-interp/src/eval.rs:326-359):
    acc = +0.0, then acc = acc + a[i,kk]*b[kk,j] for kk ascending, each
    product and each sum rounded to f32. numpy's float32 ufuncs round every
    operation and never contract, so the restatement is exact. Checks the
    given rows of this rank's block over every column (or over `cols`)."""
    import numpy as np
    ri = torch.tensor(rows, dtype=torch.long, device=A.device)
    a = A.view(m, k).index_select(0, ri).cpu().numpy()
    Bv = B.view(k, n)
    Cv = C.view(m, n).index_select(0, ri)
    if cols is not None:
        ci = torch.tensor(cols, dtype=torch.long, device=A.device)
        Bv = Bv.index_select(1, ci)
        Cv = Cv.index_select(1, ci)
    b = Bv.cpu().numpy()
    got = Cv.cpu().numpy()
    acc = np.zeros((len(rows), b.shape[1]), np.float32)
    tmp = np.empty_like(acc)
    for kk in range(k):
        np.multiply(a[:, kk:kk + 1], b[kk], out=tmp)
        np.add(acc, tmp, out=acc)
    return bool(np.array_equal(got.view(np.uint32), acc.view(np.uint32)))


def tf32x3_rows_error(torch, A, B, C, m: int, n: int, k: int, rows, cols=None) -> float:
    """max |C - A.B| / (||A_i|| ||B_j||) over the given cells, A.B in f64."""
    import numpy as np
    ri = torch.tensor(rows, dtype=torch.long, device=A.device)
    a = A.view(m, k).index_select(0, ri).double().cpu().numpy()
    Bv, Cv = B.view(k, n), C.view(m, n).index_select(0, ri)
    if cols is not None:
        ci = torch.tensor(cols, dtype=torch.long, device=A.device)
        Bv, Cv = Bv.index_select(1, ci), Cv.index_select(1, ci)
    b = Bv.double().cpu().numpy()
    exact = a @ b
    scale = np.sqrt((a * a).sum(1))[:, None] * np.sqrt((b * b).sum(0))[None, :]
    return float(np.max(np.abs(Cv.double().cpu().numpy() - exact) / np.maximum(scale, 1e-300)))


# ---- our arm -----------------------------------------------------------------------------------

class Dist:
    def __init__(self, n_gpus: int):
        self.world = env_int("WORLD_SIZE", 1)
        self.rank = env_int("RANK", 0)
        self.local = env_int("LOCAL_RANK", 0)
        if self.world != n_gpus and not (self.world == 1 and n_gpus == 1):
            raise SystemExit(f"--gpus {n_gpus} but WORLD_SIZE={self.world}")
        import torch
        self.torch = torch
        torch.cuda.set_device(self.local)
        self.pg = None
        if self.world > 1:
            import datetime
            import torch.distributed as dist
            dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                    device_id=torch.device("cuda", self.local))
            self.dist = dist

    def barrier(self):
        if self.world > 1:
            self.dist.barrier()

    def max(self, v: float) -> float:
        if self.world == 1:
            return v
        t = self.torch.tensor([v], dtype=self.torch.float64, device="cuda")
        self.dist.all_reduce(t, op=self.dist.ReduceOp.MAX)
        return float(t.item())

    def sum(self, v: float) -> float:
        if self.world == 1:
            return v
        t = self.torch.tensor([v], dtype=self.torch.float64, device="cuda")
        self.dist.all_reduce(t)
        return float(t.item())

    def bcast_bytes(self, b: bytes | None) -> bytes:
        if self.world == 1:
            return b
        obj = [b]
        self.dist.broadcast_object_list(obj, src=0)
        return obj[0]

    def close(self):
        if self.world > 1:
            self.dist.destroy_process_group()


def run_ours(args) -> int:
    d = Dist(args.gpus)
    torch = d.torch
    import flow_b200 as fb

    nccl_id = d.bcast_bytes(fb.nccl_unique_id() if d.rank == 0 and d.world > 1 else None)
    if d.world > 1:
        ctx = fb.Context((d.local,), rank=d.rank, nranks=d.world, nccl_id=nccl_id, sync=False)
    else:
        ctx = fb.Context((d.local,), sync=False)
    stream = torch.cuda.current_stream()
    # L2 flush by READING 256 MiB (twice the L2): the flush leaves only clean
    # lines behind, so the timed kernel never pays to write back the flush.
    flush_buf = torch.ones(64 << 20, dtype=torch.float32, device="cuda")
    flush_out = torch.empty((), dtype=torch.float32, device="cuda")

    def flush():
        torch.sum(flush_buf, dim=0, out=flush_out)

    mode = fb.TF32X3 if args.mode == "tf32x3" else fb.STRICT
    n = N_MM
    lo, hi = fb.shard_range(n, d.world, d.rank)
    m = hi - lo
    A = torch.empty(m * n, dtype=torch.float32, device="cuda")
    B = torch.empty(n * n, dtype=torch.float32, device="cuda")
    C = torch.empty(max(m, 1) * n, dtype=torch.float32, device="cuda")
    ctx.gen(A, SEED_MM, lo * n)
    if d.rank == 0:
        ctx.gen(B, SEED_MM, n * n)
    else:
        B.fill_(float("nan"))  # B arrives by broadcast inside every step
    local_site = fb.matmul_site(m, n, n)
    ctx.synchronize()

    full_site = fb.matmul_site(n, n, n)

    def step(ev0=None, ev1=None, ev2=None):
        # One pass of the site. With N ranks: mapal_gpu_matmul_f32_sharded,
        # whose B broadcast (NCCL, from rank 0) overlaps the multiply in
        # k-ranges; ev1 is then not meaningful and the kernel-only time is
        # measured separately below.
        if ev0 is not None:
            ev0.record(stream)
        if d.world > 1:
            ctx.matmul_sharded(full_site, [A], [B], [C], [m], root=0, mode=mode)
        else:
            if ev1 is not None:
                ev1.record(stream)
            ctx.matmul(local_site, A, B, C, mode)
        if ev2 is not None:
            ev2.record(stream)

    # The sampler starts before the warm-up (nvidia-smi needs a moment to
    # begin) and stops after the timed steps.
    clocks = Clocks(smi_device(d.local))
    clocks.start()
    time.sleep(1.0)
    for _ in range(args.warmup):
        flush()
        step()
    ctx.synchronize()
    torch.cuda.synchronize()

    evs = [[torch.cuda.Event(enable_timing=True) for _ in range(3)] for _ in range(args.steps)]
    d.barrier()
    torch.cuda.synchronize()
    launches0 = fb.launch_count()
    for i in range(args.steps):
        flush()
        step(*evs[i])
    ctx.synchronize()
    torch.cuda.synchronize()
    launches = fb.launch_count() - launches0  # this library's kernels in the timed region
    d.barrier()
    clk = clocks.stop()
    step_ms = [e[0].elapsed_time(e[2]) for e in evs]
    ms = d.max(sum(step_ms) / len(step_ms))
    if d.world == 1:
        kern_ms = [e[1].elapsed_time(e[2]) for e in evs]
        kms = d.max(sum(kern_ms) / len(kern_ms))
    else:
        # kernel-only: this rank's row block alone, same flush discipline
        kms = d.max(time_launches(torch, stream, lambda: ctx.matmul(local_site, A, B, C, mode), flush,
                                  max(3, min(args.steps, 10))))
    flops = 2.0 * n ** 3
    value = flops / (ms * 1e-3) / 1e12

    # Bit-exactness of this run's output, on every rank: the first, a middle
    # and the last row of the rank's block, every column, against a float32
    # restatement of the interpreter's fold (strict mode); the verdict is the
    # AND over ranks, so a multi-GPU line proves the sharded result too.
    check = None
    if mode == fb.STRICT and not args.no_check:
        ok = True
        if m > 0:
            ok = strict_rows_check(torch, A, B, C, m, n, n, sorted({0, m // 2, m - 1}))
        check = d.sum(0.0 if ok else 1.0) == 0.0

    # e2e through the public API with host buffers: the host-array entry on
    # this rank's row block, its pinned copy of B beside it. The uploads, the
    # multiply and the download of the C block overlap in k-range phases; over
    # several ranks each rank uploads only its slice of every phase's B rows
    # and the slices cross NVLink (mapal_gpu_matmul_f32_host_sharded). The
    # device result is the check.
    e2e = None
    if not args.no_e2e:
        A_h = torch.empty(m * n, dtype=torch.float32, pin_memory=True)
        B_h = torch.empty(n * n, dtype=torch.float32, pin_memory=True)
        C_h = torch.empty(max(m, 1) * n, dtype=torch.float32, pin_memory=True)
        A_h.copy_(A.cpu())
        b_full = torch.empty(n * n, dtype=torch.float32, device="cuda")
        ctx.gen(b_full, SEED_MM, n * n)  # B as rank 0 holds it (other ranks' B arrives by broadcast)
        ctx.synchronize()
        B_h.copy_(b_full.cpu())
        del b_full
        e_steps = max(2, min(args.steps, 5))

        if d.world > 1:
            def e2e_step():
                ctx.matmul_host_sharded(local_site, [A_h], [B_h], [C_h], [m], mode)
        else:
            def e2e_step():
                ctx.matmul_host(local_site, A_h, B_h, C_h, mode)

        e2e_step()
        ctx.synchronize()
        torch.cuda.synchronize()
        ev = [torch.cuda.Event(enable_timing=True) for _ in range(2)]
        d.barrier()
        ev[0].record(stream)
        for _ in range(e_steps):
            e2e_step()
        ev[1].record(stream)
        ctx.synchronize()
        torch.cuda.synchronize()
        e_ms = d.max(ev[0].elapsed_time(ev[1]) / e_steps)
        same = d.sum(0.0 if torch.equal(C_h[:m * n], C[:m * n].cpu()) else 1.0) == 0.0
        shared_b = d.world > 1 and mode == fb.STRICT and n >= 512
        b_up = n * n * 4 // d.world if shared_b else n * n * 4  # this rank's share of B (about 1/R)
        h2d = d.sum(float(m * n * 4 + b_up))
        d2h = d.sum(float(m * n * 4))
        e2e = {"value": flops / (e_ms * 1e-3) / 1e12, "unit": "TFLOP/s", "ms_per_step": e_ms,
               "h2d_bytes_per_step": int(h2d), "d2h_bytes_per_step": int(d2h), "steps": e_steps,
               "matches_device_result": bool(same),
               "path": ("pinned host A block + 1/R of B per rank -> mapal_gpu_matmul_f32_host_sharded "
                        "(B slices gathered over NVLink) -> pinned host C block" if shared_b else
                        "pinned host A, B -> mapal_gpu_matmul_f32_host -> pinned host C")}

    pk = peaks()
    sm_mhz = clk["sm_mhz"] if clk else pk["sm_max_mhz"]
    sms = ctx.profile().sm_count
    # strict: one FP32 op per lane per clock (a MAC is a rounded mul + a rounded add)
    peak_max = sms * 128 * pk["sm_max_mhz"] * 1e6 / 1e12
    per_rank_flops = 2.0 * m * n * n
    achieved = per_rank_flops / (kms * 1e-3) / 1e12 if kms > 0 else None
    traffic = None
    tpath = os.path.join(ROOT, "profiles", "traffic.json")
    if os.path.exists(tpath):
        t = json.load(open(tpath)).get("mm_strict_kernel" if mode == fb.STRICT else "mm_tf32x3")
        if t and t.get("m") == m:
            traffic = t.get("bytes")
    roofline = {
        "bound": "fp32" if mode == fb.STRICT else "tensor",
        "kernel": "mm_strict_kernel" if mode == fb.STRICT else "mm_tf32x3",
        "achieved": achieved, "unit": "TFLOP/s",
        "peak": peak_max, "frac": achieved / peak_max if achieved else None,
        "peak_basis": f"{sms} SMs x 128 FP32 lanes x {pk['sm_max_mhz']:.0f} MHz (max clock, "
                      f"MEASURED_PEAKS sm_max_mhz), 1 op per lane per clock",
        "frac_at_sampled_clock": (achieved / (sms * 128 * sm_mhz * 1e6 / 1e12)) if achieved else None,
        "frac_of_ffma_peak": achieved / (2 * peak_max) if achieved else None,
        "traffic": traffic, "per_launch_flops": per_rank_flops,
    }

    # The opt-in tensor-core mode on the same workload (one call = split pass
    # + tcgen05 GEMM), against the tensor pipe's TF32 rate divided by 3
    # products. That rate is measured here by the library's probe (the GEMM's
    # own MMA shape, operands resident in shared memory); its bf16 form is
    # reported beside the measured cuBLAS bf16 rate as a check of the method.
    tf32 = None
    if mode == fb.STRICT and not args.no_tf32:
        ctx.set_sync(False)
        tf_probe = max(ctx.probe_mma_peak(0, 8192) for _ in range(3))
        bf_probe = max(ctx.probe_mma_peak(1, 4096) for _ in range(3))
        tms = d.max(time_launches(torch, stream, lambda: ctx.matmul(local_site, A, B, C, fb.TF32X3), flush, 10))
        ctx.synchronize()
        cols = list(range(0, n, 7))
        tf_err = d.max(tf32x3_rows_error(torch, A, B, C, m, n, n, sorted({0, m // 2, m - 1}), cols)
                       if m > 0 else 0.0)
        eff = flops / (tms * 1e-3) / 1e12
        tf32 = {"value": eff, "unit": "TFLOP/s", "ms_per_step": tms,
                "roofline": {"bound": "tensor", "achieved_tensor_tflops": 3 * eff * m / n,
                             "peak": tf_probe, "unit": "TFLOP/s",
                             "frac": 3 * eff * m / n / tf_probe,
                             "peak_basis": "measured TF32 tensor-pipe rate (mapal_gpu_probe_mma_peak kind 0: "
                                           "M128 N256 K8 tcgen05.mma, operands resident in shared memory, "
                                           "one CTA per SM, best of 3); 3 TF32 products per f32 product; "
                                           "time includes the split pass",
                             "bf16_probe_tflops": bf_probe,
                             "bf16_cublas_measured_tflops": pk["bf16_tflops"],
                             "frac_of_bf16_div2": 3 * eff * m / n / (pk["bf16_tflops"] / 2.0)},
                "max_normalised_error": tf_err,
                "error_cells": "first, middle and last row of each rank's block x every 7th column, "
                               "against the f64 product",
                "tolerance": "|C - C_ref| <= 2e-6 * ||A_i|| * ||B_j|| per cell"}

    streaming = None
    if not args.no_streaming:
        streaming = run_streaming(ctx, d, fb, torch, flush, pk)

    big_mm = None
    if not args.no_16384:
        # free the 4096^2 operands first
        del A, B, C
        torch.cuda.empty_cache()
        big_mm = run_matmul_16384(ctx, d, fb, torch, pk)

    cb = None
    if d.rank == 0 and d.world == 1 and not args.no_cpu:
        try:
            cb = cpu_baseline(N_MM, 1)
        except Exception as e:  # the bench line still stands without it
            cb = {"error": str(e)[:200]}
        if streaming is not None:
            for key, leg in streaming_cpu_legs(host_cores()).items():
                if key in streaming:
                    streaming[key]["cpu_baseline"] = leg

    line = {
        "metric": METRIC, "value": value, "unit": "TFLOP/s", "n_gpus": d.world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "strong",
        "vs_baseline": value / PUBLISHED_REF_TFLOPS,
        "vs_baseline_ref": "reference rung-0 CUDA matmul N=4096 f32, 57.2 ms = 2.40 TFLOP/s on RTX 4090 "
                           "(docs/performance/matmul/s23.md:18)",
        "dtype": "f32", "data": "synthetic: A, B uniform[-1,1) from seed 2 (seeded i32-hash stream), on device",
        "config": {"workload": f"f32 matmul site M=N=K=4096, {args.mode}"
                               + (" (bit-exact with the interpreter)" if mode == fb.STRICT else ""),
                   "M": n, "N": n, "K": n, "mode": args.mode,
                   "parallelism": f"row-shard x{d.world}, B broadcast (NCCL) inside each step",
                   "l2": "flushed between timed steps (256 MiB read)"},
        "roofline": roofline, "cpu_baseline": cb, "e2e": e2e,
        "gpu_launches": launches,
        "clocks": clk, "kernel_ms_per_step": kms, "strict_row_check": check,
        "matmul_tf32x3": tf32, "streaming": streaming, "matmul_16384": big_mm,
    }
    if d.rank == 0:
        emit_line(line)
    ctx.close()
    d.close()
    return 0


def run_matmul_16384(ctx, d, fb, torch, pk) -> dict:
    """The 16384^2 row-sharded matmul (the row-sharded 16384^2 workload): A, B uniform[-1,1)
    from seed 4, A row blocks per rank, B broadcast from rank 0 inside every
    step; strict and 3xTF32, 1 warm-up + 2 timed steps each (inputs are 1 GiB
    each, far beyond L2)."""
    n = 16384
    lo, hi = fb.shard_range(n, d.world, d.rank)
    m = hi - lo
    A = torch.empty(m * n, dtype=torch.float32, device="cuda")
    B = torch.empty(n * n, dtype=torch.float32, device="cuda")
    C = torch.empty(max(m, 1) * n, dtype=torch.float32, device="cuda")
    ctx.gen(A, 4, lo * n)
    ctx.gen(B, 4, n * n)
    ctx.synchronize()
    site = fb.matmul_site(n, n, n)
    stream = torch.cuda.current_stream()
    out = {"workload": "f32 matmul M=N=K=16384, row blocks per rank, B broadcast (NCCL) in each step",
           "data": "uniform[-1,1) from seed 4"}
    sms = ctx.profile().sm_count
    tf_peak = ctx.probe_mma_peak(0, 8192)
    rows = sorted({0, m // 2, m - 1}) if m > 0 else []
    cols = list(range(3, n, 61))
    for name, mode in (("strict", fb.STRICT), ("tf32x3", fb.TF32X3)):
        def step():
            if d.world > 1:
                ctx.matmul_sharded(site, [A], [B], [C], [m], root=0, mode=mode)
            else:
                ctx.matmul(site, A, B, C, mode)
        ms = d.max(time_launches(torch, stream, step, lambda: None, 2, d))
        tf = 2.0 * n ** 3 / (ms * 1e-3) / 1e12
        r = {"ms_per_step": ms, "value": tf, "unit": "TFLOP/s", "per_gpu": tf / d.world}
        # this rank's C block is the last step's result: check it
        if mode == fb.STRICT:
            ok = strict_rows_check(torch, A, B, C, m, n, n, rows, cols) if m > 0 else True
            r["row_check"] = d.sum(0.0 if ok else 1.0) == 0.0
            r["row_check_cells"] = "first, middle and last row of each rank's block x every 61st column, bit-exact"
        else:
            r["max_normalised_error"] = d.max(tf32x3_rows_error(torch, A, B, C, m, n, n, rows, cols)
                                              if m > 0 else 0.0)
        if d.world > 1:
            # the split of a step: this rank's multiply alone (B resident) and
            # the broadcast of B alone
            local = fb.matmul_site(m, n, n)
            r["kernel_ms"] = d.max(time_launches(torch, stream, lambda: ctx.matmul(local, A, B, C, mode),
                                                 lambda: None, 2))
            r["broadcast_ms"] = d.max(time_launches(torch, stream, lambda: ctx.broadcast([B], root=0),
                                                    lambda: None, 2, d))
        if mode == fb.STRICT:
            r["frac_per_gpu"] = tf / d.world / (sms * 128 * pk["sm_max_mhz"] * 1e6 / 1e12)
        else:
            r["frac_per_gpu_of_tf32_div3"] = 3 * tf / d.world / tf_peak
            r["tf32_peak_tflops"] = tf_peak
        out[name] = r
    ctx.synchronize()
    del A, B, C
    torch.cuda.empty_cache()
    return out


def time_launches(torch, stream, fn, flush, reps: int, d=None) -> float:
    """Mean device ms of fn over reps launches, L2 flushed before each. With
    `d` (several ranks), every rank's device is idle and the ranks have met at
    a barrier before the first timed launch, so a collective launch does not
    time another rank's late start."""
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(reps)]
    fn()
    if d is not None and d.world > 1:
        torch.cuda.synchronize()
        d.barrier()
        torch.cuda.synchronize()
    for a, b in evs:
        flush()
        a.record(stream)
        fn()
        b.record(stream)
    torch.cuda.synchronize()
    return sum(a.elapsed_time(b) for a, b in evs) / reps


def run_streaming(ctx, d, fb, torch, flush, pk) -> dict:
    stream = torch.cuda.current_stream()
    hbm = pk["hbm_gbs"]
    out = {"hbm_peak_gbs": hbm, "peak_source": pk["source"]}

    def rec(name, nbytes, ms, extra=None):
        gbs = nbytes / (ms * 1e-3) / 1e9
        r = {"ms": ms, "bytes": nbytes, "gbs": gbs, "frac_hbm": gbs / hbm}
        if extra:
            r.update(extra)
        out[name] = r

    if d.world == 1:
        # 2^20-class sites (the streaming shapes at 2^20 elements): back-to-back launches rotating
        # over enough buffer sets to exceed twice the L2, so no launch finds
        # its inputs in L2, timed as a CUDA graph replay (flow_b200.sitebench).
        from flow_b200 import sitebench
        l2 = ctx.profile().l2_bytes
        sms = ctx.profile().sm_count
        for key, site, size, k in [("saxpy_2^20", "saxpy", 1 << 20, None),
                                   ("transpose_1024^2", "transpose", 1024 * 1024, None),
                                   ("gather_2^20", "gather", 1 << 20, None),
                                   ("sum_2^20", "sum", 1 << 20, None),
                                   ("fir_2^20x64", "fir", 1 << 20, 64),
                                   ("conv2d_1024^2_3x3", "conv2d", 1024 * 1024, None)]:
            r = sitebench.measure(ctx, torch, site, size, k, reps=50, warmup=3, l2_bytes=l2)
            extra = {"buffer_sets": r["buffer_sets"], "launches": r["launches"], "timing": r["timing"],
                     "ms_host_issued": r["ms_host_issued"]}
            if site == "gather":
                extra["bytes_basis"] = "algorithmic 12 B/element"
            if site == "fir":
                extra["fp32_frac"] = r["gflops"] * 1e9 / (sms * 128 * pk["sm_max_mhz"] * 1e6)
            rec(key, r["bytes"], r["ms"], extra)
        # What this class cannot beat, timed the same way: an empty kernel, and
        # the sum fold's own grid and loads over 2^20 floats without its
        # cross-block combine.
        fe = sitebench.measure(ctx, torch, "floor_empty", 1, None, reps=50, warmup=3, l2_bytes=l2)
        fr = sitebench.measure(ctx, torch, "floor_read", 1 << 20, None, reps=50, warmup=3, l2_bytes=l2)
        out["floor_2^20"] = {"empty_kernel_us": fe["ms"] * 1e3, "read_4MiB_us": fr["ms"] * 1e3,
                             "read_4MiB_frac_hbm": fr["gbs"] / hbm,
                             "basis": "CUDA graph replay, inputs outside L2, as the sites; the read has the sum "
                                      "fold's grid and loads and no cross-block combine"}
        out["l2"] = ("2^20 class: launches rotate over buffer sets totalling > 2x L2 and are replayed "
                     "from a CUDA graph (ms_host_issued: the same launches issued from Python); "
                     "2^30 class: inputs far larger than L2")

    # 2^30-class, sharded over the ranks (each rank its contiguous share).
    big = {}
    n = 1 << 30
    lo, hi = fb.shard_range(n, d.world, d.rank)
    m = hi - lo
    x = torch.empty(m, dtype=torch.float32, device="cuda")
    y0 = torch.empty_like(x)
    y = torch.empty_like(x)
    ctx.gen(x, 3, lo)
    ctx.gen(y0, 3, n + lo)
    ms = d.max(time_launches(torch, stream, lambda: ctx.saxpy_sharded(2.5, [x], [y0], [y]), lambda: None, 3, d))
    big["saxpy_2^30"] = {"ms": ms, "gbs": 12 * n / (ms * 1e-3) / 1e9}
    del y0, y
    s = torch.empty(1, dtype=torch.float32, device="cuda")
    ctx.gen(x, 3, lo, fb.U01)
    ms = d.max(time_launches(torch, stream, lambda: ctx.fold_sum_sharded([x], [s]), lambda: None, 3, d))
    comb = ctx.sum_combine()
    big["sum_2^30"] = {"ms": ms, "gbs": 4 * n / (ms * 1e-3) / 1e9,
                       "collective": ("none (one rank)" if d.world == 1 else
                                      "f64 partials exchanged over peer memory inside the fold kernel"
                                      if comb == 1 else "NCCL all-reduce f64")}
    del x
    ng = 1 << 28
    lo, hi = fb.shard_range(ng, d.world, d.rank)
    xg = torch.empty(ng, dtype=torch.float32, device="cuda")
    if d.rank == 0:
        ctx.gen(xg, 3, 0)
    ctx.broadcast([xg], root=0)  # x replicated once, outside the timed region
    idx = torch.empty(hi - lo, dtype=torch.int32, device="cuda")
    ctx.gen_index(idx, 3, ng + lo, ng)
    yg = torch.empty(hi - lo, dtype=torch.float32, device="cuda")
    ms = d.max(time_launches(torch, stream, lambda: ctx.gather_sharded([xg], [idx], [yg]), lambda: None, 3, d))
    big["gather_2^28"] = {"ms": ms, "gbs": 12 * ng / (ms * 1e-3) / 1e9,
                          "bytes_basis": "algorithmic 12 B/element; x replicated by NCCL broadcast at setup"}
    ctx.synchronize()
    for k, v in big.items():
        v["frac_hbm_per_gpu"] = v["gbs"] / d.world / hbm
    out["sharded_2^30"] = big
    return out


def main() -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--no-tf32", action="store_true", help="skip the opt-in 3xTF32 measurement")
    ap.add_argument("--no-16384", action="store_true", help="skip the 16384^2 sharded matmul lines")
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--mode", choices=["strict", "tf32x3"], default="strict")
    ap.add_argument("--no-streaming", action="store_true")
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-check", action="store_true", help="skip the bit-exact check of output rows")
    args = ap.parse_args()
    quiet_stdout()
    if args.warmup < 3 and args.impl == "ours":
        args.warmup = 3
    if args.impl == "reference":
        return reference_arm(args)
    return run_ours(args)


if __name__ == "__main__":
    sys.exit(main())
