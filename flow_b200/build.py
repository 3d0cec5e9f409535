"""Build libmapal_gpu.so in-tree (flow_b200/libmapal_gpu.so) for sm_100a.

    python -m flow_b200.build          # incremental
    python -m flow_b200.build --force  # rebuild everything

Each .cu / .cpp under flow_b200/csrc compiles to an object in
flow_b200/_build; objects are rebuilt when their source or any header
changed. nvcc links the CUDA runtime statically, so the library depends on
the driver only; NCCL is bound at run time with dlopen.
"""
from __future__ import annotations

import argparse
import concurrent.futures as cf
import glob
import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
BUILD = os.path.join(HERE, "_build")
INCLUDE = os.path.join(os.path.dirname(HERE), "include")
LIB = os.path.join(HERE, "libmapal_gpu.so")
DRIVER_SRC = os.path.join(HERE, "driver", "mapal_run.cpp")
DRIVER = os.path.join(HERE, "mapal-run")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
# -fmad=false: no multiply and add is ever contracted into an FMA (the
# interpreter rounds each separately); it covers the packed f32x2 forms too.
NVCC_FLAGS = ARCH + [
    "-O3", "-lineinfo", "-std=c++17", "-fmad=false", "-Xcompiler", "-fPIC",
    "-Xcompiler", "-fvisibility=hidden", "-Xptxas", "-warn-spills", "-I", INCLUDE,
]
CXX_FLAGS = ["-O2", "-std=c++17", "-fPIC", "-fvisibility=hidden", "-ffp-contract=off", "-I", INCLUDE]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), os.path.join(os.environ.get("CUDA_HOME", "/usr/local/cuda"),
                                                       "bin", "nvcc"), shutil.which("nvcc")):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found (set NVCC or CUDA_HOME)")


def _headers_mtime() -> float:
    hs = glob.glob(os.path.join(CSRC, "*.cuh")) + glob.glob(os.path.join(INCLUDE, "*.h"))
    return max((os.path.getmtime(h) for h in hs), default=0.0)


def _compile(src: str, force: bool, hdr_mtime: float) -> str:
    obj = os.path.join(BUILD, os.path.basename(src) + ".o")
    if not force and os.path.exists(obj):
        if os.path.getmtime(obj) >= max(os.path.getmtime(src), hdr_mtime):
            return obj
    if src.endswith(".cu"):
        cmd = [nvcc()] + NVCC_FLAGS + ["-c", src, "-o", obj]
    else:
        cmd = ["g++"] + CXX_FLAGS + ["-c", src, "-o", obj]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"compile failed: {' '.join(cmd)}\n{r.stdout}\n{r.stderr}")
    if "spill" in r.stderr and "0 bytes spill" not in r.stderr:
        sys.stderr.write(r.stderr)
    return obj


def build(force: bool = False, verbose: bool = False) -> str:
    os.makedirs(BUILD, exist_ok=True)
    # A change of compiler flags invalidates every object.
    stamp = os.path.join(BUILD, "flags.txt")
    flags = " ".join(NVCC_FLAGS + CXX_FLAGS)
    if not os.path.exists(stamp) or open(stamp).read() != flags:
        force = True
        with open(stamp, "w") as f:
            f.write(flags)
    srcs = sorted(glob.glob(os.path.join(CSRC, "*.cu")) + glob.glob(os.path.join(CSRC, "*.cpp")))
    hdr = _headers_mtime()
    with cf.ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 1)) as ex:
        objs = list(ex.map(lambda s: _compile(s, force, hdr), srcs))
    newest = max(os.path.getmtime(o) for o in objs)
    if force or not os.path.exists(LIB) or os.path.getmtime(LIB) < newest:
        cmd = [nvcc()] + ARCH + ["-shared", "-o", LIB] + objs + ["-ldl", "-lpthread"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed: {' '.join(cmd)}\n{r.stdout}\n{r.stderr}")
    build_driver(force)
    if verbose:
        print(LIB)
        print(DRIVER)
    return LIB


def build_driver(force: bool = False) -> str:
    """Link the program driver (flow_b200/mapal-run) against the library.

    The CUDA runtime is linked statically; the library is found next to the
    binary through its rpath."""
    newest = max(os.path.getmtime(DRIVER_SRC), os.path.getmtime(LIB), _headers_mtime())
    if force or not os.path.exists(DRIVER) or os.path.getmtime(DRIVER) < newest:
        cuda = os.path.dirname(os.path.dirname(nvcc()))
        cmd = ["g++", "-O2", "-std=c++17", "-ffp-contract=off", "-I", INCLUDE, "-I",
               os.path.join(cuda, "include"), DRIVER_SRC, "-o", DRIVER, "-L", HERE, "-lmapal_gpu",
               "-L", os.path.join(cuda, "lib64"), "-lcudart_static", "-ldl", "-lrt", "-lpthread",
               "-Wl,-rpath,$ORIGIN"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"driver link failed: {' '.join(cmd)}\n{r.stdout}\n{r.stderr}")
    return DRIVER


def main() -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    args = ap.parse_args()
    build(force=args.force, verbose=True)
    return 0


if __name__ == "__main__":
    sys.exit(main())
