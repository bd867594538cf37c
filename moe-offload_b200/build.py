"""Build recipe for libmoe_b200.so: every CUDA/C++ source under csrc/ compiled for sm_100a
with nvcc and linked into one shared library next to this file (in-tree, so the built
library travels with the source tree)."""
from __future__ import annotations

import glob
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
LIB = os.path.join(HERE, "libmoe_b200.so")
OBJ = os.path.join(HERE, "_build")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")


def _flags() -> list[str]:
    return ARCH + [
        "-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "-Xcompiler", "-O3",
        "--expt-relaxed-constexpr", "-rdc=true", "-I", os.path.join(ROOT, "include"), "-I", CSRC,
        "-ccbin", "/usr/bin/g++",
    ]


def sources() -> list[str]:
    return sorted(glob.glob(os.path.join(CSRC, "*.cu")) + glob.glob(os.path.join(CSRC, "*.cpp")))


def _stale(obj: str, src: str) -> bool:
    if not os.path.exists(obj):
        return True
    deps = [src] + glob.glob(os.path.join(CSRC, "*.cuh")) + glob.glob(os.path.join(CSRC, "*.h")) + \
        glob.glob(os.path.join(ROOT, "include", "*.h"))
    t = os.path.getmtime(obj)
    return any(os.path.getmtime(d) > t for d in deps)


TRACE_LIB = os.path.join(HERE, "libmoe_b200_trace.so")
TRACE_OBJ = os.path.join(HERE, "_build_trace")


def build(verbose: bool = False, ptxas_info: bool = False, jobs: int = 8, trace: bool = False) -> str:
    """Builds libmoe_b200.so; trace=True builds the profiling variant libmoe_b200_trace.so
    instead (the persistent decode kernel records per-phase timestamps, MOE_STACK_TRACE)."""
    obj_dir, lib = (TRACE_OBJ, TRACE_LIB) if trace else (OBJ, LIB)
    os.makedirs(obj_dir, exist_ok=True)
    objs, cmds = [], []
    for src in sources():
        obj = os.path.join(obj_dir, os.path.basename(src) + ".o")
        objs.append(obj)
        if _stale(obj, src) or ptxas_info:
            extra = ["-Xptxas", "-v"] if ptxas_info else []
            if trace:
                extra.append("-DMOE_STACK_TRACE")
            cmds.append([NVCC] + _flags() + extra + ["-c", src, "-o", obj])
    procs = []
    for cmd in cmds:
        if verbose:
            print(" ".join(cmd))
        procs.append((cmd, subprocess.Popen(cmd, stdout=subprocess.PIPE, stderr=subprocess.STDOUT, text=True)))
        if len(procs) >= jobs:
            _drain(procs, verbose or ptxas_info)
    _drain(procs, verbose or ptxas_info)
    if cmds or not os.path.exists(lib):
        link = [NVCC] + ARCH + ["-shared", "-rdc=true", "-o", lib] + objs
        if verbose:
            print(" ".join(link))
        subprocess.run(link, check=True)
    return lib


def _drain(procs, show: bool) -> None:
    while procs:
        cmd, p = procs.pop(0)
        out, _ = p.communicate()
        if p.returncode != 0:
            sys.stderr.write(out)
            raise RuntimeError(f"nvcc failed: {' '.join(cmd)}")
        if show and out:
            sys.stdout.write(out)


if __name__ == "__main__":
    print(build(verbose="-v" in sys.argv, ptxas_info="--ptxas" in sys.argv, trace="--trace" in sys.argv))
