"""Builds the in-tree C-ABI library ``flashact_b200/_lib/libflashact.so`` for sm_100a with nvcc.

The library has no torch dependency: it exports the functions declared in include/flashact.h.
"""
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
LIB_DIR = os.path.join(HERE, "_lib")
LIB = os.path.join(LIB_DIR, "libflashact.so")
SOURCES = ["pi05_kernel.cu", "ma2_kernel.cu", "host_pi05.cu", "host_ma2.cu", "host_quant.cu"]
DEPS = SOURCES + ["fa_pi05.cuh", "fa_ma2.cuh", "fa_ptx.cuh", "fa_engine.cuh", "fa_engine_types.cuh", "host_common.cuh"]
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a", "-lineinfo", "-O3", "-std=c++17",
         "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden", "--expt-relaxed-constexpr"]


def _stale() -> bool:
    if not os.path.exists(LIB):
        return True
    t = os.path.getmtime(LIB)
    srcs = [os.path.join(CSRC, f) for f in DEPS] + [os.path.join(ROOT, "include", "flashact.h")]
    return any(os.path.getmtime(s) > t for s in srcs)


def build(force: bool = False, verbose: bool = False, out: str = None, extra_flags=()) -> str:
    """Compiles SOURCES into LIB (or `out`, with `extra_flags` added: for side-by-side variants)."""
    lib = out or LIB
    if out is None and not extra_flags and not force and not _stale():
        return LIB
    os.makedirs(LIB_DIR, exist_ok=True)
    objs = []
    for src in SOURCES:
        obj = os.path.join(LIB_DIR, src.replace(".cu", ".o"))
        cmd = [NVCC, *FLAGS, *extra_flags, "-rdc=false", "-c", os.path.join(CSRC, src), "-o", obj]
        if verbose:
            cmd.insert(1, "-Xptxas=-v")
            print(" ".join(cmd), file=sys.stderr)
        subprocess.run(cmd, check=True)
        objs.append(obj)
    subprocess.run([NVCC, "-shared", "-gencode", "arch=compute_100a,code=sm_100a", *objs, "-o", lib], check=True)
    for o in objs:
        os.remove(o)
    return lib


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose="-v" in sys.argv))
