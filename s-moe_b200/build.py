"""Build libsmoe_cuda.so (sm_100a) in-tree with nvcc.

    python s-moe_b200/build.py [--force] [--trace]

--trace builds libsmoe_cuda_trace.so instead: the same library with the
layer kernel's phase timestamps compiled in (smoe_cuda_debug_trace; read by
trace_layer.py). The product library has none of that code - the kernel's
instruction footprint is on its critical path.
"""
from __future__ import annotations

import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
LIB = os.path.join(HERE, "libsmoe_cuda.so")
LIB_TRACE = os.path.join(HERE, "libsmoe_cuda_trace.so")
SOURCES = [os.path.join(HERE, "csrc", "smoe_cuda.cu"), os.path.join(HERE, "csrc", "smoe_noalloc.cu"),
           os.path.join(HERE, "csrc", "smoe_vault.cpp")]
DEPS = SOURCES + [os.path.join(HERE, "csrc", f) for f in os.listdir(os.path.join(HERE, "csrc"))] + [
    os.path.join(ROOT, "include", "smoe_cuda.h")]

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-lineinfo", "-O3", "-std=c++17",
    "-Xcompiler", "-fPIC", "-shared",
    "-Xptxas", "-v",
    "-lcublas",
]


def nvcc() -> str:
    for c in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", "nvcc"):
        if c and (os.path.isabs(c) and os.path.exists(c) or not os.path.isabs(c)):
            return c
    return "nvcc"


def up_to_date(lib: str = LIB) -> bool:
    if not os.path.exists(lib):
        return False
    t = os.path.getmtime(lib)
    return all(os.path.getmtime(p) <= t for p in DEPS if os.path.exists(p))


def build(force: bool = False, verbose: bool = False, trace: bool = False) -> str:
    lib = LIB_TRACE if trace else LIB
    if not force and up_to_date(lib):
        return lib
    cmd = [nvcc(), *NVCC_FLAGS, *(["-DSMOE_TRACE"] if trace else []), *SOURCES, "-o", lib]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if verbose or r.returncode != 0:
        sys.stderr.write(r.stdout + r.stderr)
    if r.returncode != 0:
        raise RuntimeError("nvcc failed building " + os.path.basename(lib))
    return lib


ENGINE = os.path.join(HERE, "smoe_engine")
ENGINE_SRC = os.path.join(HERE, "engine", "smoe_engine.cu")


def build_engine(force: bool = False, verbose: bool = False) -> str:
    """The C++ engine binary (engine/smoe_engine.cu), linked against the
    library beside it (rpath $ORIGIN)."""
    lib = build(force=force, verbose=verbose)
    if not force and os.path.exists(ENGINE) and os.path.getmtime(ENGINE) >= max(
            os.path.getmtime(ENGINE_SRC), os.path.getmtime(lib), os.path.getmtime(os.path.join(ROOT, "include", "smoe_cuda.h"))):
        return ENGINE
    cmd = [nvcc(), "-gencode", "arch=compute_100a,code=sm_100a", "-O3", "-std=c++17", ENGINE_SRC, "-o", ENGINE,
           "-L" + HERE, "-lsmoe_cuda", "-Xlinker", "-rpath,$ORIGIN"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if verbose or r.returncode != 0:
        sys.stderr.write(r.stdout + r.stderr)
    if r.returncode != 0:
        raise RuntimeError("nvcc failed building smoe_engine")
    return ENGINE


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose=True, trace="--trace" in sys.argv))
    if "--trace" not in sys.argv:
        print(build_engine(force="--force" in sys.argv))
