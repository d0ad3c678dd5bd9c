"""Build the in-tree CUDA library libgalactus_b200.so for sm_100a.

Run as ``python -m galactus_b200.build``. Steps:
  1. generate csrc/_gen/iq1s_grid.inc, the IQ1_S codebook, from the installed
     gguf-py package (the table is read from the package, never retyped);
  2. compile the kernels, the slot policy and the C-ABI with nvcc into
     galactus_b200/libgalactus_b200.so (static cudart, -gencode sm_100a).
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
CSRC = PKG / "csrc"
GEN = CSRC / "_gen"
LIB = PKG / "libgalactus_b200.so"

SOURCES = ["gx_kernels.cu", "gx_capi.cpp", "gx_policy.cpp", "gx_noalloc.cu", "gx_ep.cpp", "gx_plan.cpp", "gx_observer.cpp", "gx_gguf.cpp"]
HEADERS = ["gx_device.cuh", "gx_moe.cuh", "gx_stack.cuh", "gx_prefill.cuh", "gx_mma.cuh", "gx_tc.cuh", "gx_stack_tc.cuh", "gx_stack_tma.cuh", "gx_router.cuh", "gx_formats.h", "gx_kernels.h", "gx_policy.hpp", "gx_observer.hpp"]

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-lineinfo", "-O3", "-std=c++17",
    # every float operation in the kernels carries an explicit rounding
    # intrinsic; no contraction and no approximation may be introduced
    "--fmad=false", "-prec-div=true", "-prec-sqrt=true", "-ftz=false",
    "-Xcompiler", "-fPIC", "-Xcompiler", "-O2",
    "-cudart", "static",
]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found")


def gen_iq1s_grid() -> None:
    out = GEN / "iq1s_grid.inc"
    GEN.mkdir(parents=True, exist_ok=True)
    try:
        import numpy as np
        from gguf.quants import IQ1_S
    except Exception as exc:  # pragma: no cover - gguf is part of the image
        if out.exists():
            return
        raise RuntimeError(f"cannot generate the IQ1_S grid: {exc}")
    IQ1_S.init_grid()
    grid = np.asarray(IQ1_S.grid).reshape(2048, 8).astype(np.int8)
    words = np.ascontiguousarray(grid).view(np.uint32).reshape(2048, 2)
    text = "".join("{0x%08xu, 0x%08xu},\n" % (int(a), int(b)) for a, b in words)
    if not out.exists() or out.read_text() != text:
        out.write_text(text)


def needs_build() -> bool:
    if not LIB.exists():
        return True
    t = LIB.stat().st_mtime
    deps = [CSRC / s for s in SOURCES + HEADERS] + [PKG.parent / "include" / "galactus_b200.h", Path(__file__)]
    return any(d.exists() and d.stat().st_mtime > t for d in deps)


def build(force: bool = False, verbose: bool = False) -> Path:
    gen_iq1s_grid()
    if not force and not needs_build():
        return LIB
    objs = []
    tmp = CSRC / "_gen" / "obj"
    tmp.mkdir(parents=True, exist_ok=True)
    for src in SOURCES:
        obj = tmp / (Path(src).stem + ".o")
        cmd = [nvcc(), *NVCC_FLAGS, "-I", str(CSRC), "-I", str(PKG.parent / "include"), "-c", str(CSRC / src), "-o", str(obj)]
        if verbose:
            print(" ".join(cmd))
        subprocess.run(cmd, check=True)
        objs.append(str(obj))
    cmd = [nvcc(), "-gencode", "arch=compute_100a,code=sm_100a", "-shared", "-cudart", "static",
           "-o", str(LIB), *objs, "-lpthread", "-ldl"]
    if verbose:
        print(" ".join(cmd))
    subprocess.run(cmd, check=True)
    return LIB


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose=True)
    print(LIB)
