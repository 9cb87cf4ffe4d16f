"""Builds libnf_moe.so (the C-ABI library of include/nf_moe.h) for sm_100a.

Steps:
  1. compile and run csrc/gen_sigmoid_table.c, which records where the host
     libm's expf-based sigmoid (the reference router's) differs from a
     correctly rounded one, into csrc/_gen/sigmoid_table.inc;
  2. nvcc every csrc/*.cu to an object with
     -gencode arch=compute_100a,code=sm_100a and link lib/libnf_moe.so
     (static CUDA runtime, so the library does not depend on the runtime
     version another component of the process loaded).

Incremental: a step is skipped when its outputs are newer than its inputs.
Run:  python build.py [--verbose-ptxas]
"""
from __future__ import annotations

import os
import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
REPO = HERE.parent
CSRC = HERE / "csrc"
GEN = CSRC / "_gen"
OBJ = HERE / "_build"
LIB = HERE / "lib" / "libnf_moe.so"
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
CU_SOURCES = ["nf_kernels.cu", "nf_gemm.cu", "nf_gemm2.cu", "nf_moe.cu", "nf_noalloc.cu", "nf_ep.cu", "nf_tp.cu", "nf_attn.cu",
              "nf_stack.cu"]
HEADERS = ["nf_handle.h", "nf_common.cuh", "nf_internal.h", "nf_nccl.h", "nf_gemm_shared.cuh"]


def _newer(out: Path, inputs: list[Path]) -> bool:
    if not out.exists():
        return False
    t = out.stat().st_mtime
    return all(p.stat().st_mtime <= t for p in inputs)


def _run(cmd: list[str], **kw) -> None:
    print("+", " ".join(str(c) for c in cmd), flush=True)
    subprocess.run([str(c) for c in cmd], check=True, **kw)


def gen_sigmoid_table() -> Path:
    out = GEN / "sigmoid_table.inc"
    src = CSRC / "gen_sigmoid_table.c"
    if _newer(out, [src]):
        return out
    GEN.mkdir(parents=True, exist_ok=True)
    exe = OBJ / "gen_sigmoid_table"
    OBJ.mkdir(parents=True, exist_ok=True)
    # gcc from PATH: the reference's sigmoid uses the host libm expf, so the
    # table must come from that same libm.
    _run(["gcc", "-O2", "-ffp-contract=off", "-fopenmp", str(src), "-o", str(exe), "-lm"])
    _run([str(exe), str(out)])
    return out


def build(verbose_ptxas: bool = False) -> Path:
    table = gen_sigmoid_table()
    OBJ.mkdir(parents=True, exist_ok=True)
    LIB.parent.mkdir(parents=True, exist_ok=True)
    headers = [CSRC / h for h in HEADERS] + [REPO / "include" / "nf_moe.h", table]
    objs = []
    for name in CU_SOURCES:
        src = CSRC / name
        obj = OBJ / (name + ".o")
        objs.append(obj)
        if _newer(obj, [src] + headers) and not verbose_ptxas:
            continue
        cmd = [NVCC, *ARCH, "-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
               "-I", REPO / "include", "-I", CSRC, "-c", src, "-o", obj]
        if verbose_ptxas:
            cmd[1:1] = ["-Xptxas", "-v"]
        _run(cmd)
    if not _newer(LIB, objs):
        _run([NVCC, *ARCH, "-shared", "-Xcompiler", "-fPIC", *objs, "-o", LIB, "-ldl"])
    # the C++ host example (host/): header-only class over the C ABI + a demo program
    demo = LIB.parent / "moe_demo"
    host = HERE / "host"
    if not _newer(demo, [host / "moe_demo.cpp", host / "nf_moe_layer.hpp", host / "nf_safetensors.hpp",
                         REPO / "include" / "nf_moe.h", LIB]):
        _run(["g++", "-O2", "-std=c++17", "-I", REPO / "include", "-I", host, host / "moe_demo.cpp", "-o", demo,
              "-L", LIB.parent, "-lnf_moe", "-Wl,-rpath,$ORIGIN"])
    return LIB


if __name__ == "__main__":
    build(verbose_ptxas="--verbose-ptxas" in sys.argv)
    print(LIB)
