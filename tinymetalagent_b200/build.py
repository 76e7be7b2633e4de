"""Builds libtinyengine.so in-tree: sm_100a CUDA kernels + C/C++ host layer.

Usage: ``python -m tinymetalagent_b200.build`` (or ``build()`` from Python).
nvcc cross-compiles for sm_100a without a GPU.  cudart is linked statically so
the library does not depend on which CUDA runtime the host process loaded.
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

PKG = Path(__file__).resolve().parent
CSRC = PKG / "csrc"
OUT = PKG / "libtinyengine.so"
BUILD = PKG / "_build"
CUDA_HOME = Path(os.environ.get("CUDA_HOME", "/usr/local/cuda"))

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
CU_SOURCES = ["k_decode.cu", "k_rope.cu", "k_prefill.cu", "k_exchange.cu", "k_gemv.cu", "k_step.cu"]
CXX_SOURCES = ["te_api.cpp"]
C_SOURCES = ["rope_table.c"]


def _nvcc() -> str:
    p = CUDA_HOME / "bin" / "nvcc"
    return str(p) if p.exists() else "nvcc"


def _compile_cmds(verbose_ptxas: bool = False) -> list[list[str]]:
    cmds = []
    inc = ["-I", str(CSRC), "-I", str(PKG.parent / "include")]
    for s in CU_SOURCES:
        if not (CSRC / s).exists():
            continue
        cmd = [_nvcc(), *ARCH, "-lineinfo", "-O3", "-std=c++17", "--expt-relaxed-constexpr",
               "-Xcompiler", "-fPIC,-fvisibility=hidden", *inc, "-c", str(CSRC / s),
               "-o", str(BUILD / (s + ".o"))]
        if verbose_ptxas:
            cmd.insert(1, "-Xptxas=-v")
        cmds.append(cmd)
    for s in CXX_SOURCES:
        cmds.append(["g++", "-O2", "-std=c++17", "-fPIC", "-fvisibility=hidden", "-Wall", "-Wextra",
                     "-I", str(CUDA_HOME / "include"), *inc, "-c", str(CSRC / s), "-o", str(BUILD / (s + ".o"))])
    for s in C_SOURCES:
        # -ffp-contract=off and the baseline x86-64 ISA keep the RoPE table bit-identical
        # to the reference's CPU computation.
        cmds.append(["gcc", "-O2", "-std=c11", "-fPIC", "-fvisibility=hidden", "-ffp-contract=off", "-Wall",
                     "-c", str(CSRC / s), "-o", str(BUILD / (s + ".o"))])
    return cmds


def build(verbose: bool = False, verbose_ptxas: bool = False) -> Path:
    BUILD.mkdir(exist_ok=True)
    cmds = _compile_cmds(verbose_ptxas)

    def run(cmd):
        if verbose:
            print(" ".join(cmd), flush=True)
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0 or (verbose_ptxas and r.stderr):
            sys.stderr.write(r.stdout + r.stderr)
        if r.returncode != 0:
            raise RuntimeError(f"compile failed: {' '.join(cmd)}")

    with ThreadPoolExecutor(max_workers=min(8, len(cmds))) as ex:
        list(ex.map(run, cmds))
    srcs = [s for s in CU_SOURCES if (CSRC / s).exists()] + CXX_SOURCES + C_SOURCES
    objs = [str(BUILD / (s + ".o")) for s in srcs]
    tmp = OUT.with_suffix(".so.tmp")
    link = ["g++", "-shared", "-o", str(tmp), *objs, "-L", str(CUDA_HOME / "lib64"),
            "-lcudart_static", "-lrt", "-ldl", "-lpthread", "-Wl,--exclude-libs,ALL", "-Wl,-z,defs",
            f"-Wl,--version-script={CSRC / 'exports.map'}"]
    if verbose:
        print(" ".join(link), flush=True)
    r = subprocess.run(link, capture_output=True, text=True)
    if r.returncode != 0:
        sys.stderr.write(r.stdout + r.stderr)
        raise RuntimeError("link failed")
    shutil.move(str(tmp), str(OUT))
    return OUT


if __name__ == "__main__":
    build(verbose=True, verbose_ptxas="--ptxas" in sys.argv)
    print(f"built {OUT}")
