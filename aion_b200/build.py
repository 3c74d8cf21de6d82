"""Build recipe for libaion.so and the `aion` CLI (in-tree, sm_100a only).

    python -m aion_b200.build          # builds aion_b200/lib/libaion.so and aion_b200/bin/aion

The CUDA sources compile with nvcc for sm_100a (`-gencode
arch=compute_100a,code=sm_100a`); the host C tools compile with gcc and
`-ffp-contract=off` (the int4 quantizer must round like the reference
converter).  Objects go to aion_b200/_build/, outputs stay inside the
package so the built library travels with the source tree.
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
CSRC = PKG / "csrc"
BUILD = PKG / "_build"
LIB = PKG / "lib" / "libaion.so"
CLI = PKG / "bin" / "aion"
INCLUDE = PKG.parent / "include"

NVCC_ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC,-fvisibility=hidden", "--expt-relaxed-constexpr",
              "-Xptxas", "-warn-spills"]
CC_FLAGS = ["-O2", "-std=gnu11", "-fPIC", "-fvisibility=hidden", "-ffp-contract=off", "-pthread", "-Wall",
            "-Wno-unused-result"]

CUDA_SOURCES = ["aion_runtime.cu"]
C_SOURCES = ["aion_ckpt.c", "aion_tok.c"]


def _nvcc() -> str:
    for cand in (shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found")


def _run(cmd: list[str]) -> None:
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        sys.stderr.write(" ".join(cmd) + "\n" + r.stdout + r.stderr)
        raise RuntimeError(f"build step failed: {cmd[0]} {cmd[-1]}")
    if r.stderr.strip():
        sys.stderr.write(r.stderr)


def _stale(out: Path, deps: list[Path]) -> bool:
    if not out.exists():
        return True
    t = out.stat().st_mtime
    return any(d.stat().st_mtime > t for d in deps)


def build(verbose: bool = False, ptxas_info: bool = False) -> Path:
    BUILD.mkdir(exist_ok=True)
    LIB.parent.mkdir(exist_ok=True)
    CLI.parent.mkdir(exist_ok=True)
    headers = list(CSRC.glob("*.cuh")) + list(CSRC.glob("*.h")) + [INCLUDE / "aion.h"]
    objs: list[Path] = []
    nvcc = _nvcc()
    for src in CUDA_SOURCES:
        obj = BUILD / (Path(src).stem + ".o")
        if _stale(obj, [CSRC / src] + headers) or ptxas_info:
            cmd = [nvcc, *NVCC_ARCH, *NVCC_FLAGS, "-I", str(INCLUDE), "-c", str(CSRC / src), "-o", str(obj)]
            if ptxas_info:
                cmd[1:1] = ["-Xptxas", "-v"]
            if verbose:
                print(" ".join(cmd))
            _run(cmd)
        objs.append(obj)
    for src in C_SOURCES:
        obj = BUILD / (Path(src).stem + ".o")
        if _stale(obj, [CSRC / src] + headers):
            cmd = ["gcc", *CC_FLAGS, "-I", str(INCLUDE), "-c", str(CSRC / src), "-o", str(obj)]
            if verbose:
                print(" ".join(cmd))
            _run(cmd)
        objs.append(obj)
    if _stale(LIB, objs):
        cmd = [nvcc, *NVCC_ARCH, "-shared", "-o", str(LIB), *map(str, objs), "-lcudart", "-lpthread", "-lm"]
        if verbose:
            print(" ".join(cmd))
        _run(cmd)
    cli_src = CSRC / "aion_cli.c"
    if cli_src.exists() and _stale(CLI, [cli_src, LIB, INCLUDE / "aion.h"]):
        cmd = ["gcc", "-O2", "-std=gnu11", "-Wall", "-I", str(INCLUDE), "-o", str(CLI), str(cli_src),
               "-L", str(LIB.parent), "-laion", "-Wl,-rpath,$ORIGIN/../lib", "-lm"]
        _run(cmd)
    return LIB


if __name__ == "__main__":
    build(verbose="-v" in sys.argv, ptxas_info="--ptxas" in sys.argv)
    print(LIB)
