"""Build recipe of libtabnet_stage.so (sm_100a) and of the oracle library.

The engine is plain CUDA C++ compiled by nvcc for sm_100a only, with the CUDA
runtime linked statically so the shared library has no dependency beyond the
driver.  Objects go to _build/ beside this file; the library lands in the
package directory, where the Python host binding loads it.
"""
from __future__ import annotations

import concurrent.futures as cf
import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
CSRC = PKG / "csrc"
BUILD = PKG / "_build"
LIB = PKG / "libtabnet_stage.so"
SOURCES = ["tn_synth.cu", "tn_kernels.cu", "tn_mmv.cu", "tn_gemm.cu", "tn_attn.cu", "tn_stage.cu", "tn_abi.cu"]
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ARCH + [
    "-O3", "-lineinfo", "-std=c++17", "--expt-relaxed-constexpr",
    "-Xcompiler", "-fPIC", "-Xcompiler", "-ffp-contract=off",
    "-Xcompiler", "-Wall", "-Xcompiler", "-Wno-unused-function",
]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", shutil.which("nvcc")):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found: the stage engine needs the CUDA toolkit to build")


def _run(cmd: list[str]) -> None:
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"command failed ({r.returncode}): {' '.join(cmd)}\n{r.stdout}\n{r.stderr}")


def build_engine(verbose: bool = False, ptxas_info: bool = False) -> Path:
    """Compile csrc/*.cu for sm_100a and link libtabnet_stage.so (incremental)."""
    BUILD.mkdir(exist_ok=True)
    headers = list(CSRC.glob("*.cuh")) + [PKG.parent / "include" / "tabnet_stage.h"]
    newest_header = max(h.stat().st_mtime for h in headers)
    objs, jobs = [], []
    for src in SOURCES:
        s = CSRC / src
        o = BUILD / (s.stem + ".o")
        objs.append(o)
        if o.exists() and o.stat().st_mtime >= max(s.stat().st_mtime, newest_header) and not ptxas_info:
            continue
        cmd = [nvcc()] + NVCC_FLAGS + (["-Xptxas", "-v"] if ptxas_info else []) + ["-c", str(s), "-o", str(o)]
        jobs.append(cmd)
    with cf.ThreadPoolExecutor(max_workers=len(SOURCES)) as ex:
        for cmd, fut in [(c, ex.submit(subprocess.run, c, capture_output=True, text=True)) for c in jobs]:
            r = fut.result()
            if r.returncode != 0:
                raise RuntimeError(f"nvcc failed: {' '.join(cmd)}\n{r.stdout}\n{r.stderr}")
            if verbose or ptxas_info:
                sys.stderr.write(r.stderr)
    if jobs or not LIB.exists() or LIB.stat().st_mtime < max(o.stat().st_mtime for o in objs):
        tmp = LIB.with_suffix(".so.tmp")
        _run([nvcc()] + ARCH + ["-shared", "-cudart", "static", "-o", str(tmp)] + [str(o) for o in objs])
        os.replace(tmp, LIB)
    return LIB


def build_oracle() -> Path:
    """Compile the oracle (test infrastructure) with its Makefile."""
    oracle = PKG.parent / "oracle"
    _run(["make", "-s", "-C", str(oracle)])
    return oracle / "libref_cpu.so"


if __name__ == "__main__":
    print(build_engine(verbose=True, ptxas_info="-v" in sys.argv))
    print(build_oracle())
