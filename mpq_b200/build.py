"""Build ``libmpq_b200.so`` in-tree with nvcc for sm_100a (``python -m mpq_b200.build``)."""
from __future__ import annotations

import os
import shutil
import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
CSRC = HERE / "csrc"
OUT = HERE / "libmpq_b200.so"

SOURCES = ["capi.cu", "uniform_prior.cu", "vamp_uniform.cu", "gemm_simt.cu", "scalar_cd.cu", "hadamard.cu", "gemm_tc.cu", "e8p12.cu",
           "gram_cd.cu", "hessian.cu", "block_cd.cu", "pack.cu", "topk.cu"]

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-lineinfo", "-std=c++17",
    "-shared", "-Xcompiler", "-fPIC,-fvisibility=hidden",
]


def nvcc_path() -> str:
    cand = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not Path(cand).exists():
        raise RuntimeError("nvcc not found; the CUDA 12.9 toolkit is required to build libmpq_b200.so")
    return cand


def build(verbose: bool = False, force: bool = False) -> Path:
    srcs = [CSRC / s for s in SOURCES]
    deps = srcs + sorted(CSRC.glob("*.cuh"))
    if OUT.exists() and not force:
        newest = max(p.stat().st_mtime for p in deps)
        if OUT.stat().st_mtime >= newest:
            return OUT
    tmp = OUT.with_suffix(f".so.tmp{os.getpid()}")
    cmd = [nvcc_path(), *NVCC_FLAGS, *(["-Xptxas", "-v"] if verbose else []), "-o", str(tmp), *map(str, srcs)]
    res = subprocess.run(cmd, cwd=str(CSRC), capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc failed ({res.returncode}):\n{res.stdout}\n{res.stderr}")
    if verbose:
        print(res.stdout, res.stderr, sep="\n")
    tmp.replace(OUT)
    return OUT


if __name__ == "__main__":
    p = build(verbose="-v" in sys.argv, force=True)
    print("built", p)
