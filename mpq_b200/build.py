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

SOURCES = ["capi.cu", "peer.cu", "uniform_prior.cu", "vamp_uniform.cu", "gemm_simt.cu", "scalar_cd.cu", "hadamard.cu", "gemm_tc.cu", "e8p12.cu",
           "gram_cd.cu", "hessian.cu", "block_cd.cu", "pack.cu", "topk.cu", "vamp_ctl.cu"]

ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a", "-O3", "-lineinfo", "-std=c++17"]
COMPILE_FLAGS = ARCH_FLAGS + ["-Xcompiler", "-fPIC,-fvisibility=hidden"]
LINK_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a", "-shared"]


def nvcc_path() -> str:
    cand = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not Path(cand).exists():
        raise RuntimeError("nvcc not found; the CUDA 12.9 toolkit is required to build libmpq_b200.so")
    return cand


def _compile(nvcc: str, src: Path, obj: Path, verbose: bool) -> str:
    cmd = [nvcc, *COMPILE_FLAGS, *(["-Xptxas", "-v"] if verbose else []), "-c", "-o", str(obj), str(src)]
    res = subprocess.run(cmd, cwd=str(CSRC), capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc failed on {src.name} ({res.returncode}):\n{res.stdout}\n{res.stderr}")
    return res.stdout + res.stderr


def build(verbose: bool = False, force: bool = False) -> Path:
    """Compile every source to an object (in parallel, sm_100a) and link libmpq_b200.so in place."""
    from concurrent.futures import ThreadPoolExecutor
    srcs = [CSRC / s for s in SOURCES]
    deps = srcs + sorted(CSRC.glob("*.cuh"))
    if OUT.exists() and not force:
        newest = max(p.stat().st_mtime for p in deps)
        if OUT.stat().st_mtime >= newest:
            return OUT
    nvcc = nvcc_path()
    objdir = HERE / "_build" / f"obj{os.getpid()}"
    objdir.mkdir(parents=True, exist_ok=True)
    objs = [objdir / (s.stem + ".o") for s in srcs]
    with ThreadPoolExecutor(max_workers=min(len(srcs), os.cpu_count() or 4)) as ex:
        logs = list(ex.map(lambda so: _compile(nvcc, so[0], so[1], verbose), zip(srcs, objs)))
    tmp = OUT.with_suffix(f".so.tmp{os.getpid()}")
    res = subprocess.run([nvcc, *LINK_FLAGS, "-o", str(tmp), *map(str, objs)], cwd=str(CSRC), capture_output=True,
                         text=True)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc link failed ({res.returncode}):\n{res.stdout}\n{res.stderr}")
    if verbose:
        print("\n".join(logs))
    tmp.replace(OUT)
    shutil.rmtree(objdir, ignore_errors=True)
    return OUT


if __name__ == "__main__":
    p = build(verbose="-v" in sys.argv, force=True)
    print("built", p)
