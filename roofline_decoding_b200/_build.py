"""Builds libw4b200.so (the sm_100a CUDA library) in-tree with nvcc.

The shared object lands next to this file so that it ships with the source
tree; object files go to ``_build/`` beside it. Only sm_100a is targeted.
"""
from __future__ import annotations

import os
import shutil
import subprocess
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

PKG_DIR = Path(__file__).resolve().parent
REPO_DIR = PKG_DIR.parent
CSRC = PKG_DIR / "csrc"
BUILD_DIR = PKG_DIR / "_build"
LIB_PATH = PKG_DIR / "libw4b200.so"
SOURCES = ["w4_api.cu", "w4_pack.cu", "w4_gemv.cu", "w4_gemv_ops.cu", "w4_gemv_fused.cu",
           "w4_decode.cu", "w4_mega.cu",
           "w4_gemm.cu", "w4_gptq.cu", "w4_tune.cu"]
ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc_path() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found: set NVCC or put the CUDA toolkit on PATH")


def common_flags() -> list[str]:
    return ARCH_FLAGS + [
        "-O3", "-lineinfo", "-std=c++17", "--expt-relaxed-constexpr",
        "-Xcompiler", "-fPIC,-O3", f"-I{REPO_DIR / 'include'}", f"-I{CSRC}",
    ]


def _stale(target: Path, deps: list[Path]) -> bool:
    if not target.exists():
        return True
    t = target.stat().st_mtime
    return any(d.stat().st_mtime > t for d in deps)


def build_library(verbose: bool = False, force: bool = False, ptxas_verbose: bool = False) -> Path:
    """Compiles every CUDA source and links libw4b200.so; returns its path."""
    BUILD_DIR.mkdir(exist_ok=True)
    nvcc = nvcc_path()
    headers = sorted(CSRC.glob("*.cuh")) + sorted(CSRC.glob("*.h")) + [REPO_DIR / "include" / "w4b200.h"]
    objs = []
    jobs = []
    for src in SOURCES:
        s = CSRC / src
        o = BUILD_DIR / (src + ".o")
        objs.append(o)
        if force or _stale(o, [s] + headers):
            cmd = [nvcc, *common_flags(), "-c", str(s), "-o", str(o)]
            if ptxas_verbose:
                cmd += ["-Xptxas", "-v"]
            jobs.append(cmd)

    def run(cmd):
        if verbose:
            print(" ".join(cmd), flush=True)
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"nvcc failed ({' '.join(cmd)}):\n{r.stdout}\n{r.stderr}")
        return r.stdout + r.stderr

    with ThreadPoolExecutor(max_workers=min(8, max(1, len(jobs)))) as ex:
        for out in ex.map(run, jobs):
            if (verbose or ptxas_verbose) and out.strip():
                print(out)
    if force or jobs or _stale(LIB_PATH, objs):
        run([nvcc, *ARCH_FLAGS, "-shared", "-Xcompiler", "-fPIC", *map(str, objs),
             "-o", str(LIB_PATH)])
    return LIB_PATH


if __name__ == "__main__":
    import sys

    print(build_library(verbose=True, force="--force" in sys.argv,
                        ptxas_verbose="-v" in sys.argv))
