"""Build ``libkvbp.so`` (the C-ABI CUDA library) in-tree with nvcc for sm_100a.

    python -m kvcacheboundaryprotection_b200.build [--force] [--verbose]

The library links the CUDA runtime statically and resolves the driver entry point
``cuTensorMapEncodeTiled`` at run time, so it loads on hosts without a GPU driver
(its compute entry points then fail with KVBP_ERR_CUDA).
"""

from __future__ import annotations

import argparse
import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
CSRC = PKG / "csrc"
LIB_DIR = PKG / "lib"
LIB = LIB_DIR / "libkvbp.so"
INCLUDE = PKG.parent / "include"
SOURCES = ["capi.cu", "attn_decode.cu", "dense.cu", "evict.cu", "gemm_decode.cu", "prefill_attn.cu", "prefill_gemm.cu"]
HEADERS = ["common.cuh", "kvbp_internal.h"]

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", "-Xcompiler", "-O3", "--expt-relaxed-constexpr"]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found: the CUDA toolkit is required to build libkvbp.so")


def _inputs():
    return [CSRC / s for s in SOURCES] + [CSRC / h for h in HEADERS] + [INCLUDE / "kvbp.h", Path(__file__)]


def up_to_date() -> bool:
    if not LIB.exists():
        return False
    t = LIB.stat().st_mtime
    return all(p.stat().st_mtime <= t for p in _inputs())


def build(force: bool = False, verbose: bool = False, ptxas_verbose: bool = False) -> Path:
    if not force and up_to_date():
        return LIB
    LIB_DIR.mkdir(parents=True, exist_ok=True)
    tmp = LIB_DIR / "libkvbp.so.tmp"
    cmd = [nvcc(), *ARCH, *FLAGS, "-shared", "-o", str(tmp), *[str(CSRC / s) for s in SOURCES]]
    if ptxas_verbose:
        cmd += ["-Xptxas", "-v"]
    if verbose:
        print(" ".join(cmd), flush=True)
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        sys.stderr.write(r.stdout + r.stderr)
        raise RuntimeError(f"nvcc failed with exit code {r.returncode}")
    if verbose or ptxas_verbose:
        sys.stdout.write(r.stdout + r.stderr)
    os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose", action="store_true")
    ap.add_argument("--ptxas", action="store_true", help="print ptxas register/smem usage")
    a = ap.parse_args()
    print(build(force=a.force or a.ptxas, verbose=a.verbose, ptxas_verbose=a.ptxas))
