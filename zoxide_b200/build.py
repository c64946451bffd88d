"""Build libzoxide_b200.so in-tree with nvcc for sm_100a.

The shared library is the product: the C ABI of include/zoxide_gemm.h plus every tcgen05
kernel behind it. It is written to zoxide_b200/_build/ so it travels with the source tree.
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
BUILD = PKG / "_build"
LIB = BUILD / "libzoxide_b200.so"

SOURCES = ["zx_api.cu"]
HEADERS = ["zx_ptx.cuh", "zx_gemm_tc.cuh", "zx_gemm_tc2.cuh", "zx_unpack.cuh", "zx_gemm_sp2.cuh",
           "zx_compat.cuh", "zx_gemm_w4s.cuh", "zx_gemm_tc2w.cuh", "zx_gemm_w4t.cuh", "zx_gemm_sp2w.cuh", "zx_layout.cuh", "zx_gemm_sp4.cuh"]
# Reference-contract kernels as standalone cubins named by the reference's harness stems.
CUBINS = {f"{stem}.cubin": "zx_compat_cubin.cu"
          for stem in ("imma_s8", "imma_s4", "imma_sp_s8", "imma_sp_s4", "hgemm_bf16", "hgemm_wgmma_bf16",
                       "hgemm_tma")}

GENCODE = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", shutil.which("nvcc")):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found: the sm_100a library cannot be built")


def _stale() -> bool:
    if not LIB.exists():
        return True
    t = LIB.stat().st_mtime
    deps = [CSRC / s for s in SOURCES + HEADERS + list(CUBINS.values())]
    deps += [ROOT / "include" / "zoxide_gemm.h", Path(__file__)]
    if any(not (BUILD / n).exists() for n in CUBINS):
        return True
    return any(d.stat().st_mtime > t for d in deps if d.exists())


def build(force: bool = False, verbose: bool = False, ptxas_verbose: bool = False) -> Path:
    if not force and not _stale():
        return LIB
    BUILD.mkdir(parents=True, exist_ok=True)
    cmd = [
        nvcc(), *GENCODE, "-O3", "-lineinfo", "-std=c++17", "-shared", "-Xcompiler", "-fPIC",
        "-Xcompiler", "-fvisibility=hidden", "-I", str(ROOT / "include"),
        "--expt-relaxed-constexpr", "-o", str(LIB) + ".tmp",
        *[str(CSRC / s) for s in SOURCES],
    ]
    if ptxas_verbose:
        cmd += ["-Xptxas", "-v"]
    if verbose:
        print(" ".join(cmd), file=sys.stderr)
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc failed ({res.returncode}):\n{res.stdout}\n{res.stderr}")
    if ptxas_verbose or verbose:
        sys.stderr.write(res.stdout + res.stderr)
    os.replace(str(LIB) + ".tmp", LIB)
    for name, src in CUBINS.items():
        out = BUILD / name
        cmd = [nvcc(), *GENCODE, "-O3", "-lineinfo", "-std=c++17", "-cubin", "-o", str(out) + ".tmp",
               str(CSRC / src)]
        res = subprocess.run(cmd, capture_output=True, text=True)
        if res.returncode != 0:
            raise RuntimeError(f"nvcc -cubin failed ({res.returncode}):\n{res.stdout}\n{res.stderr}")
        os.replace(str(out) + ".tmp", out)
    return LIB


if __name__ == "__main__":
    p = build(force="--force" in sys.argv, verbose=True, ptxas_verbose="-v" in sys.argv)
    print(p)
