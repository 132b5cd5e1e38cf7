"""Build libctu_b200.so (the C-ABI CUDA library) in-tree for sm_100a.

Usage: python comfyui-turing-utils_b200/build.py [--force] [-v]

The shared library lands next to the Python package that loads it
(comfyui_turing_utils_kernel/libctu_b200.so), so it travels with the source tree.
"""

from __future__ import annotations

import argparse
import concurrent.futures as cf
import os
import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
CSRC = HERE / "csrc"
INCLUDE = HERE.parent / "include"
OUT_DIR = HERE / "comfyui_turing_utils_kernel"
LIB = OUT_DIR / "libctu_b200.so"
OBJ_DIR = HERE / "_build"

SOURCES = ["capi.cu", "convrot_quant.cu", "convrot_quant_reg.cu", "convrot_quant_t4.cu", "convrot_quant_k8.cu", "gemm_i8.cu", "gemm_pair.cu", "gemm_grouped.cu", "dequant.cu", "noalloc.cu", "codebook.cu", "unpack_s4.cu", "norm_adaln.cu"]
NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-std=c++17", "-lineinfo",
    "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
    "--expt-relaxed-constexpr",
    # Kernel templates are declared in headers and instantiated in their own .cu files.
    "-diag-suppress", "20281",
]


def _nvcc() -> str:
    cuda = os.environ.get("CUDA_HOME", "/usr/local/cuda")
    cand = Path(cuda) / "bin" / "nvcc"
    return str(cand) if cand.exists() else "nvcc"


def _stale(target: Path, deps) -> bool:
    if not target.exists():
        return True
    t = target.stat().st_mtime
    return any(Path(d).stat().st_mtime > t for d in deps)


def build(force: bool = False, verbose: bool = False) -> Path:
    OBJ_DIR.mkdir(exist_ok=True)
    headers = sorted(CSRC.glob("*.cuh")) + sorted(INCLUDE.glob("*.h"))
    jobs = []
    for src in SOURCES:
        obj = OBJ_DIR / (Path(src).stem + ".o")
        if force or _stale(obj, [CSRC / src, *headers]):
            cmd = [_nvcc(), *NVCC_FLAGS, f"-I{INCLUDE}", "-c", str(CSRC / src), "-o", str(obj)]
            if verbose:
                cmd.insert(1, "-Xptxas=-v")
            jobs.append(cmd)
    with cf.ThreadPoolExecutor(max_workers=len(SOURCES)) as pool:
        for res in pool.map(lambda c: subprocess.run(c, capture_output=True, text=True), jobs):
            if verbose or res.returncode != 0:
                sys.stderr.write(res.stdout + res.stderr)
            if res.returncode != 0:
                raise RuntimeError("nvcc failed: " + " ".join(res.args))
    objs = [OBJ_DIR / (Path(s).stem + ".o") for s in SOURCES]
    if force or jobs or _stale(LIB, objs):
        tmp = LIB.with_suffix(f".so.{os.getpid()}.tmp")
        cmd = [_nvcc(), "-gencode", "arch=compute_100a,code=sm_100a", "-shared", "-o", str(tmp), *map(str, objs)]
        res = subprocess.run(cmd, capture_output=True, text=True)
        if res.returncode != 0:
            sys.stderr.write(res.stdout + res.stderr)
            raise RuntimeError("link failed")
        os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("-v", "--verbose", action="store_true")
    a = ap.parse_args()
    print(build(force=a.force, verbose=a.verbose))
