"""Builds libgrxcp.so (grxBLAS + grxDNN + the libgrxrt subset) in-tree.

Every CUDA source is compiled for sm_100a only
(``-gencode arch=compute_100a,code=sm_100a``); the CUDA runtime is linked
statically so the library loads without any LD_LIBRARY_PATH set-up, and the
driver is reached through cudaGetDriverEntryPoint, so loading the library
needs no libcuda.so (a CPU-only machine can load it and inspect its symbols).

Usage: ``python -m grxcp_b200.build`` (incremental; ``--force`` rebuilds).
"""
from __future__ import annotations

import concurrent.futures as cf
import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
BUILD = ROOT / "_build" / "grxcp"
LIB = PKG / "libgrxcp.so"

SOURCES = [
    "runtime.cpp",
    "host_common.cpp",
    "blas_host.cpp",
    "dnn_host.cpp",
    "gemm_tc.cu",
    "blas_kernels.cu",
    "norm.cu",
    "norm_bwd.cu",
    "attention.cu",
    "attention_bwd.cu",
    "gemm_noalloc.cu",
    "softmax.cu",
    "conv.cu",
    "profile.cpp",
    "shard.cpp",
]

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", shutil.which("nvcc")):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found (set $NVCC)")


def _flags() -> list[str]:
    return ARCH + [
        "-O3",
        "-std=c++17",
        "-lineinfo",
        "-Xcompiler",
        "-fPIC",
        "-I" + str(ROOT / "include"),
        "-I" + str(CSRC),
    ]


def _deps_mtime() -> float:
    hdrs = list(CSRC.glob("*.h")) + list(CSRC.glob("*.cuh")) + list((ROOT / "include" / "grx").glob("*.h"))
    return max([p.stat().st_mtime for p in hdrs] + [Path(__file__).stat().st_mtime])


def _compile(src: Path, obj: Path, force: bool) -> str:
    if not force and obj.exists() and obj.stat().st_mtime >= max(src.stat().st_mtime, _deps_mtime()):
        return f"up to date: {src.name}"
    cmd = [nvcc()] + _flags() + ["-c", str(src), "-o", str(obj)]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"compile failed: {src.name}\n{' '.join(cmd)}\n{r.stdout}\n{r.stderr}")
    return f"compiled: {src.name}"


def build(force: bool = False, verbose: bool = False) -> Path:
    BUILD.mkdir(parents=True, exist_ok=True)
    objs = []
    with cf.ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 2)) as ex:
        futs = []
        for s in SOURCES:
            src = CSRC / s
            obj = BUILD / (s + ".o")
            objs.append(obj)
            futs.append(ex.submit(_compile, src, obj, force))
        for f in futs:
            msg = f.result()
            if verbose:
                print(msg)
    if force or not LIB.exists() or LIB.stat().st_mtime < max(o.stat().st_mtime for o in objs):
        # Exported symbols: the extern "C" API only (sources build with hidden
        # visibility; the API is marked visible by the version script).
        vs = BUILD / "exports.map"
        vs.write_text("{ global: grx*; local: *; };\n")
        cmd = [nvcc()] + ARCH + ["-shared", "-cudart", "static", "-o", str(LIB)] + [str(o) for o in objs] + [
            "-Xlinker",
            f"--version-script={vs}",
            "-ldl",
            "-lpthread",
            "-lrt",
        ]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed\n{' '.join(cmd)}\n{r.stdout}\n{r.stderr}")
        if verbose:
            print(f"linked: {LIB}")
    return LIB


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose=True)
