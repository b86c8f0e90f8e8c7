"""Builds oracle/_ref/: the reference's own code compiled for this host, as a checker.

  libref_sgemm.so   the reference sgemm kernel source (src/libs/grxblas/kernels/
                    sgemm.cpp), compiled as host C++ against oracle/refshim (a stand-in
                    for the GRX-G100 device headers) and driven by ref_sgemm_driver.cpp.
  test_npu_c930     the reference's CPU-only NPU unit test (src/backends/npu_c930/
                    test_npu_c930.cc + npu_c930.cpp), whose int8 known-answer GEMMs pin
                    the oracle's int8 loop.
  test_grxblas, test_grxblas_ex, test_grxblas_l12, gemm_cycles
                    the reference's own grxBLAS gate programs (tests/libs/*.cpp,
                    tests/bench/gemm_cycles.cpp), compiled UNMODIFIED against this
                    repository's include/ and linked to grxcp_b200/libgrxcp.so: the
                    drop-in check, run on a B200 by tests/test_ref_gates_gpu.py.

Sources are compiled where they lie under the reference tree (read-only); outputs go
to oracle/_ref only. Needs the reference tree, so it runs in the build container; the
built files travel with the repository snapshot. TEST INFRASTRUCTURE ONLY.
"""
from __future__ import annotations

import os
import subprocess
from pathlib import Path

HERE = Path(__file__).resolve().parent
OUT = HERE / "_ref"
ROOT = HERE.parent

# The reference's gate programs: (source under the reference tree, output name).
GATES = [
    ("tests/libs/test_grxblas.cpp", "test_grxblas"),
    ("tests/libs/test_grxblas_ex.cpp", "test_grxblas_ex"),
    ("tests/libs/test_grxblas_l12.cpp", "test_grxblas_l12"),
    ("tests/bench/gemm_cycles.cpp", "gemm_cycles"),
]


def _gate_programs(ref: Path, force: bool) -> None:
    lib = ROOT / "grxcp_b200" / "libgrxcp.so"
    if not lib.exists():
        return
    for src, name in GATES:
        out = OUT / name
        if not force and out.exists() and out.stat().st_mtime >= lib.stat().st_mtime:
            continue
        # This repository's include/ comes first, so <grx/grx.h> and <grx/grxblas.h>
        # resolve to the drop-in headers; the programs' relative includes
        # ("../unit/grx_test.h", "../common/fp16.h") resolve beside their source.
        cmd = ["g++", "-O1", "-std=c++17", "-I", str(ROOT / "include"), str(ref / src), "-o", str(out),
               "-L", str(lib.parent), "-lgrxcp", "-Wl,-rpath,$ORIGIN/../../grxcp_b200"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"reference gate program {src} does not build against include/:\n{r.stdout}{r.stderr}")


def build(force: bool = False, ref: str | None = None) -> bool:
    """Builds oracle/_ref from the reference tree at `ref` (or $GRXCP_REFERENCE);
    returns False, building nothing, when neither names an existing directory."""
    ref = ref or os.environ.get("GRXCP_REFERENCE")
    if not ref or not Path(ref).is_dir():
        return False
    REF = Path(ref)
    OUT.mkdir(exist_ok=True)
    kernel = REF / "src/libs/grxblas/kernels/sgemm.cpp"
    lib = OUT / "libref_sgemm.so"
    if force or not lib.exists():
        subprocess.run(["g++", "-O2", "-std=c++17", "-fPIC", "-shared", "-ffp-contract=off",
                        "-I", str(HERE / "refshim"), "-I", str(REF / "src/libs/grxblas"),
                        str(kernel), str(HERE / "ref_sgemm_driver.cpp"), "-o", str(lib)], check=True)
    npu = OUT / "test_npu_c930"
    npu_dir = REF / "src/backends/npu_c930"
    if force or not npu.exists():
        r = subprocess.run(["g++", "-O1", "-std=c++17", "-I", str(npu_dir), str(npu_dir / "test_npu_c930.cc"),
                            str(npu_dir / "npu_c930.cpp"), "-o", str(npu)], capture_output=True, text=True)
        if r.returncode != 0:
            (OUT / "test_npu_c930.build.log").write_text(r.stdout + r.stderr)
    _gate_programs(REF, force)
    return True


if __name__ == "__main__":
    import sys

    print(build(force=True, ref=sys.argv[1] if len(sys.argv) > 1 else None))
