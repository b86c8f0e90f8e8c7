"""Builds oracle/_ref/: the reference's own code compiled for this host, as a checker.

  libref_sgemm.so   the reference sgemm kernel source (src/libs/grxblas/kernels/
                    sgemm.cpp), compiled as host C++ against oracle/refshim (a stand-in
                    for the GRX-G100 device headers) and driven by ref_sgemm_driver.cpp.
  test_npu_c930     the reference's CPU-only NPU unit test (src/backends/npu_c930/
                    test_npu_c930.cc + npu_c930.cpp), whose int8 known-answer GEMMs pin
                    the oracle's int8 loop.

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
REF = Path(os.environ.get("GRXCP_REFERENCE", "/root/reference"))


def build(force: bool = False) -> bool:
    if not REF.exists():
        return False
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
    return True


if __name__ == "__main__":
    print(build(force=True))
