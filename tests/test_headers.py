"""The drop-in headers, on the CPU: include/grx compiles as C and C++ for a
reference-style caller, grxCycleSummarize follows the reference's summary rules
(include/grx/grx_cycles.h:67-99 of the reference), and the reference's gate
programs built against these headers link to libgrxcp.so and report "no
device" (exit 77) on a machine without a GPU."""
from __future__ import annotations

import shutil
import subprocess
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
INC = ROOT / "include"

CALLER = r"""
#include <grx/grx.h>
#include <grx/grxblas.h>
#include <grx/grxdnn.h>
#include <grx/grx_cycles.h>
int main(void) {
  grxTensorMapDesc_t d;
  grxCycleSlot s;
  (void)d; (void)s;
  return (int)GRXBLAS_STATUS_SUCCESS + (int)grxTensorMapLayoutKMajor - 1;
}
"""

SUMMARY = r"""
#include <grx/grx_cycles.h>
#include <cstdio>
int main() {
  grxCycleSlot one_sm[4] = {{100, 160, 3, 0}, {0, 0, 0, 1}, {110, 140, 3, 2}, {105, 200, 3, 3}};
  grxCycleSummary s;
  grxCycleSummarize(one_sm, 4, &s);
  std::printf("%d %d %d %llu %llu %llu %llu\n", s.warps, s.cores, s.spanIsValid, (unsigned long long)s.span,
              (unsigned long long)s.busyMin, (unsigned long long)s.busyMedian, (unsigned long long)s.busyMax);
  grxCycleSlot two_sm[2] = {{100, 160, 3, 0}, {90, 170, 4, 1}};
  grxCycleSummarize(two_sm, 2, &s);
  std::printf("%d %d %d %llu\n", s.warps, s.cores, s.spanIsValid, (unsigned long long)s.span);
  grxCycleSummarize(nullptr, 3, &s);
  std::printf("%d %d\n", s.warps, s.spanIsValid);
  return 0;
}
"""


def _cc(tmp_path, compiler, src, suffix, extra=()):
    if shutil.which(compiler) is None:
        pytest.skip(f"{compiler} not available")
    f = tmp_path / f"t{suffix}"
    f.write_text(src)
    exe = tmp_path / "t.out"
    subprocess.run([compiler, "-I", str(INC), str(f), "-o", str(exe), *extra], check=True, capture_output=True)
    return exe


def test_headers_compile_as_c_and_cpp(tmp_path):
    for compiler, suffix, std in (("gcc", ".c", "-std=c99"), ("g++", ".cpp", "-std=c++17")):
        exe = _cc(tmp_path, compiler, CALLER, suffix, ["-c", "-o", str(tmp_path / "t.o"), std])
        assert (tmp_path / "t.o").exists(), exe


def test_cycle_summary_rules(tmp_path):
    exe = _cc(tmp_path, "g++", SUMMARY, ".cpp", ["-std=c++17"])
    out = subprocess.run([str(exe)], check=True, capture_output=True, text=True).stdout.split("\n")
    # 3 written slots on SM 3 (the all-zero one skipped): span 200 - 100, busy {60, 30, 95}
    assert out[0].split() == ["3", "1", "1", "100", "30", "60", "95"]
    # two SMs: no span
    assert out[1].split() == ["2", "2", "0", "0"]
    assert out[2].split() == ["0", "0"]


@pytest.mark.parametrize("name", ["test_grxblas", "test_grxblas_ex", "test_grxblas_l12", "gemm_cycles"])
def test_reference_gate_programs_report_no_device(name):
    import torch

    if torch.cuda.is_available():
        pytest.skip("a GPU is present: tests/test_ref_gates_gpu.py runs these for real")
    exe = ROOT / "oracle" / "_ref" / name
    if not exe.exists():
        pytest.skip("built only where the reference tree is present")
    r = subprocess.run([str(exe)], capture_output=True, text=True, timeout=60)
    assert r.returncode == 77 and "no devices" in r.stdout, r.stdout + r.stderr
