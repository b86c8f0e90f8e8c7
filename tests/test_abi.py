"""CPU checks of the C-ABI boundary: the library loads without a GPU, exports
every function include/grx/*.h declares, and the host-side validation refuses
bad arguments exactly as the reference does -- these refusals happen before
any device is touched (reference src/libs/grxblas/grxblas.cpp:506-524,
:882-897; tests/libs/test_grxblas.cpp:349-367, test_grxblas_ex.cpp:345-371)."""
from __future__ import annotations

import ctypes as C
import re
import subprocess
from pathlib import Path

import pytest

from grxcp_b200 import _native as N
from grxcp_b200 import blas as B
from grxcp_b200 import dnn as D

ROOT = Path(__file__).resolve().parent.parent


def header_functions() -> set[str]:
    names = set()
    for h in sorted((ROOT / "include" / "grx").glob("*.h")):
        text = h.read_text()
        text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
        text = re.sub(r"//[^\n]*", "", text)
        text = "\n".join(l for l in text.splitlines() if not l.lstrip().startswith("#"))
        # header-only inline helpers (grxCycleSummarize) are not library symbols
        text = re.sub(r"\binline\b.*", "", text, flags=re.S)
        for m in re.finditer(r"\b(grx\w*)\s*\(", text):
            names.add(m.group(1))
    return names


def test_every_header_function_is_exported_and_bound():
    names = header_functions()
    assert len(names) > 60
    out = subprocess.run(["nm", "-D", "--defined-only", str(N.LIB_PATH)], capture_output=True, text=True,
                         check=True).stdout
    exported = {l.split()[-1] for l in out.splitlines() if l.strip()}
    missing = names - exported
    assert not missing, f"declared but not exported: {sorted(missing)}"
    assert names == set(N.PROTOTYPES), (sorted(names - set(N.PROTOTYPES)), sorted(set(N.PROTOTYPES) - names))
    # nothing but the C API (plus the one internal test hook) leaks out
    assert exported - names <= {"grxcpTestBoundedWait"}


def test_library_has_no_cuda_shared_dependency():
    out = subprocess.run(["ldd", str(N.LIB_PATH)], capture_output=True, text=True).stdout
    assert "libcuda" not in out and "libcudart" not in out


def test_status_strings():
    for s in range(8):
        assert N.lib.grxblasGetStatusString(s)
        assert N.lib.grxdnnGetStatusString(s)
    assert N.lib.grxGetErrorString(0) == b"no error"
    assert N.lib.grxGetErrorName(15) == b"grxErrorTimeout"


def test_enum_values_match_reference():
    # include/grx/grx_types.h:120-134 and CUDA's numbering for the additive types
    assert (N.GRX_R_32F, N.GRX_R_16F, N.GRX_R_8I, N.GRX_R_32I, N.GRX_R_16BF, N.GRX_R_8F_E4M3) == (0, 2, 3, 10, 14, 28)


@pytest.fixture()
def h():
    hh = B.Handle()
    yield hh
    hh.close()


def test_null_handle_is_not_initialized():
    one = C.byref(C.c_float(1.0))
    assert N.lib.grxblasSgemm(None, 0, 0, 4, 4, 4, one, 1, 4, 1, 4, one, 1, 4) == N.NOT_INITIALIZED
    assert N.lib.grxblasGemmEx(None, 0, 0, 8, 4, 8, one, 1, N.GRX_R_16F, 8, 1, N.GRX_R_16F, 8, one, 1, N.GRX_R_32F,
                               8) == N.NOT_INITIALIZED
    assert N.lib.grxblasDestroy(None) == N.NOT_INITIALIZED
    assert N.lib.grxblasSetStream(None, None) == N.NOT_INITIALIZED
    assert N.lib.grxblasSaxpy(None, 4, one, 1, 1, 1, 1) == N.NOT_INITIALIZED
    assert N.lib.grxdnnRMSNormForward(None, 1, 1, 1, N.GRX_R_16BF, 1, 1, 1e-5, 1, N.GRX_R_16BF, 1,
                                      None) == N.NOT_INITIALIZED
    assert N.lib.grxblasCreate(None) == N.INVALID_VALUE


def test_sgemm_validation(h):
    d = 1 << 20  # any non-null address: validation returns before it is touched
    assert h.sgemm(0, 0, 4, 4, 4, 1.0, d, 2, d, 4, 0.0, d, 4) == N.INVALID_VALUE  # lda < m
    assert h.sgemm(0, 0, 4, 4, 4, 1.0, d, 4, d, 4, 0.0, d, 1) == N.INVALID_VALUE  # ldc < m
    assert h.sgemm(1, 0, 4, 4, 8, 1.0, d, 4, d, 8, 0.0, d, 4) == N.INVALID_VALUE  # transposed A: lda >= k
    assert h.sgemm(0, 0, 0, 4, 4, 1.0, d, 4, d, 4, 0.0, d, 4) == N.SUCCESS  # empty problem
    assert h.sgemm(0, 0, 4, 0, 4, 1.0, d, 4, d, 4, 0.0, d, 4) == N.SUCCESS
    assert h.sgemm(0, 0, -1, 4, 4, 1.0, d, 4, d, 4, 0.0, d, 4) == N.INVALID_VALUE
    assert h.sgemm(0, 0, 4, 4, 4, None, d, 4, d, 4, 0.0, d, 4) == N.INVALID_VALUE  # null alpha
    assert h.sgemm(0, 0, 4, 4, 4, 1.0, None, 4, d, 4, 0.0, d, 4) == N.INVALID_VALUE  # null A with k > 0
    assert h.sgemm(0, 0, 4, 4, 4, 1.0, d, 4, d, 4, 0.0, None, 4) == N.INVALID_VALUE  # null C
    assert h.sgemm_strided_batched(0, 0, 4, 4, 4, 1.0, d, 4, 16, d, 4, 16, 0.0, d, 4, 16, 0) == N.SUCCESS
    assert h.sgemm_strided_batched(0, 0, 4, 4, 4, 1.0, d, 4, 16, d, 4, 16, 0.0, d, 4, 16, -1) == N.INVALID_VALUE


def test_gemmex_validation(h):
    d = 1 << 20
    # lda bounds k when A is transposed (test_grxblas_ex.cpp:349-352)
    assert h.gemm_ex(1, 0, 4, 4, 8, 1.0, d, N.GRX_R_16F, 4, d, N.GRX_R_16F, 8, 0.0, d, N.GRX_R_32F, 4) == \
        N.INVALID_VALUE
    assert h.gemm_ex(0, 0, 8, 4, 8, 1.0, d, N.GRX_R_16F, 2, d, N.GRX_R_16F, 8, 0.0, d, N.GRX_R_32F, 8) == \
        N.INVALID_VALUE
    assert h.gemm_ex(0, 1, 8, 4, 8, 1.0, d, N.GRX_R_16F, 8, d, N.GRX_R_16F, 2, 0.0, d, N.GRX_R_32F, 8) == \
        N.INVALID_VALUE  # transposed B: ldb >= n
    assert h.gemm_ex(0, 0, 0, 4, 8, 1.0, d, N.GRX_R_16F, 8, d, N.GRX_R_16F, 8, 0.0, d, N.GRX_R_32F, 8) == N.SUCCESS
    assert h.gemm_ex(0, 0, 8, 4, 8, None, d, N.GRX_R_16F, 8, d, N.GRX_R_16F, 8, 0.0, d, N.GRX_R_32F, 8) == \
        N.INVALID_VALUE
    assert h.gemm_strided_batched_ex(0, 0, 8, 4, 8, 1.0, d, N.GRX_R_16BF, 8, 64, d, N.GRX_R_16BF, 8, 32, 0.0, d,
                                     N.GRX_R_16BF, 8, 32, -1) == N.INVALID_VALUE
    assert h.gemm_strided_batched_ex(0, 0, 8, 4, 8, 1.0, d, N.GRX_R_16BF, 8, 64, d, N.GRX_R_16BF, 8, 32, 0.0, d,
                                     N.GRX_R_16BF, 8, 32, 0) == N.SUCCESS


def test_level12_validation(h):
    d = 1 << 20
    assert h.saxpy(4, 1.0, d, 0, d, 1) == N.INVALID_VALUE  # zero increment refused
    assert h.saxpy(0, 1.0, d, 1, d, 1) == N.SUCCESS
    assert h.saxpy(-1, 1.0, d, 1, d, 1) == N.INVALID_VALUE
    assert h.sscal(4, 1.0, d, -1) == N.INVALID_VALUE  # scal needs incx > 0
    assert h.sgemv(0, 4, 4, 1.0, d, 2, d, 1, 0.0, d, 1) == N.INVALID_VALUE  # lda < m
    assert h.sgemv(0, 0, 4, 1.0, d, 4, d, 1, 0.0, d, 1) == N.SUCCESS


def test_handle_state(h):
    assert h.set_tensor_map_slots(2, 3) == N.SUCCESS
    assert h.set_tensor_map_slots(2, 2) == N.INVALID_VALUE
    assert h.set_tensor_map_slots(-1, 3) == N.INVALID_VALUE
    assert h.set_tensor_map_slots(0, 16) == N.INVALID_VALUE
    assert h.set_stream(0x1234) == N.SUCCESS
    assert h.get_stream() == 0x1234
    assert h.set_stream(None) == N.SUCCESS
    assert h.set_cycle_probe(0x1000, 0) == N.INVALID_VALUE
    assert h.set_cycle_probe(None, 0) == N.SUCCESS
    assert h.set_epilogue(scale_mode=7) == N.INVALID_VALUE
    assert h.set_epilogue(bias=0x1000, bias_type=N.GRX_R_32F) == N.SUCCESS
    assert h.clear_epilogue() == N.SUCCESS
    assert h.loaded_kernel_path() is None  # nothing launched yet
    assert B.cycle_slots_needed(256, 256) == 64  # sgemm at 32 x 32 tiles (no 148-CTA grid at 128 or 64)
    assert h.set_workspace(0x1001, 100) == N.INVALID_VALUE  # workspace must be 256-byte aligned


def test_dnn_validation():
    with D.Handle() as h:
        d = 1 << 20
        R = N.lib.grxdnnRMSNormForward
        assert R(h.h, 0, 8, d, N.GRX_R_16BF, 8, d, 1e-5, d, N.GRX_R_16BF, 8, None) == N.SUCCESS
        assert R(h.h, -1, 8, d, N.GRX_R_16BF, 8, d, 1e-5, d, N.GRX_R_16BF, 8, None) == N.INVALID_VALUE
        assert R(h.h, 4, 8, d, N.GRX_R_16BF, 4, d, 1e-5, d, N.GRX_R_16BF, 8, None) == N.INVALID_VALUE
        assert R(h.h, 4, 8, d, N.GRX_R_16BF, 8, d, -1.0, d, N.GRX_R_16BF, 8, None) == N.INVALID_VALUE
        assert R(h.h, 4, 8, d, N.GRX_R_16BF, 8, d, 1e-5, d, N.GRX_R_16F, 8, None) == N.NOT_SUPPORTED
        assert R(h.h, 4, 8, d, N.GRX_R_8I, 8, d, 1e-5, d, N.GRX_R_8I, 8, None) == N.NOT_SUPPORTED
        dq = D.attn_desc(None, 1, 1, 128, 128)
        bad = D.attn_desc(None, 1, 1, 128, 128)
        bad.strideSeq = 64
        A = N.lib.grxdnnAttentionForward
        assert A(h.h, C.byref(bad), d, C.byref(dq), d, C.byref(dq), d, C.byref(dq), d, 0.1, 1, None) == \
            N.INVALID_VALUE
        z = D.attn_desc(None, 0, 1, 128, 128)
        assert A(h.h, C.byref(z), d, C.byref(z), d, C.byref(z), d, C.byref(z), d, 0.1, 1, None) == N.SUCCESS
        assert A(h.h, C.byref(dq), d, C.byref(dq), d, C.byref(dq), d, C.byref(dq), d, 0.0, 1, None) == \
            N.INVALID_VALUE
        dk = D.attn_desc(None, 1, 1, 256, 128)
        assert A(h.h, C.byref(dq), d, C.byref(dk), d, C.byref(dk), d, C.byref(dq), d, 0.1, 1, None) == \
            N.NOT_SUPPORTED  # causal needs equal lengths


def test_kernel_path_rule(tmp_path):
    # A configured path that is not this library refuses (no fallback past it).
    with B.Handle() as h:
        try:
            assert B.set_kernel_path(str(tmp_path)) == N.SUCCESS
            st, _ = h.tensor_types()
            assert st == N.NOT_INITIALIZED
        finally:
            B.set_kernel_path(None)
