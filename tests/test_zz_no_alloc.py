"""grxblasGemmExNoAlloc against grxblasGemmEx, through the C-ABI.

grxblasGemmExNoAlloc serves callers that may not allocate device memory
(their device memory belongs to another allocator, or they must not trigger
cudaMalloc's implicit synchronisation). It packs unaligned operands into a
fixed array inside the library instead of a handle workspace. Here it must
produce what grxblasGemmEx produces on the same inputs (within the GEMM tests'
tolerance |d| <= 1e-2 + 2e-2*|ref|), on two calls in a row with different
shapes and types -- the second call must not see the first call's scratch --
and it must refuse a problem whose packing scratch exceeds the array.
This file is collected last so a stop-at-first-failure run has already run
every other test; it passes both alone and after them.
"""
import ctypes as C

import numpy as np
import pytest
import torch

from grxcp_b200 import _native as N
from grxcp_b200 import blas as B

pytestmark = pytest.mark.gpu

TOL_ABS, TOL_REL = 1e-2, 2e-2


def _f(v):
    return C.byref(C.c_float(v))


def _noalloc(ta, tb, m, n, k, alpha, A, at, lda, Bm, bt, ldb, beta, Cm, ct, ldc, err):
    return N.lib.grxblasGemmExNoAlloc(torch.cuda.current_stream().cuda_stream, ta, tb, m, n, k, _f(alpha),
                                      A.data_ptr(), at, lda, Bm.data_ptr(), bt, ldb, _f(beta), Cm.data_ptr(), ct,
                                      ldc, err.data_ptr())


def _close(got, ref):
    got = got.double().cpu().numpy()
    ref = ref.double().cpu().numpy()
    return np.all(np.abs(got - ref) <= TOL_ABS + TOL_REL * np.abs(ref))


def test_noalloc_matches_gemmex_on_two_calls_in_a_row():
    torch.cuda.set_device(0)
    g = torch.Generator(device="cuda").manual_seed(2024)
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    with B.Handle() as h:
        B.check(h.set_stream(torch.cuda.current_stream()))

        # Call 1: bf16 in/out, NN, odd lda (A must be packed), beta != 0.
        m, n, k, lda, ldb, ldc = 200, 136, 77, 201, 80, 208
        A = torch.randn(lda * k, device="cuda", generator=g).to(torch.bfloat16)
        Bm = torch.randn(ldb * n, device="cuda", generator=g).to(torch.bfloat16)
        C0 = torch.randn(ldc * n, device="cuda", generator=g).to(torch.bfloat16)
        c_ref, c_new = C0.clone(), C0.clone()
        assert h.gemm_ex(0, 0, m, n, k, 1.25, A, N.GRX_R_16BF, lda, Bm, N.GRX_R_16BF, ldb, -0.5, c_ref,
                         N.GRX_R_16BF, ldc) == N.SUCCESS
        assert _noalloc(0, 0, m, n, k, 1.25, A, N.GRX_R_16BF, lda, Bm, N.GRX_R_16BF, ldb, -0.5, c_new,
                        N.GRX_R_16BF, ldc, err) == N.SUCCESS
        torch.cuda.synchronize()
        assert _close(c_new, c_ref)
        assert torch.equal(c_new[m:ldc], C0[m:ldc]), "ld padding of C was written"

        # Call 2: fp16 in, fp32 out, TT, both operands packed (odd leading dimensions), a
        # different size than call 1 so stale scratch would show.
        m, n, k, lda, ldb, ldc = 129, 263, 150, 151, 265, 129
        A = torch.randn(lda * m, device="cuda", generator=g).to(torch.float16)
        Bm = torch.randn(ldb * k, device="cuda", generator=g).to(torch.float16)
        c_ref = torch.full((ldc * n,), float("nan"), device="cuda")
        c_new = torch.full((ldc * n,), float("nan"), device="cuda")
        assert h.gemm_ex(1, 1, m, n, k, 1.0, A, N.GRX_R_16F, lda, Bm, N.GRX_R_16F, ldb, 0.0, c_ref, N.GRX_R_32F,
                         ldc) == N.SUCCESS
        assert _noalloc(1, 1, m, n, k, 1.0, A, N.GRX_R_16F, lda, Bm, N.GRX_R_16F, ldb, 0.0, c_new, N.GRX_R_32F,
                        ldc, err) == N.SUCCESS
        torch.cuda.synchronize()
        assert not torch.isnan(c_new).any()
        assert _close(c_new, c_ref)
        assert h.execution_status() == N.SUCCESS
    assert int(err.item()) == 0, "a kernel reported a bounded-wait timeout"


def test_noalloc_refuses_problems_beyond_its_scratch():
    torch.cuda.set_device(0)
    small = torch.zeros(64, dtype=torch.bfloat16, device="cuda")
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    # A 8192 x 1024 bf16 operand with an odd lda needs 16 MiB of packing alone, plus B: over the limit.
    st = _noalloc(0, 0, 8192, 8192, 1024, 1.0, small, N.GRX_R_16BF, 8193, small, N.GRX_R_16BF, 1025, 0.0, small,
                  N.GRX_R_16BF, 8192, err)
    assert st == N.INVALID_VALUE


def _int8(shape, g):
    return torch.randint(-128, 128, shape, device="cuda", generator=g, dtype=torch.int32).to(torch.int8)


def _fp8(shape, g):
    return (torch.randn(shape, device="cuda", generator=g) * 0.5).to(torch.float8_e4m3fn)


# (Atype, Ctype, make operand, make C, bit-exact?) -- the 8-bit pairings grxblasGemmEx accepts.
_EIGHT_BIT = [
    ("i8->s32", N.GRX_R_8I, N.GRX_R_32I, _int8, torch.int32, True),
    ("i8->bf16", N.GRX_R_8I, N.GRX_R_16BF, _int8, torch.bfloat16, False),
    ("i8->f32", N.GRX_R_8I, N.GRX_R_32F, _int8, torch.float32, False),
    ("e4m3->bf16", N.GRX_R_8F_E4M3, N.GRX_R_16BF, _fp8, torch.bfloat16, False),
    ("e4m3->f32", N.GRX_R_8F_E4M3, N.GRX_R_32F, _fp8, torch.float32, False),
]


@pytest.mark.parametrize("name,at,ct,make,cdt,exact", _EIGHT_BIT, ids=[c[0] for c in _EIGHT_BIT])
def test_noalloc_eight_bit_pairings_match_gemmex(name, at, ct, make, cdt, exact):
    torch.cuda.set_device(0)
    g = torch.Generator(device="cuda").manual_seed(7)
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    # TN with an odd lda (A packed) and an aligned B; beta = 2 exercises the C read.
    m, n, k, lda, ldb, ldc = 192, 160, 200, 203, 208, 200
    A = make((lda * m,), g)
    Bm = make((ldb * n,), g)
    C0 = (torch.randint(-50, 50, (ldc * n,), device="cuda", generator=g)).to(cdt)
    c_ref, c_new = C0.clone(), C0.clone()
    alpha, beta = 3.0, 2.0
    with B.Handle() as h:
        B.check(h.set_stream(torch.cuda.current_stream()))
        assert h.gemm_ex(1, 0, m, n, k, alpha, A, at, lda, Bm, at, ldb, beta, c_ref, ct, ldc) == N.SUCCESS
        for _ in range(2):  # twice: the second call reuses the scratch the first call left behind
            c_new.copy_(C0)
            assert _noalloc(1, 0, m, n, k, alpha, A, at, lda, Bm, at, ldb, beta, c_new, ct, ldc, err) == N.SUCCESS
            torch.cuda.synchronize()
            if exact:
                assert torch.equal(c_new, c_ref)
            else:
                assert _close(c_new, c_ref)
        assert h.execution_status() == N.SUCCESS
    assert int(err.item()) == 0
    # non-integer alpha is refused for the exact int32 output only
    st = _noalloc(1, 0, m, n, k, 0.5, A, at, lda, Bm, at, ldb, beta, c_new, ct, ldc, err)
    assert st == (N.INVALID_VALUE if ct == N.GRX_R_32I else N.SUCCESS)
    torch.cuda.synchronize()


def test_noalloc_k_zero_scales_c_like_gemmex():
    torch.cuda.set_device(0)
    g = torch.Generator(device="cuda").manual_seed(11)
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    m, n, ldc = 70, 33, 72
    C0 = torch.randn(ldc * n, device="cuda", generator=g)
    c_ref, c_new = C0.clone(), C0.clone()
    dummy = torch.zeros(16, dtype=torch.bfloat16, device="cuda")
    with B.Handle() as h:
        B.check(h.set_stream(torch.cuda.current_stream()))
        assert h.gemm_ex(0, 0, m, n, 0, 1.0, dummy, N.GRX_R_16BF, m, dummy, N.GRX_R_16BF, 1, -1.5, c_ref,
                         N.GRX_R_32F, ldc) == N.SUCCESS
    assert _noalloc(0, 0, m, n, 0, 1.0, dummy, N.GRX_R_16BF, m, dummy, N.GRX_R_16BF, 1, -1.5, c_new, N.GRX_R_32F,
                    ldc, err) == N.SUCCESS
    torch.cuda.synchronize()
    assert torch.equal(c_new, c_ref)


def test_noalloc_takes_no_device_memory():
    """The point of the entry point: after its first call on a device, further calls
    (packing included) leave the device's free memory exactly where it was."""
    torch.cuda.set_device(0)
    g = torch.Generator(device="cuda").manual_seed(5)
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    m, n, k, lda, ldb, ldc = 300, 520, 333, 301, 335, 300
    A = torch.randn(lda * k, device="cuda", generator=g).to(torch.bfloat16)
    Bm = torch.randn(ldb * n, device="cuda", generator=g).to(torch.bfloat16)
    Cm = torch.empty(ldc * n, device="cuda", dtype=torch.bfloat16)
    assert _noalloc(0, 0, m, n, k, 1.0, A, N.GRX_R_16BF, lda, Bm, N.GRX_R_16BF, ldb, 0.0, Cm, N.GRX_R_16BF, ldc,
                    err) == N.SUCCESS
    torch.cuda.synchronize()
    free0, _ = torch.cuda.mem_get_info()
    for _ in range(3):
        assert _noalloc(0, 0, m, n, k, 1.0, A, N.GRX_R_16BF, lda, Bm, N.GRX_R_16BF, ldb, 0.0, Cm, N.GRX_R_16BF,
                        ldc, err) == N.SUCCESS
    torch.cuda.synchronize()
    free1, _ = torch.cuda.mem_get_info()
    assert free1 == free0, f"device free memory moved by {free0 - free1} bytes across no-alloc calls"
