"""Generates tests/golden/ref_sgemm.npz from the reference's own sgemm kernel.

The reference's sgemm kernel source (src/libs/grxblas/kernels/sgemm.cpp) is
compiled for this host by oracle/build_ref.py into oracle/_ref/libref_sgemm.so;
this script runs it on the reference's gate cases (tests/libs/test_grxblas.cpp
:306-331, LCG fills :190-195) and stores every output C buffer. It needs the
reference tree, so it runs in the build container; the fixture is committed.

    python tests/golden/make_golden.py
"""
import ctypes as C
import sys
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(ROOT))
sys.path.insert(0, str(ROOT / "tests"))

from gates import SGEMM_BATCHED_CASES, SGEMM_CASES, lcg_fill  # noqa: E402
from oracle import build_ref  # noqa: E402


def main():
    assert build_ref.build(), "reference tree not available"
    lib = C.CDLL(str(ROOT / "oracle/_ref/libref_sgemm.so"))
    f = lib.ref_sgemm_run
    vp, i, ll, fl = C.c_void_p, C.c_int, C.c_longlong, C.c_float
    f.argtypes = [i, i, i, i, i, fl, vp, i, ll, vp, i, ll, fl, vp, i, ll, i]
    out = {}
    for ta, tb, m, n, k, alpha, beta, pad, label in SGEMM_CASES:
        lda, ldb, ldc = max(1, (k if ta else m) + pad), max(1, (n if tb else k) + pad), max(1, m + pad)
        A = lcg_fill(lda * (m if ta else k), 1)
        B = lcg_fill(ldb * (k if tb else n), 7)
        Cb = lcg_fill(ldc * n, 13)
        Ab = A if A.size else np.zeros(1, np.float32)
        Bb = B if B.size else np.zeros(1, np.float32)
        f(ta, tb, m, n, k, alpha, Ab.ctypes.data, lda, 0, Bb.ctypes.data, ldb, 0, beta, Cb.ctypes.data, ldc, 0, 1)
        out["single/" + label] = Cb
    for ta, tb, m, n, k, alpha, beta, batch, gap, bcast, label in SGEMM_BATCHED_CASES:
        lda, ldb, ldc = max(1, k if ta else m), max(1, n if tb else k), max(1, m)
        ae, be, ce = lda * (m if ta else k), ldb * (k if tb else n), ldc * n
        sa, sb, sc = ae + gap, 0 if bcast else be + gap, ce + gap
        A = lcg_fill(sa * (batch - 1) + ae + gap, 3)
        B = lcg_fill(be + gap if bcast else sb * (batch - 1) + be + gap, 11)
        Cb = lcg_fill(sc * (batch - 1) + ce + gap, 17)
        f(ta, tb, m, n, k, alpha, A.ctypes.data, lda, sa, B.ctypes.data, ldb, sb, beta, Cb.ctypes.data, ldc, sc,
          batch)
        out["batched/" + label] = Cb
    np.savez_compressed(ROOT / "tests/golden/ref_sgemm.npz", **out)
    print(f"wrote {len(out)} cases")


if __name__ == "__main__":
    main()
