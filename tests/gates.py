"""Test-data generators and case lists of the reference's grxBLAS gates.

Each generator restates one fill of kubeworkz/grxcp's tests (cited) so the
parity tests run the same inputs through this library and through the oracle.
"""
from __future__ import annotations

import numpy as np


def lcg_fill(n: int, seed: int) -> np.ndarray:
    """tests/libs/test_grxblas.cpp:190-195: seed = seed*1664525 + 1013904223,
    v = ((int)(seed >> 16) % 17 - 8) * 0.25 -- a mix of signs and magnitudes."""
    out = np.empty(n, np.float32)
    s = seed & 0xFFFFFFFF
    for i in range(n):
        s = (s * 1664525 + 1013904223) & 0xFFFFFFFF
        out[i] = np.float32(((s >> 16) % 17 - 8) * 0.25)
    return out


class HalfSampler:
    """tests/libs/test_grxblas_ex.cpp:33-36: multiples of 0.5 in [-4, 4], each exact in
    fp16 (and bf16), one running seed across A, B and C."""

    def __init__(self, seed: int = 99):
        self.s = seed & 0xFFFFFFFF

    def take(self, n: int) -> np.ndarray:
        out = np.empty(n, np.float32)
        s = self.s
        for i in range(n):
            s = (s * 1664525 + 1013904223) & 0xFFFFFFFF
            out[i] = np.float32((((s >> 16) % 17) - 8) * 0.5)
        self.s = s
        return out


def int8_patterns(na: int, nb: int, nc: int):
    """tests/libs/test_grxblas_ex.cpp:263-265."""
    i = np.arange(na, dtype=np.int64)
    A = ((i * 7 % 15) - 7).astype(np.int8)
    j = np.arange(nb, dtype=np.int64)
    B = ((j * 5 % 13) - 6).astype(np.int8)
    c = np.arange(nc, dtype=np.int64)
    C = ((c * 3 % 41) - 20).astype(np.int32)
    return A, B, C


# tests/libs/test_grxblas.cpp:306-317 -- (ta, tb, m, n, k, alpha, beta, pad, label)
SGEMM_CASES = [
    (0, 0, 4, 4, 4, 1.0, 0.0, 0, "4x4x4 NN alpha=1 beta=0"),
    (0, 0, 8, 5, 3, 1.0, 0.0, 0, "8x5x3 NN rectangular"),
    (0, 0, 7, 6, 5, 2.5, -1.5, 0, "7x6x5 NN alpha/beta"),
    (1, 0, 6, 4, 5, 1.0, 0.0, 0, "6x4x5 TN transpose A"),
    (0, 1, 5, 7, 4, 1.0, 0.0, 0, "5x7x4 NT transpose B"),
    (1, 1, 4, 5, 6, 1.0, 0.5, 0, "4x5x6 TT both"),
    (0, 0, 16, 16, 16, 1.0, 0.0, 0, "16x16x16 NN"),
    (1, 1, 16, 16, 16, 1.0, 0.0, 0, "16x16x16 TT"),
    (0, 0, 1, 1, 9, 1.0, 0.0, 0, "1x1x9 degenerate"),
    (0, 0, 5, 4, 6, 1.0, 0.0, 3, "5x4x6 NN padded ld"),
    (1, 1, 6, 5, 4, 2.0, -1.0, 2, "6x5x4 TT padded ld"),
    (0, 0, 4, 3, 0, 1.0, 2.0, 0, "4x3x0 k=0 scales C by beta"),
]

# tests/libs/test_grxblas.cpp:323-331 -- (ta, tb, m, n, k, alpha, beta, batch, gap, broadcast_b, label)
SGEMM_BATCHED_CASES = [
    (0, 0, 6, 5, 4, 1.0, 0.0, 3, 0, False, "3 matrices, tight strides"),
    (0, 0, 6, 5, 4, 2.0, -1.0, 4, 7, False, "4 matrices, slack between them, alpha and beta"),
    (0, 0, 6, 5, 4, 1.0, 0.0, 3, 5, True, "strideB = 0 broadcasts one B across the batch"),
    (1, 1, 5, 4, 6, 1.0, 0.5, 3, 3, False, "transposed operands, batched"),
    (0, 0, 7, 3, 5, 1.0, 0.0, 1, 4, False, "batchCount = 1 is the unbatched path"),
]


def gemmex_cases(tm: int, tn: int, tk: int):
    """tests/libs/test_grxblas_ex.cpp:209-241 -- (ta, tb, m, n, k, alpha, beta, pad, label),
    with the tile (tm, tn, tk) this device reports."""
    cases = [
        (0, 0, tm, tn, tk, 1.0, 0.0, 0, "exactly one tile, one k step"),
        (0, 0, tm * 2, tn * 2, tk * 2, 1.0, 0.0, 0, "four tiles, two k steps"),
        (0, 0, 16, 16, 16, 1.0, 0.0, 0, "16x16x16"),
        (0, 0, 5, 3, 7, 1.0, 0.0, 0, "5x3x7 every dimension ragged"),
        (0, 0, 17, 9, 13, 1.0, 0.0, 0, "17x9x13 ragged and larger"),
        (0, 0, 1, 1, 1, 1.0, 0.0, 0, "1x1x1"),
        (0, 0, 12, 6, 10, 2.5, -1.5, 0, "alpha and beta"),
        (0, 0, 12, 6, 10, 1.0, 0.0, 3, "padded leading dimensions"),
        (0, 0, 6, 5, 0, 1.0, 2.0, 0, "k = 0 scales C by beta"),
    ]
    for which in range(3):
        ta, tb = int(which != 1), int(which != 0)
        nm = "TT" if ta and tb else ("TN" if ta else "NT")
        cases += [
            (ta, tb, tm, tn, tk, 1.0, 0.0, 0, f"{nm} exactly one tile"),
            (ta, tb, tm * 2, tn * 2, tk * 2, 1.0, 0.0, 0, f"{nm} four tiles, two k steps"),
            (ta, tb, 5, 3, 7, 1.0, 0.0, 0, f"{nm} 5x3x7 ragged"),
            (ta, tb, 17, 9, 13, 1.0, 0.0, 0, f"{nm} 17x9x13 ragged and larger"),
            (ta, tb, 12, 6, 10, 2.5, -1.5, 3, f"{nm} alpha, beta and padded lds"),
        ]
    return cases


def int8_cases(tm: int, tn: int):
    """tests/libs/test_grxblas_ex.cpp:325-331 -- (ta, tb, m, n, k, alpha, beta, pad, label)."""
    return [
        (0, 0, tm, tn, 16, 1.0, 0.0, 0, "one tile, one k step"),
        (0, 0, 16, 16, 32, 1.0, 0.0, 0, "16x16x32"),
        (0, 0, 5, 3, 7, 1.0, 0.0, 0, "5x3x7 ragged, k < the tile depth"),
        (0, 0, 17, 9, 29, 2.0, -1.0, 3, "17x9x29 ragged, alpha/beta, padded lds"),
        (1, 0, 13, 7, 19, 1.0, 0.0, 0, "TN"),
        (0, 1, 13, 7, 19, 1.0, 0.0, 0, "NT"),
        (1, 1, 13, 7, 19, 1.0, 1.0, 0, "TT with beta"),
    ]


def storage_shape(trans: int, rows: int, cols: int):
    """Stored (rows, cols) of an operand whose op() is rows x cols."""
    return (cols, rows) if trans else (rows, cols)
