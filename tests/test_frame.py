"""The mapping from wgblas's layouts onto the column-major C-ABI frame
(wgblas_b200.gemm.to_column_major_frame, the twin of src/sgemm/sgemm.mjs:151-167)
computes the same product as the reference's own per-layout semantics
(tests/sgemm/helpers.js:8-16). CPU only, with the oracle as the column-major GEMM."""
from __future__ import annotations

import itertools

import numpy as np


def _ref_elem(M, ld, layout, trans, r, c):
    sr, sc = (c, r) if trans == "transpose" else (r, c)
    return M[sc * ld + sr] if layout == "column-major" else M[sr * ld + sc]


def test_all_layout_and_trans_combinations(wg, oracle):
    rng = np.random.default_rng(3)
    m, n, k = 5, 4, 3
    for la, lb, lc in itertools.product(("row-major", "column-major"), repeat=3):
        for ta, tb in itertools.product(("no-transpose", "transpose"), repeat=2):
            a_rows, a_cols = (m, k) if ta == "no-transpose" else (k, m)
            b_rows, b_cols = (k, n) if tb == "no-transpose" else (n, k)
            lda = (a_cols if la == "row-major" else a_rows) + 1
            ldb = (b_cols if lb == "row-major" else b_rows) + 2
            ldc = (n if lc == "row-major" else m) + 1
            A = rng.integers(-4, 5, lda * (a_rows if la == "row-major" else a_cols)).astype(np.float32)
            B = rng.integers(-4, 5, ldb * (b_rows if lb == "row-major" else b_cols)).astype(np.float32)
            C = rng.integers(-4, 5, ldc * (m if lc == "row-major" else n)).astype(np.float32)
            want = C.copy()
            for i in range(m):
                for j in range(n):
                    s = sum(_ref_elem(A, lda, la, ta, i, p) * _ref_elem(B, ldb, lb, tb, p, j) for p in range(k))
                    ci = j * ldc + i if lc == "column-major" else i * ldc + j
                    want[ci] = 2 * s + 3 * C[ci]
            fa, fb, mm, nn, AA, la2, BB, lb2 = wg.to_column_major_frame(ta, tb, m, n, A, lda, B, ldb, la, lb, lc)
            got = oracle.sgemm(fa, fb, mm, nn, k, 2.0, AA, la2, BB, lb2, 3.0, C, ldc)
            assert np.array_equal(got, want), (la, lb, lc, ta, tb)
