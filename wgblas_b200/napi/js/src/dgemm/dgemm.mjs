// dgemm(device, transA, transB, m, n, k, alpha, A, lda, B, ldb, beta, C, ldc, layout?)
// (src/dgemm/dgemm.mjs:23-39): the same as sgemm with Float64Array operands,
// computed in native fp64.
import { gemm } from "../gemm.mjs";

export function dgemm(device, transA, transB, m, n, k, alpha, A, lda, B, ldb, beta, C, ldc, layout = "row-major") {
  return gemm("dgemm", device, transA, transB, m, n, k, alpha, A, lda, B, ldb, beta, C, ldc, layout);
}
