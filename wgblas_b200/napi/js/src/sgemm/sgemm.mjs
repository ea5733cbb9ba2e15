// sgemm(device, transA, transB, m, n, k, alpha, A, lda, B, ldb, beta, C, ldc, layout?)
// (src/sgemm/sgemm.mjs:25-41): C := alpha*op(A)*op(B) + beta*C in fp32.
// Float32Array operands -> Promise<{C: Float32Array, gpuTimeMs?}> (a new C);
// all-GpuMatrix operands -> Promise<{gpuTimeMs?}> with C updated in place.
import { gemm } from "../gemm.mjs";

export function sgemm(device, transA, transB, m, n, k, alpha, A, lda, B, ldb, beta, C, ldc, layout = "row-major") {
  return gemm("sgemm", device, transA, transB, m, n, k, alpha, A, lda, B, ldb, beta, C, ldc, layout);
}
