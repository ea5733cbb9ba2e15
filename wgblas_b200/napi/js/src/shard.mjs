// The row-sharded GEMM over several GPUs (one process per GPU): rank r holds its
// row block of op(A) and C as GpuMatrix (column-major, ld = its rows) and the root
// holds B; every call sends B to the other ranks over NVLink in column panels, each
// panel's GEMM starting as soon as it has arrived. The communicator id comes
// from commUniqueId() on rank 0 and reaches the other ranks out of band.
import { addon } from "./addon.mjs";

export function commUniqueId() {
  return addon.commUniqueId();
}

export class Comm {
  constructor(device, nranks, rank, id, timeoutMs = 60000) {
    this.device = device;
    this.nranks = nranks;
    this.rank = rank;
    this.handle = addon.commInitRank(device.handle, nranks, rank, id, timeoutMs);
  }

  destroy() {
    if (this.handle) {
      addon.commDestroy(this.handle);
      this.handle = null;
    }
  }
}

function sharded(f64, comm, transA, transB, mLocal, n, k, alpha, A, B, ldb, beta, C, root = 0, panelCols = 0) {
  return addon.gemmSharded(comm.handle, transA === "transpose" ? 1 : 0, transB === "transpose" ? 1 : 0, mLocal, n,
                           k, alpha, A.buffer, A.lda, B ? B.buffer : null, ldb, root, beta, C.buffer, C.lda,
                           panelCols, f64);
}

export function sgemmSharded(comm, transA, transB, mLocal, n, k, alpha, A, B, ldb, beta, C, root = 0, panelCols = 0) {
  return sharded(false, comm, transA, transB, mLocal, n, k, alpha, A, B, ldb, beta, C, root, panelCols);
}

export function dgemmSharded(comm, transA, transB, mLocal, n, k, alpha, A, B, ldb, beta, C, root = 0, panelCols = 0) {
  return sharded(true, comm, transA, transB, mLocal, n, k, alpha, A, B, ldb, beta, C, root, panelCols);
}
