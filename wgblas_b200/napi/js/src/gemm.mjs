// sgemm / dgemm: the argument checks of src/sgemm/sgemm.mjs:42-149 (and
// dgemm.mjs) in the same order with the same messages, the mapping of layouts
// onto the column-major frame of the C ABI (the twin of the row-major frame
// swap at src/sgemm/sgemm.mjs:151-167), and the addon call: typed arrays ->
// {C: new array, gpuTimeMs?}, all-GpuMatrix -> {gpuTimeMs?} with C in place.
import { addon } from "./addon.mjs";
import { requireGpuDevice, requireSameDevice } from "./init.mjs";
import { GpuMatrix } from "./classes/GpuMatrix.mjs";

const TRANS = ["no-transpose", "transpose"];
const LAYOUTS = ["row-major", "column-major"];

function validate(routine, device, transA, transB, m, n, k, alpha, A, lda, B, ldb, beta, C, ldc, layout) {
  const f64 = routine === "dgemm";
  const Arr = f64 ? Float64Array : Float32Array;
  const arrName = f64 ? "Float64Array" : "Float32Array";
  const aGpu = A instanceof GpuMatrix, bGpu = B instanceof GpuMatrix, cGpu = C instanceof GpuMatrix;
  requireGpuDevice(device);
  requireSameDevice(device, routine, { A, B, C });
  if (!TRANS.includes(transA)) throw new Error("transA must be 'no-transpose' or 'transpose'.");
  if (!TRANS.includes(transB)) throw new Error("transB must be 'no-transpose' or 'transpose'.");
  if (!LAYOUTS.includes(layout)) throw new Error("layout must be 'row-major' or 'column-major'.");
  for (const [name, v] of [["alpha", alpha], ["beta", beta]]) {
    if (typeof v !== "number") throw new Error(`${name} must be a number.`);
    if (Number.isNaN(v)) throw new Error(`${name} must not be NaN.`);
    if (!Number.isFinite(v)) throw new Error(`${name} must be finite.`);
  }
  if (![m, n, k, lda, ldb, ldc].every(Number.isInteger))
    throw new Error("m, n, k, lda, ldb, and ldc must be integers.");
  if (!aGpu && !(A instanceof Arr)) throw new Error(`A must be a ${arrName} or GpuMatrix.`);
  if (!bGpu && !(B instanceof Arr)) throw new Error(`B must be a ${arrName} or GpuMatrix.`);
  if (!cGpu && !(C instanceof Arr)) throw new Error(`C must be a ${arrName} or GpuMatrix.`);
  if (f64) {
    for (const [name, X, g] of [["A", A, aGpu], ["B", B, bGpu], ["C", C, cGpu]])
      if (g && X.dtype !== Float64Array) throw new Error(`${name} must be a Float64Array-backed GpuMatrix.`);
  }
  if ((aGpu || bGpu) && !cGpu) throw new Error("C must be a GpuMatrix when A or B is a GpuMatrix.");
  if (cGpu && (!aGpu || !bGpu)) throw new Error("A and B must be GpuMatrix when C is a GpuMatrix.");
  if (m < 0 || n < 0 || k < 0) throw new Error("m, n, and k must be non-negative.");
  if (lda <= 0 || ldb <= 0 || ldc <= 0) throw new Error("lda, ldb, and ldc must be positive.");
  if (m === 0 || n === 0) return cGpu ? {} : { C };

  const la = aGpu ? A.layout : layout, lb = bGpu ? B.layout : layout, lc = cGpu ? C.layout : layout;
  const [aRows, aCols] = la === "column-major" ? [k, m] : [m, k];
  const aOuter = transA === "no-transpose" ? aRows : aCols;
  const aInner = transA === "no-transpose" ? aCols : aRows;
  if (lda < aInner) throw new Error(`lda must be >= ${la === "column-major" ? "rows" : "cols"} of A as stored.`);
  if (aGpu) {
    if (lda !== A.lda) throw new Error("lda must match A.lda when A is a GpuMatrix.");
    const [lr, lcl] = transA === "no-transpose" ? [m, k] : [k, m];
    if (A.rows < lr || A.cols < lcl) throw new Error("A is too small for the given m, k, and transA.");
  } else if (A.length < (aOuter - 1) * lda + aInner) {
    throw new Error("A does not have enough elements for the given dimensions and lda.");
  }
  const [bRows, bCols] = lb === "column-major" ? [n, k] : [k, n];
  const bOuter = transB === "no-transpose" ? bRows : bCols;
  const bInner = transB === "no-transpose" ? bCols : bRows;
  if (ldb < bInner) throw new Error(`ldb must be >= ${lb === "column-major" ? "rows" : "cols"} of B as stored.`);
  if (bGpu) {
    if (ldb !== B.lda) throw new Error("ldb must match B.lda when B is a GpuMatrix.");
    const [lr, lcl] = transB === "no-transpose" ? [k, n] : [n, k];
    if (B.rows < lr || B.cols < lcl) throw new Error("B is too small for the given n, k, and transB.");
  } else if (B.length < (bOuter - 1) * ldb + bInner) {
    throw new Error("B does not have enough elements for the given dimensions and ldb.");
  }
  const cOuter = lc === "column-major" ? n : m;
  const cInner = lc === "column-major" ? m : n;
  if (ldc < cInner) throw new Error(`ldc must be >= ${lc === "column-major" ? "rows" : "cols"} of C as stored.`);
  if (cGpu) {
    if (ldc !== C.lda) throw new Error("ldc must match C.lda when C is a GpuMatrix.");
    if (C.rows < m || C.cols < n) throw new Error("C is too small for the given m and n.");
  } else if (C.length < (cOuter - 1) * ldc + cInner) {
    throw new Error("C does not have enough elements for the given dimensions and ldc.");
  }
  return null;
}

/** Column-major-frame arguments: a row-major operand flips its trans flag; a
 * row-major C computes C^T = op(B)^T op(A)^T (operands and m/n swapped). */
export function toColumnMajorFrame(transA, transB, m, n, A, lda, B, ldb, la, lb, lc) {
  const ta = (transA === "transpose") === (la === "column-major");
  const tb = (transB === "transpose") === (lb === "column-major");
  if (lc === "column-major") return [Number(ta), Number(tb), m, n, A, lda, B, ldb];
  return [Number(!tb), Number(!ta), n, m, B, ldb, A, lda];
}

export async function gemm(routine, device, transA, transB, m, n, k, alpha, A, lda, B, ldb, beta, C, ldc,
                           layout = "row-major") {
  const early = validate(routine, device, transA, transB, m, n, k, alpha, A, lda, B, ldb, beta, C, ldc, layout);
  if (early) return early;
  const f64 = routine === "dgemm";
  const cGpu = C instanceof GpuMatrix;
  // dgemm's BLAS quick return (src/dgemm/dgemm.mjs:177-179): C comes back as it is.
  if (f64 && (alpha === 0 || k === 0) && beta === 1) return cGpu ? {} : { C };
  const la = cGpu ? A.layout : layout, lb = cGpu ? B.layout : layout, lc = cGpu ? C.layout : layout;
  const [ta, tb, mm, nn, AA, lda2, BB, ldb2] = toColumnMajorFrame(transA, transB, m, n, A, lda, B, ldb, la, lb, lc);
  let res;
  if (cGpu) {
    await Promise.all([AA.ready, BB.ready, C.ready]);
    res = await addon.gemm(device.handle, ta, tb, mm, nn, k, alpha, AA.buffer, 0, lda2, BB.buffer, 0, ldb2, beta,
                           C.buffer, 0, ldc, f64);
    delete res.C;
  } else {
    res = await addon.gemmHost(device.handle, ta, tb, mm, nn, k, alpha, AA, lda2, BB, ldb2, beta, C, ldc, f64);
  }
  if (!device.benchmark) delete res.gpuTimeMs;
  return res;
}
