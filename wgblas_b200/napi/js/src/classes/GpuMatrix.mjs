// A matrix resident in device memory (src/classes/GpuMatrix.mjs:13-207): one
// device buffer holding the matrix in its own layout and leading dimension.
// f64 matrices are native doubles (the reference keeps hi/lo f32 pairs).
import { addon } from "../addon.mjs";
import { getDevice, Device } from "../init.mjs";

export class GpuMatrix {
  constructor(buffer, rows, cols, lda, loBuffer = null, layout = "row-major", device = undefined,
              dtype = Float32Array) {
    this.buffer = buffer;
    this.loBuffer = loBuffer;
    this.rows = rows;
    this.cols = cols;
    this.lda = lda;
    this.layout = layout;
    this.dtype = dtype;
    this.device = device ?? getDevice();
  }

  /**
   * GpuMatrix.from([device,] data, rows, cols, lda?, layout?): validates and
   * uploads outer*lda elements (outer = rows for row-major, cols for column-major).
   * The upload is queued on the device's stream; later calls on the device are
   * ordered after it.
   */
  static from(...args) {
    const explicit = args[0] instanceof Device;
    const device = explicit ? args.shift() : getDevice();
    const [data, rows, cols] = args;
    let lda = args[3];
    const layout = args[4] ?? "row-major";
    if (layout !== "row-major" && layout !== "column-major")
      throw new Error("layout must be 'row-major' or 'column-major'.");
    const isRow = layout === "row-major";
    if (lda === undefined || lda === null) lda = isRow ? cols : rows;
    if (!(data instanceof Float32Array) && !(data instanceof Float64Array))
      throw new Error("GpuMatrix.from expects a Float32Array, Float64Array, Complex32Array, or Complex64Array.");
    if (!Number.isInteger(rows) || rows <= 0) throw new Error("rows must be a positive integer.");
    if (!Number.isInteger(cols) || cols <= 0) throw new Error("cols must be a positive integer.");
    const minLda = isRow ? cols : rows;
    if (!Number.isInteger(lda) || lda < minLda) throw new Error(`lda must be an integer >= ${isRow ? "cols" : "rows"}.`);
    const outer = isRow ? rows : cols;
    if (data.length < outer * lda) throw new Error("data does not have enough elements for the given rows, cols, and lda.");
    const src = data.subarray(0, outer * lda);
    const buffer = addon.bufferAlloc(device.handle, src.byteLength);
    const m = new GpuMatrix(buffer, rows, cols, lda, null, layout, device, data.constructor);
    m.ready = addon.bufferUpload(device.handle, buffer, src, 0); // staged: `data` may be reused at once
    return m;
  }

  /** The matrix as a dense typed array in its own layout, lda padding stripped. */
  async read() {
    if (!this.buffer) throw new Error("GpuMatrix has been destroyed.");
    const isRow = this.layout !== "column-major";
    const outer = isRow ? this.rows : this.cols;
    const inner = isRow ? this.cols : this.rows;
    const bytes = this.dtype === Float64Array ? 8 : 4;
    const { data } = await addon.bufferRead(this.device.handle, this.buffer, 0, bytes, outer, inner, this.lda);
    return data;
  }

  destroy() {
    if (this.buffer) {
      addon.bufferFree(this.buffer);
      this.buffer = null;
    }
  }
}
