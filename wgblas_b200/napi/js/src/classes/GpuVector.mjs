// A vector resident in device memory (src/classes/GpuVector.mjs:13-106).
import { addon } from "../addon.mjs";
import { getDevice, Device } from "../init.mjs";

export class GpuVector {
  constructor(buffer, length, dtype = Float32Array, loBuffer = null, device = undefined) {
    this.buffer = buffer;
    this.loBuffer = loBuffer;
    this.length = length;
    this.dtype = dtype;
    this.device = device ?? getDevice();
  }

  static from(...args) {
    const explicit = args[0] instanceof Device;
    const device = explicit ? args.shift() : getDevice();
    const [data] = args;
    if (!(data instanceof Float32Array) && !(data instanceof Float64Array))
      throw new Error("GpuVector.from expects a Float32Array, Float64Array, Complex32Array, or Complex64Array.");
    const buffer = addon.bufferAlloc(device.handle, Math.max(data.byteLength, 1));
    const v = new GpuVector(buffer, data.length, data.constructor, null, device);
    v.ready = addon.bufferUpload(device.handle, buffer, data, 0);
    return v;
  }

  async read() {
    if (!this.buffer) throw new Error("GpuVector has been destroyed.");
    const bytes = this.dtype === Float64Array ? 8 : 4;
    const { data } = await addon.bufferRead(this.device.handle, this.buffer, 0, bytes, 1, this.length, this.length);
    return data;
  }

  destroy() {
    if (this.buffer) {
      addon.bufferFree(this.buffer);
      this.buffer = null;
    }
  }
}
