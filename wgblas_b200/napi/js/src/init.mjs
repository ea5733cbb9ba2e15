// Device lifecycle: init / cleanup / gpuName / getDevice / getAdapter /
// isBenchmarkEnabled, with src/init.mjs:31-182's semantics on CUDA devices.
// init() caches one device per option set; the first becomes the primary that
// getDevice() returns; cleanup(device) releases one and promotes a survivor,
// cleanup() releases all. powerPreference "high-performance" opens the first
// CUDA ordinal and "low-power" the last, so the reference's two-device example
// (examples/init-two-gpus/init-two-gpus.js) lands on two GPUs when there are two;
// options.device names an ordinal explicitly.
import { addon } from "./addon.mjs";

/** A CUDA device handle: stands where the reference hands out a GPUDevice. */
export class Device {
  constructor(handle, ordinal, benchmark, options, adapter) {
    this.handle = handle;
    this.ordinal = ordinal;
    this.benchmark = benchmark;
    this.options = options;
    this.adapter = adapter;
    this.destroyed = false;
  }
}

const _devices = new Map(); // options key -> Device
const _meta = new Map();    // Device -> { adapter, benchmark, options }
let _primary = null;

function optionsKey(o) {
  return `${o.powerPreference}::${o.benchmark}::${o.device}`;
}

function ordinalFor(powerPreference, explicit) {
  const count = addon.deviceCount();
  if (count === 0) throw new Error("No CUDA device found.");
  if (explicit !== undefined && explicit !== null) {
    if (!Number.isInteger(explicit) || explicit < 0 || explicit >= count)
      throw new Error(`device must be a CUDA ordinal in [0, ${count}).`);
    return explicit;
  }
  return powerPreference === "low-power" ? count - 1 : 0;
}

/**
 * Returns the cached device for this option set, creating it on first use.
 * @param {{powerPreference?: string, benchmark?: boolean, dumpShaders?: boolean, device?: number}} [options]
 * @returns {Promise<Device>}
 */
export async function init(options = {}) {
  const opts = {
    powerPreference: options.powerPreference ?? "high-performance",
    benchmark: Boolean(options.benchmark),
    device: options.device ?? null,
  };
  const key = optionsKey(opts);
  const cached = _devices.get(key);
  if (cached) return cached;
  if (options.dumpShaders) {
    console.warn("dumpShaders has no effect on the CUDA backend (there are no WGSL shaders).");
  }
  const ordinal = ordinalFor(opts.powerPreference, opts.device);
  const handle = addon.deviceOpen(ordinal, opts.benchmark);
  const info = addon.deviceInfo(handle);
  const adapter = {
    info: { vendor: "nvidia", architecture: info.architecture, device: info.name, description: `cuda:${ordinal}` },
    limits: { smCount: info.smCount, totalMemory: info.totalMemory },
  };
  const device = new Device(handle, ordinal, opts.benchmark, opts, adapter);
  _meta.set(device, { adapter, benchmark: opts.benchmark, options: opts });
  _devices.set(key, device);
  if (!_primary) _primary = device;
  return device;
}

/** Releases one device, or every device without an argument (src/init.mjs:110-131). */
export function cleanup(device) {
  if (device === undefined) {
    for (const d of _devices.values()) close(d);
    _devices.clear();
    _meta.clear();
    _primary = null;
    return;
  }
  const meta = _meta.get(device);
  if (!meta) return; // unknown or already released: a no-op
  _devices.delete(optionsKey(meta.options));
  _meta.delete(device);
  close(device);
  if (_primary === device) _primary = _devices.values().next().value ?? null;
}

function close(d) {
  if (!d.destroyed) {
    addon.deviceClose(d.handle);
    d.destroyed = true;
  }
}

/** `{description, device}` of a device's adapter, "unknown" where empty (src/init.mjs:133-143). */
export function gpuName(device = _primary) {
  const meta = device && _meta.get(device);
  if (!meta) throw new Error("CUDA device not initialized — call init() first.");
  const { description, device: name } = meta.adapter.info ?? {};
  return { description: description || "unknown", device: name || "unknown" };
}

/** Whether `device` (default: the primary) was created with benchmark: true. */
export function isBenchmarkEnabled(device = _primary) {
  return _meta.get(device)?.benchmark ?? false;
}

/** The device of the first init() call. */
export function getDevice() {
  if (!_primary) throw new Error("CUDA device not initialized — call init() first.");
  return _primary;
}

/** The adapter behind `device` (default: the primary). */
export function getAdapter(device = _primary) {
  const meta = device && _meta.get(device);
  if (!meta) throw new Error("CUDA adapter not initialized — call init() first.");
  return meta.adapter;
}

/** requireGpuDevice (src/util/device.mjs:14-17). */
export function requireGpuDevice(device) {
  if (!(device instanceof Device) || device.destroyed) throw new Error("device must be a GPUDevice.");
}

/** requireSameDevice (src/util/device.mjs:37-49). */
export function requireSameDevice(device, routine, operands) {
  for (const [name, value] of Object.entries(operands)) {
    if (value && typeof value === "object" && "device" in value && value.device !== device) {
      throw new Error(
        `${routine}: ${name} belongs to a different GPUDevice than the one passed in. ` +
          "GPU buffers cannot be shared across devices — recreate the operand on this " +
          "device, or call the routine with the device that owns it.",
      );
    }
  }
}
