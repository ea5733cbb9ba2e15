"""Device runtime: ``init`` / ``cleanup`` / ``gpuName`` on CUDA devices.

Mirrors src/init.mjs:31-182. A ``Device`` stands where the reference hands out
a ``GPUDevice``: ``init()`` caches one handle per option set and the first one
becomes the primary device that ``getDevice()`` returns; ``cleanup(device)``
releases one handle (promoting a survivor to primary) and ``cleanup()`` all of
them. Several handles may sit on one GPU, each with its own CUDA stream, as
the reference creates one GPUDevice per option set (src/init.mjs:14-29).

Device choice: ``init(device=k)`` opens CUDA ordinal k. Without it the
ordinal comes from ``WGBLAS_CUDA_DEVICES`` (a comma list; the first entry for
"high-performance", the last for "low-power"), else "high-performance" maps to
ordinal 0 and "low-power" to the last visible ordinal — so the reference's
two-device example (examples/init-two-gpus/init-two-gpus.js) lands on two
GPUs when there are two.
"""
from __future__ import annotations

import ctypes as ct
import os
import warnings

from . import _native as nat


class Error(Exception):
    """Raised with the reference's error messages (its ``throw new Error(msg)``)."""


class Adapter:
    """What the reference's GPUAdapter stands for here: the CUDA device behind a
    handle (src/init.mjs:153-168 hands it out through getAdapter). ``info``
    holds the fields gpuName reads (``description``, ``device``) plus the
    vendor and architecture; ``limits`` the device's SM count and memory."""

    __slots__ = ("ordinal", "info", "limits")

    def __init__(self, ordinal: int, info: dict, limits: dict):
        self.ordinal = ordinal
        self.info = info
        self.limits = limits

    def __repr__(self):
        return f"<wgblas Adapter cuda:{self.ordinal} {self.info.get('device', '')}>"


# Device.set_sgemm_path's names for the WG_SGEMM_* codes of include/wgblas.h.
SGEMM_PATHS = {"auto": nat.WG_SGEMM_AUTO, "simt": nat.WG_SGEMM_SIMT, "tf32x3": nat.WG_SGEMM_TF32X3,
               "tf32x3_packed": nat.WG_SGEMM_TF32X3_PACKED,
               "tf32x3_fused_bn256": nat.WG_SGEMM_TF32X3_FUSED_BN256,
               "tf32x3_fused_bn128": nat.WG_SGEMM_TF32X3_FUSED_BN128,
               "tf32x3_fused_bn64": nat.WG_SGEMM_TF32X3_FUSED_BN64,
               "tf32x3_pair": nat.WG_SGEMM_TF32X3_PAIR,
               "simt_small": nat.WG_SGEMM_SIMT_SMALL}


class Device:
    """A CUDA device handle: the counterpart of the reference's GPUDevice."""

    __slots__ = ("_handle", "ordinal", "benchmark", "options", "_name", "adapter", "__weakref__")

    def __init__(self, handle, ordinal, benchmark, options, name, adapter=None):
        self._handle = handle
        self.ordinal = ordinal
        self.benchmark = benchmark
        self.options = options
        self._name = name
        self.adapter = adapter

    @property
    def handle(self):
        if self._handle is None:
            raise Error("device has been destroyed — call init() again.")
        return self._handle

    @property
    def destroyed(self) -> bool:
        return self._handle is None

    def stream(self) -> int:
        """The cudaStream_t (as an int) this device's work is ordered on."""
        s = ct.c_void_p()
        nat.check(nat.lib.wg_device_stream(self.handle, ct.byref(s)))
        return s.value or 0

    def set_stream(self, stream: int | None) -> None:
        """Orders this device's work on a caller-owned stream (None: its own)."""
        nat.check(nat.lib.wg_device_set_stream(self.handle, ct.c_void_p(stream or None)))

    def synchronize(self) -> None:
        nat.check(nat.lib.wg_device_sync(self.handle))

    def check(self) -> None:
        """Raises if a kernel's bounded device-side wait gave up since the last check."""
        nat.check(nat.lib.wg_device_check(self.handle))

    def props(self) -> dict:
        p = nat.DeviceProps()
        nat.check(nat.lib.wg_device_props_get(self.handle, ct.byref(p)))
        return {f: getattr(p, f) for f, _ in p._fields_}

    def sgemm_stats(self) -> dict:
        s = nat.SgemmStats()
        nat.check(nat.lib.wg_device_sgemm_stats(self.handle, ct.byref(s)))
        return {f: int(getattr(s, f)) for f, _ in s._fields_}

    def set_sgemm_path(self, path: str) -> None:
        """'auto' (default), 'simt' (FFMA kernel), 'tf32x3' (tensor cores: the fused
        kernel where the operands allow it, else split pass + MMA kernel),
        'tf32x3_packed' (split pass + MMA kernel) or 'tf32x3_fused_bn256' / '_bn128' /
        '_bn64' (the fused kernel with one tile width) or 'tf32x3_pair' (its CTA-pair form),
        or 'simt_small' (the FFMA kernel's arithmetic on 32 x 64 tiles)."""
        nat.check(nat.lib.wg_device_set_sgemm_path(self.handle, SGEMM_PATHS[path]))

    def set_dgemm_path(self, path: str) -> None:
        """'auto' (default), 'simt' (DFMA kernel) or 'dmma' (FP64 tensor-core kernel)."""
        code = {"auto": nat.WG_DGEMM_AUTO, "simt": nat.WG_DGEMM_SIMT, "dmma": nat.WG_DGEMM_DMMA}[path]
        nat.check(nat.lib.wg_device_set_dgemm_path(self.handle, code))

    def set_strsm_path(self, path: str) -> None:
        """'auto' (default), 'recursive' (GEMM updates, a launch per block) or 'flow'
        (the whole solve in cooperative launches)."""
        code = {"auto": nat.WG_STRSM_AUTO, "recursive": nat.WG_STRSM_RECURSIVE, "flow": nat.WG_STRSM_FLOW}[path]
        nat.check(nat.lib.wg_device_set_strsm_path(self.handle, code))

    def set_profiling(self, on: bool) -> None:
        nat.check(nat.lib.wg_device_set_profiling(self.handle, int(bool(on))))

    def profile_read(self) -> dict:
        """{kernel family: (launches, total_ms)} since the last read (synchronises)."""
        arr = (nat.KernelProfile * 32)()
        n = ct.c_int(0)
        nat.check(nat.lib.wg_device_profile_read(self.handle, arr, 32, ct.byref(n)))
        return {arr[i].name.decode(): (int(arr[i].launches), float(arr[i].total_ms)) for i in range(n.value)}

    def kernel_launches(self) -> int:
        v = ct.c_uint64(0)
        nat.check(nat.lib.wg_device_kernel_launches(self.handle, ct.byref(v)))
        return int(v.value)

    def probe_peak(self, kind: str) -> float:
        """Roofline probe: 'fp32' / 'fp64' FMA-chain TFLOP/s, 'fp64_dmma' FP64 tensor-core
        TFLOP/s, or HBM GB/s of a 2 GiB 'hbm' copy, 'hbm_read' read-only pass or
        'hbm_scale' in-place read-modify-write (benchmarks/roofline/wgblas/bandwidth.js
        takes the best of such patterns as the memory roof)."""
        code = {"fp32": nat.WG_PROBE_FP32_FMA, "fp64": nat.WG_PROBE_FP64_FMA, "hbm": nat.WG_PROBE_HBM_COPY,
                "fp64_dmma": nat.WG_PROBE_FP64_DMMA, "hbm_read": nat.WG_PROBE_HBM_READ,
                "hbm_scale": nat.WG_PROBE_HBM_SCALE}[kind]
        v = ct.c_double(0)
        nat.check(nat.lib.wg_probe_peak(self.handle, code, ct.byref(v)))
        return float(v.value)

    def __repr__(self):
        state = "destroyed" if self.destroyed else f"cuda:{self.ordinal}"
        return f"<wgblas Device {state} {self.options}>"


_devices: dict[str, Device] = {}
_primary: Device | None = None


def _options_key(o) -> str:
    return f"{o['powerPreference']}::{o['benchmark']}::{o['device']}"


def _ordinal_for(power_preference: str, explicit) -> int:
    count = nat.device_count()
    if count == 0:
        raise Error("No CUDA device found.")
    if explicit is not None:
        if not isinstance(explicit, int) or isinstance(explicit, bool) or not 0 <= explicit < count:
            raise Error(f"device must be a CUDA ordinal in [0, {count}).")
        return explicit
    env = os.environ.get("WGBLAS_CUDA_DEVICES")
    if env:
        ords = [int(x) for x in env.split(",") if x.strip()]
        ords = [o for o in ords if 0 <= o < count] or [0]
        return ords[-1] if power_preference == "low-power" else ords[0]
    return count - 1 if power_preference == "low-power" else 0


def init(powerPreference: str = "high-performance", benchmark: bool = False,
         dumpShaders: bool = False, device: int | None = None) -> Device:
    """Returns the cached device for this option set, creating it on first use
    (src/init.mjs:31-107). ``benchmark=True`` makes GEMM calls return
    ``gpuTimeMs``; ``dumpShaders`` has no CUDA counterpart and only warns."""
    global _primary
    options = {"powerPreference": powerPreference, "benchmark": bool(benchmark), "device": device}
    key = _options_key(options)
    cached = _devices.get(key)
    if cached is not None:
        return cached
    if dumpShaders:
        warnings.warn("dumpShaders has no effect on the CUDA backend (there are no WGSL shaders).")
    ordinal = _ordinal_for(powerPreference, device)
    h = nat.c_dev_p()
    nat.check(nat.lib.wg_device_open(ordinal, nat.WG_DEVICE_TIMING if benchmark else 0, ct.byref(h)))
    buf = ct.create_string_buffer(256)
    nat.check(nat.lib.wg_device_name(h, buf, 256))
    name = buf.value.decode()
    p = nat.DeviceProps()
    nat.check(nat.lib.wg_device_props_get(h, ct.byref(p)))
    adapter = Adapter(ordinal, {"vendor": "nvidia", "architecture": f"sm_{p.cc_major}{p.cc_minor}",
                                "device": name, "description": f"cuda:{ordinal}"},
                      {"smCount": int(p.sm_count), "totalMemory": int(p.total_mem)})
    dev = Device(h, ordinal, bool(benchmark), options, name, adapter)
    _devices[key] = dev
    if _primary is None:
        _primary = dev
    return dev


def cleanup(device: Device | None = None) -> None:
    """Releases one device, or every device when called without one
    (src/init.mjs:110-131). Unknown or released devices are a no-op."""
    global _primary
    if device is None:
        for d in list(_devices.values()):
            _close(d)
        _devices.clear()
        _primary = None
        return
    if not isinstance(device, Device) or device.destroyed:
        return
    key = next((k for k, v in _devices.items() if v is device), None)
    if key is None:
        return
    del _devices[key]
    _close(device)
    if _primary is device:
        _primary = next(iter(_devices.values()), None)


def _close(d: Device) -> None:
    if d._handle is not None:
        nat.lib.wg_device_close(d._handle)
        d._handle = None


def _registered(device) -> bool:
    return isinstance(device, Device) and not device.destroyed and any(v is device for v in _devices.values())


def gpuName(device: Device | None = None) -> dict:
    """``{description, device}`` for a device, from its adapter's info, each
    "unknown" when empty (src/init.mjs:133-143)."""
    device = _primary if device is None else device
    if not _registered(device):
        raise Error("CUDA device not initialized — call init() first.")
    info = device.adapter.info if device.adapter is not None else {}
    return {"description": info.get("description") or "unknown", "device": info.get("device") or "unknown"}


def getDevice() -> Device:
    """The device from the first init() (src/init.mjs:163-168)."""
    if _primary is None:
        raise Error("CUDA device not initialized — call init() first.")
    return _primary


def getAdapter(device: Device | None = None) -> Adapter:
    """The adapter behind ``device``, by default the primary one (src/init.mjs:170-182)."""
    device = _primary if device is None else device
    if not _registered(device) or device.adapter is None:
        raise Error("CUDA adapter not initialized — call init() first.")
    return device.adapter


def isBenchmarkEnabled(device: Device | None = None) -> bool:
    """Whether ``device`` (by default the primary one) was created with
    benchmark=True; False for anything init() did not hand out (src/init.mjs:153-155)."""
    device = _primary if device is None else device
    return bool(_registered(device) and device.benchmark)


def require_gpu_device(device) -> None:
    """requireGpuDevice (src/util/device.mjs:14-17)."""
    if not isinstance(device, Device) or device.destroyed:
        raise Error("device must be a GPUDevice.")


def require_same_device(device: Device, routine: str, operands: dict) -> None:
    """requireSameDevice (src/util/device.mjs:37-49)."""
    from .classes import GpuMatrix, GpuVector

    for name, value in operands.items():
        if not isinstance(value, (GpuMatrix, GpuVector)):
            continue
        if value.device is not device:
            raise Error(
                f"{routine}: {name} belongs to a different GPUDevice than the one passed in. "
                "GPU buffers cannot be shared across devices — recreate the operand on this "
                "device, or call the routine with the device that owns it.")
