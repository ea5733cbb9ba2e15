"""wgblas-b200: wgblas's level-3 GEMM path (sgemm / dgemm) on NVIDIA B200.

The public names follow wgblas's JavaScript API (index.mjs): ``init``,
``cleanup``, ``gpuName``, ``getDevice``, ``getAdapter``, ``sgemm``, ``dgemm``, the gemmtr family (``sgemmtr``,
``dgemmtr``, ``ssyrk``, ``dsyrk``, ``ssyr2k``, ``dsyr2k``), ``ssymm``/``dsymm``,
``strmm``/``dtrmm``, ``strsm``, ``sgemv``/``dgemv``, ``GpuMatrix``,
``GpuVector``, ``randomFloat32Array`` and ``randomFloat64Array``. Compute runs in the CUDA
library libwgblas_b200.so (include/wgblas.h) with hand-written sm_100a
kernels; importing the package without that library raises ImportError.
"""
from . import _native  # noqa: F401  (fails loudly when the CUDA library is missing)
from ._runtime import (Adapter, Device, Error, cleanup, getAdapter, getDevice, gpuName, init,  # noqa: F401
                       isBenchmarkEnabled)
from .classes import Float32Array, Float64Array, GpuMatrix, GpuVector, pinned_empty  # noqa: F401
from .gemm import dgemm, sgemm, to_column_major_frame  # noqa: F401
from .gemmtr import dgemmtr, dsyr2k, dsyrk, sgemmtr, ssyr2k, ssyrk  # noqa: F401
from .gemv import dgemv, sgemv  # noqa: F401
from .level3 import dsymm, dtrmm, ssymm, strmm, strsm  # noqa: F401
from .random import (fill_uniform, randomFloat32Array, randomFloat64Array,  # noqa: F401
                     randomNormalFloat32Array, randomNormalFloat64Array)

__all__ = [
    "init", "cleanup", "gpuName", "getDevice", "getAdapter", "isBenchmarkEnabled", "Device", "Adapter", "Error",
    "GpuMatrix", "GpuVector", "Float32Array", "Float64Array", "pinned_empty",
    "sgemm", "dgemm", "sgemmtr", "dgemmtr", "ssyrk", "dsyrk", "ssyr2k", "dsyr2k",
    "ssymm", "dsymm", "strmm", "dtrmm", "strsm", "sgemv", "dgemv",
    "randomFloat32Array", "randomFloat64Array",
    "randomNormalFloat32Array", "randomNormalFloat64Array", "fill_uniform",
]
