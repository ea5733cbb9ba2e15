"""ctypes binding of libwgblas_b200.so (include/wgblas.h).

The library is built in-tree by ``python -m wgblas_b200.build``; importing this
module without it raises ImportError — there is no CPU fallback.
"""
from __future__ import annotations

import ctypes as ct
import os

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libwgblas_b200.so")

if not os.path.exists(LIB_PATH):
    raise ImportError(
        f"{LIB_PATH} is missing: build the CUDA library with `python wgblas_b200/build.py` "
        "(wgblas_b200 has no CPU fallback)")

lib = ct.CDLL(LIB_PATH)

# status codes (wg_status)
WG_OK = 0
WG_ERR_INVALID_ARGUMENT = 1
WG_ERR_OUT_OF_MEMORY = 2
WG_ERR_CUDA = 3
WG_ERR_NO_DEVICE = 4
WG_ERR_KERNEL_TIMEOUT = 5
WG_ERR_NCCL = 6
WG_ERR_NOT_SUPPORTED = 7

WG_DEVICE_TIMING = 1
WG_SGEMM_AUTO, WG_SGEMM_SIMT, WG_SGEMM_TF32X3 = 0, 1, 2
WG_SGEMM_TF32X3_PACKED, WG_SGEMM_TF32X3_FUSED_BN256, WG_SGEMM_TF32X3_FUSED_BN128, WG_SGEMM_TF32X3_FUSED_BN64 = 3, 4, 5, 6
WG_SGEMM_TF32X3_PAIR = 7
WG_SGEMM_SIMT_SMALL = 8
WG_DGEMM_AUTO, WG_DGEMM_SIMT, WG_DGEMM_DMMA = 0, 1, 2
WG_STRSM_AUTO, WG_STRSM_RECURSIVE, WG_STRSM_FLOW = 0, 1, 2

c_dev_p = ct.c_void_p
c_buf_p = ct.c_void_p
_i64 = ct.c_int64
_f32p = ct.POINTER(ct.c_float)
_f64p = ct.POINTER(ct.c_double)


class DeviceProps(ct.Structure):
    _fields_ = [("ordinal", ct.c_int), ("sm_count", ct.c_int), ("cc_major", ct.c_int),
                ("cc_minor", ct.c_int), ("total_mem", ct.c_size_t), ("flags", ct.c_uint)]


class SgemmStats(ct.Structure):
    _fields_ = [("calls", ct.c_uint64), ("tf32x3_launches", ct.c_uint64),
                ("simt_launches", ct.c_uint64), ("fallbacks", ct.c_uint64)]


def _sig(name, restype, *argtypes):
    fn = getattr(lib, name)
    fn.restype = restype
    fn.argtypes = list(argtypes)
    return fn


_st = ct.c_int
_sig("wg_last_error", ct.c_char_p)
_sig("wg_abi_version", ct.c_int)
_sig("wg_device_count", _st, ct.POINTER(ct.c_int))
_sig("wg_device_open", _st, ct.c_int, ct.c_uint, ct.POINTER(c_dev_p))
_sig("wg_device_close", _st, c_dev_p)
_sig("wg_device_name", _st, c_dev_p, ct.c_char_p, ct.c_size_t)
_sig("wg_device_props_get", _st, c_dev_p, ct.POINTER(DeviceProps))
_sig("wg_device_stream", _st, c_dev_p, ct.POINTER(ct.c_void_p))
_sig("wg_device_set_stream", _st, c_dev_p, ct.c_void_p)
_sig("wg_device_sync", _st, c_dev_p)
_sig("wg_device_check", _st, c_dev_p)
_sig("wg_device_sgemm_stats", _st, c_dev_p, ct.POINTER(SgemmStats))
_sig("wg_device_set_sgemm_path", _st, c_dev_p, ct.c_int)
_sig("wg_device_set_dgemm_path", _st, c_dev_p, ct.c_int)
_sig("wg_device_set_strsm_path", _st, c_dev_p, ct.c_int)
class KernelProfile(ct.Structure):
    _fields_ = [("name", ct.c_char * 48), ("launches", ct.c_uint64), ("total_ms", ct.c_double)]


class TcPlan(ct.Structure):
    _fields_ = [("tiles_m", ct.c_int64), ("tiles_n", ct.c_int64), ("k_blocks", ct.c_int64), ("grid", ct.c_int),
                ("whole_tiles", ct.c_int), ("split_tiles", ct.c_int), ("split_segments", ct.c_int),
                ("workspace_bytes", ct.c_size_t)]


_sig("wg_sgemm_tc_plan", _st, ct.c_int, ct.c_int64, ct.c_int64, ct.c_int64, ct.POINTER(TcPlan))
_sig("wg_sharded_panel_plan", _st, ct.c_int, ct.c_int, ct.c_int64, ct.c_int64, ct.c_int64,
     ct.POINTER(ct.c_int64), ct.c_size_t, ct.POINTER(ct.c_size_t))
_sig("wg_selftest_bounded_wait", _st, c_dev_p, ct.c_uint)
_sig("wg_symmetrize", _st, c_dev_p, ct.c_int, ct.c_int, _i64, c_buf_p, _i64, _i64, c_buf_p, _i64, _i64)
_sig("wg_triangularize", _st, c_dev_p, ct.c_int, ct.c_int, ct.c_int, ct.c_int, _i64, c_buf_p, _i64, _i64, c_buf_p,
     _i64, _i64)
_sig("wg_buffer_copy_2d", _st, c_dev_p, c_buf_p, ct.c_size_t, ct.c_size_t, c_buf_p, ct.c_size_t, ct.c_size_t,
     ct.c_size_t, ct.c_size_t)
WG_PROBE_FP32_FMA, WG_PROBE_FP64_FMA, WG_PROBE_HBM_COPY, WG_PROBE_FP64_DMMA = 0, 1, 2, 3
WG_PROBE_HBM_READ, WG_PROBE_HBM_SCALE = 4, 5
_sig("wg_device_set_profiling", _st, c_dev_p, ct.c_int)
_sig("wg_device_profile_read", _st, c_dev_p, ct.POINTER(KernelProfile), ct.c_int, ct.POINTER(ct.c_int))
_sig("wg_device_kernel_launches", _st, c_dev_p, ct.POINTER(ct.c_uint64))
_sig("wg_probe_peak", _st, c_dev_p, ct.c_int, ct.POINTER(ct.c_double))
_sig("wg_buffer_alloc", _st, c_dev_p, ct.c_size_t, ct.POINTER(c_buf_p))
_sig("wg_buffer_alloc_async", _st, c_dev_p, ct.c_size_t, ct.POINTER(c_buf_p))
_sig("wg_buffer_free", _st, c_buf_p)
_sig("wg_buffer_size", _st, c_buf_p, ct.POINTER(ct.c_size_t))
_sig("wg_buffer_device_ptr", _st, c_buf_p, ct.POINTER(ct.c_void_p))
_sig("wg_buffer_upload", _st, c_buf_p, ct.c_size_t, ct.c_void_p, ct.c_size_t)
_sig("wg_buffer_download", _st, c_buf_p, ct.c_size_t, ct.c_void_p, ct.c_size_t)
_sig("wg_buffer_upload_2d", _st, c_buf_p, ct.c_size_t, ct.c_size_t, ct.c_void_p, ct.c_size_t,
     ct.c_size_t, ct.c_size_t)
_sig("wg_buffer_download_2d", _st, c_buf_p, ct.c_size_t, ct.c_size_t, ct.c_void_p, ct.c_size_t,
     ct.c_size_t, ct.c_size_t)
_sig("wg_host_alloc", _st, ct.c_size_t, ct.POINTER(ct.c_void_p))
_sig("wg_host_free", _st, ct.c_void_p)
_gemm_dims = [c_dev_p, ct.c_int, ct.c_int, _i64, _i64, _i64]
_sig("wg_sgemm", _st, *_gemm_dims, ct.c_float, c_buf_p, _i64, _i64, c_buf_p, _i64, _i64, ct.c_float,
     c_buf_p, _i64, _i64, _f32p)
_sig("wg_dgemm", _st, *_gemm_dims, ct.c_double, c_buf_p, _i64, _i64, c_buf_p, _i64, _i64, ct.c_double,
     c_buf_p, _i64, _i64, _f32p)
_sig("wg_sgemm_dev", _st, *_gemm_dims, ct.c_float, ct.c_void_p, _i64, ct.c_void_p, _i64, ct.c_float,
     ct.c_void_p, _i64)
_sig("wg_dgemm_dev", _st, *_gemm_dims, ct.c_double, ct.c_void_p, _i64, ct.c_void_p, _i64, ct.c_double,
     ct.c_void_p, _i64)
_sig("wg_sgemm_noalloc", _st, *_gemm_dims, ct.c_float, ct.c_void_p, _i64, ct.c_void_p, _i64, ct.c_float,
     ct.c_void_p, _i64)
_sig("wg_sgemm_host", _st, *_gemm_dims, ct.c_float, ct.c_void_p, _i64, ct.c_void_p, _i64, ct.c_float,
     ct.c_void_p, ct.c_void_p, _i64, _f32p)
_sig("wg_dgemm_host", _st, *_gemm_dims, ct.c_double, ct.c_void_p, _i64, ct.c_void_p, _i64, ct.c_double,
     ct.c_void_p, ct.c_void_p, _i64, _f32p)
WG_UPLO_FULL, WG_UPLO_LOWER, WG_UPLO_UPPER = 0, 1, 2
_tr_dims = [c_dev_p, ct.c_int] + _gemm_dims[1:]
_sig("wg_sgemmtr", _st, *_tr_dims, ct.c_float, c_buf_p, _i64, _i64, c_buf_p, _i64, _i64, ct.c_float,
     c_buf_p, _i64, _i64, _f32p)
_sig("wg_dgemmtr", _st, *_tr_dims, ct.c_double, c_buf_p, _i64, _i64, c_buf_p, _i64, _i64, ct.c_double,
     c_buf_p, _i64, _i64, _f32p)
_sig("wg_sgemmtr_dev", _st, *_tr_dims, ct.c_float, ct.c_void_p, _i64, ct.c_void_p, _i64, ct.c_float,
     ct.c_void_p, _i64)
_sig("wg_dgemmtr_dev", _st, *_tr_dims, ct.c_double, ct.c_void_p, _i64, ct.c_void_p, _i64, ct.c_double,
     ct.c_void_p, _i64)
_sig("wg_sgemmtr_host", _st, *_tr_dims, ct.c_float, ct.c_void_p, _i64, ct.c_void_p, _i64, ct.c_float,
     ct.c_void_p, ct.c_void_p, _i64, _f32p)
_sig("wg_dgemmtr_host", _st, *_tr_dims, ct.c_double, ct.c_void_p, _i64, ct.c_void_p, _i64, ct.c_double,
     ct.c_void_p, ct.c_void_p, _i64, _f32p)
WG_SIDE_LEFT, WG_SIDE_RIGHT = 0, 1
WG_DIAG_NON_UNIT, WG_DIAG_UNIT = 0, 1
_trsm_dims = [c_dev_p, ct.c_int, ct.c_int, ct.c_int, ct.c_int, _i64, _i64, ct.c_float]
_sig("wg_strsm", _st, *_trsm_dims, c_buf_p, _i64, _i64, c_buf_p, _i64, _i64, _f32p)
_sig("wg_strsm_dev", _st, *_trsm_dims, ct.c_void_p, _i64, ct.c_void_p, _i64)
_gemv_dims = [c_dev_p, ct.c_int, _i64, _i64]
_sig("wg_sgemv", _st, *_gemv_dims, ct.c_float, c_buf_p, _i64, _i64, c_buf_p, _i64, _i64, ct.c_float, c_buf_p, _i64,
     _i64, _f32p)
_sig("wg_dgemv", _st, *_gemv_dims, ct.c_double, c_buf_p, _i64, _i64, c_buf_p, _i64, _i64, ct.c_double, c_buf_p,
     _i64, _i64, _f32p)
_sig("wg_sgemv_dev", _st, *_gemv_dims, ct.c_float, ct.c_void_p, _i64, ct.c_void_p, _i64, ct.c_float, ct.c_void_p,
     _i64)
_sig("wg_dgemv_dev", _st, *_gemv_dims, ct.c_double, ct.c_void_p, _i64, ct.c_void_p, _i64, ct.c_double, ct.c_void_p,
     _i64)
c_comm_p = ct.c_void_p
_sig("wg_comm_unique_id", _st, ct.c_char_p, ct.c_size_t)
_sig("wg_comm_init_rank", _st, c_dev_p, ct.c_int, ct.c_int, ct.c_char_p, ct.c_size_t, ct.c_int, ct.POINTER(c_comm_p))
_sig("wg_comm_destroy", _st, c_comm_p)
_sig("wg_comm_abort", _st, c_comm_p)
_sig("wg_comm_rank", _st, c_comm_p, ct.POINTER(ct.c_int), ct.POINTER(ct.c_int))
_sig("wg_comm_wait", _st, c_comm_p)
_shard = [c_comm_p, ct.c_int, ct.c_int, _i64, _i64, _i64]
_sig("wg_sgemm_sharded", _st, *_shard, ct.c_float, ct.c_void_p, _i64, ct.c_void_p, _i64, ct.c_int, ct.c_float,
     ct.c_void_p, _i64, _i64)
_sig("wg_dgemm_sharded", _st, *_shard, ct.c_double, ct.c_void_p, _i64, ct.c_void_p, _i64, ct.c_int, ct.c_double,
     ct.c_void_p, _i64, _i64)
_gather = [c_comm_p, ct.c_void_p, _i64, _i64, _i64, ct.c_int, ct.c_void_p, _i64, ct.POINTER(_i64)]
_sig("wg_sgemm_gather_rows", _st, *_gather)
_sig("wg_dgemm_gather_rows", _st, *_gather)
_sig("wg_random_f32", None, _f32p, _i64, ct.c_double, ct.c_double, ct.c_uint32)
_sig("wg_random_f64", None, _f64p, _i64, ct.c_double, ct.c_double, ct.c_uint32)
_sig("wg_random_normal_f32", None, _f32p, _i64, ct.c_uint32)
_sig("wg_random_normal_f64", None, _f64p, _i64, ct.c_uint32)


class NativeError(RuntimeError):
    """A C-ABI call failed; ``status`` is its wg_status code."""

    def __init__(self, status: int, message: str):
        super().__init__(message)
        self.status = status


def check(status: int) -> None:
    if status != WG_OK:
        msg = lib.wg_last_error().decode(errors="replace")
        raise NativeError(status, msg or f"wg_status {status}")


def device_count() -> int:
    n = ct.c_int(0)
    check(lib.wg_device_count(ct.byref(n)))
    return n.value
