"""Seeded inputs: ``randomFloat32Array`` / ``randomFloat64Array`` (src/random/random.mjs:14-26).

With a seed, values come from mulberry32 (random.mjs:4-12) and match the
reference's arrays for the same (n, low, high, seed). Without one the
reference uses Math.random; here an unseeded call draws its seed from the OS.
``randomNormalFloat32Array`` / ``randomNormalFloat64Array`` (an addition) give
standard normal values by Box-Muller over the same stream.
"""
from __future__ import annotations

import ctypes as ct
import os

import numpy as np

from . import _native as nat


def _seed(seed) -> int:
    if seed is None:
        return int.from_bytes(os.urandom(4), "little")
    return int(seed) & 0xFFFFFFFF  # JS `seed >>> 0`


def randomFloat32Array(n: int, low: float = -1.0, high: float = 1.0, seed=None) -> np.ndarray:
    out = np.empty(int(n), np.float32)
    nat.lib.wg_random_f32(out.ctypes.data_as(ct.POINTER(ct.c_float)), out.size, float(low), float(high),
                          _seed(seed))
    return out


def randomFloat64Array(n: int, low: float = -1.0, high: float = 1.0, seed=None) -> np.ndarray:
    out = np.empty(int(n), np.float64)
    nat.lib.wg_random_f64(out.ctypes.data_as(ct.POINTER(ct.c_double)), out.size, float(low), float(high),
                          _seed(seed))
    return out


def randomNormalFloat32Array(n: int, seed=None, out: np.ndarray | None = None) -> np.ndarray:
    out = np.empty(int(n), np.float32) if out is None else out
    nat.lib.wg_random_normal_f32(out.ctypes.data_as(ct.POINTER(ct.c_float)), int(n), _seed(seed))
    return out


def randomNormalFloat64Array(n: int, seed=None, out: np.ndarray | None = None) -> np.ndarray:
    out = np.empty(int(n), np.float64) if out is None else out
    nat.lib.wg_random_normal_f64(out.ctypes.data_as(ct.POINTER(ct.c_double)), int(n), _seed(seed))
    return out


def fill_uniform(out: np.ndarray, low: float = -1.0, high: float = 1.0, seed=None) -> np.ndarray:
    """randomFloat*Array into an existing (e.g. page-locked) array."""
    if out.dtype == np.float32:
        nat.lib.wg_random_f32(out.ctypes.data_as(ct.POINTER(ct.c_float)), out.size, float(low), float(high),
                              _seed(seed))
    elif out.dtype == np.float64:
        nat.lib.wg_random_f64(out.ctypes.data_as(ct.POINTER(ct.c_double)), out.size, float(low), float(high),
                              _seed(seed))
    else:
        raise TypeError("out must be float32 or float64")
    return out
