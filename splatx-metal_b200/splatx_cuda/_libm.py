"""The C library's float logf / expf / powf, so that the host-side schedule and init arithmetic
rounds exactly like the reference's C++ (std::log / std::exp / std::pow on float)."""
from __future__ import annotations

import ctypes as C
import ctypes.util

import numpy as np

_m = C.CDLL(ctypes.util.find_library("m") or "libm.so.6")
for _n in ("logf", "expf"):
    getattr(_m, _n).restype = C.c_float
    getattr(_m, _n).argtypes = [C.c_float]
_m.powf.restype = C.c_float
_m.powf.argtypes = [C.c_float, C.c_float]


def logf(x: float) -> float:
    return float(_m.logf(float(x)))


def expf(x: float) -> float:
    return float(_m.expf(float(x)))


def powf(x: float, y: float) -> float:
    return float(_m.powf(float(x), float(y)))


def logf_array(a) -> np.ndarray:
    a = np.asarray(a, np.float32).ravel()
    return np.array([_m.logf(float(v)) for v in a], np.float32)
