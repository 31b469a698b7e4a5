"""ctypes binding to the reference's own ``fp4lib.c``, built unmodified into oracle/_ref/libfp4.so
by oracle/Makefile (test infrastructure only).

Argument conventions follow the reference binding (dsv41/ref/fp4lib.py:5-11): raw pointers and
``long`` sizes, the caller owns every buffer.
"""
import ctypes
import os

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "_ref", "libfp4.so")
_NEEDED_FLAGS = ("avx512f", "avx512bw", "avx512dq", "avx512vl", "avx512cd")
_lib = None


def cpu_supports() -> bool:
    try:
        flags = set()
        with open("/proc/cpuinfo") as f:
            for line in f:
                if line.startswith("flags"):
                    flags.update(line.split(":", 1)[1].split())
                    break
        return all(fl in flags for fl in _NEEDED_FLAGS)
    except OSError:
        return False


def available() -> bool:
    return os.path.exists(LIB_PATH) and cpu_supports()


def lib():
    global _lib
    if _lib is None:
        if not available():
            raise RuntimeError(f"reference fp4lib unavailable (built: {os.path.exists(LIB_PATH)}, "
                               f"AVX-512 host: {cpu_supports()})")
        L = ctypes.CDLL(LIB_PATH)
        L.dequant_fp4.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p,
                                  ctypes.c_long, ctypes.c_long]
        L.dequant_fp4.restype = None
        _lib = L
    return _lib


def dequant_fp4(q: np.ndarray, s: np.ndarray) -> np.ndarray:
    """q [rows, cols/2] uint8, s [rows, cols/32] e8m0 bytes -> float32 [rows, cols] via the reference C."""
    q = np.ascontiguousarray(q, dtype=np.uint8)
    s = np.ascontiguousarray(s, dtype=np.uint8)
    rows, half = q.shape
    assert s.shape == (rows, half * 2 // 32)
    out = np.empty((rows, half * 2), dtype=np.float32)
    lib().dequant_fp4(q.ctypes.data, s.ctypes.data, out.ctypes.data, rows, half * 2)
    return out
