"""CPU oracle for the spiral_b200 hot path.

TEST INFRASTRUCTURE ONLY.  Only tests/, __graft_entry__.smoke() and bench.py
(its cpu_baseline and --impl reference legs) may import this package, and only
as the checker or the timed CPU baseline.  The product library
(spiral_b200/libspiral_b200.so) never calls into it and has no CPU fallback.

* ``oracle.formats`` — NumPy restatement of the reference oracle plus the
  seeded BASELINE generators.
* ``oracle.lib()``   — ctypes handle to liboracle.so, the C/OpenMP
  restatement (oracle.c), built by ``make -C oracle``.
"""

from __future__ import annotations

import ctypes
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIB_PATH = HERE / "liboracle.so"
_lib = None


def build() -> Path:
    subprocess.run(["make", "-s", "-C", str(HERE), "liboracle.so"], check=True)
    return LIB_PATH


def lib():
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            build()
        L = ctypes.CDLL(str(LIB_PATH))
        i64, vp, i32 = ctypes.c_int64, ctypes.c_void_p, ctypes.c_int
        L.oracle_block_k.argtypes = [i32]
        L.oracle_block_k.restype = i64
        L.oracle_block_bytes.argtypes = [i32]
        L.oracle_block_bytes.restype = i64
        L.oracle_fp16_to_f32.argtypes = [ctypes.c_uint16, i32]
        L.oracle_fp16_to_f32.restype = ctypes.c_float
        L.oracle_f32_to_bf16.argtypes = [ctypes.c_float]
        L.oracle_f32_to_bf16.restype = ctypes.c_uint16
        for name in ("oracle_dequant_f32", "oracle_dequant_bf16"):
            f = getattr(L, name)
            f.argtypes = [i32, vp, i64, vp, i64, i64, i32, i32]
            f.restype = None
        for name in ("oracle_mul_mat_f64", "oracle_mul_mat_f32"):
            f = getattr(L, name)
            f.argtypes = [i32, vp, i64, vp, i64, vp, i64, i64, i64, i32, i32]
            f.restype = None
        _lib = L
    return _lib


def _ptr(a: np.ndarray) -> int:
    return a.ctypes.data


def dequant_bf16(fmt: int, raw: np.ndarray, K: int, N: int, ftz: bool = False, threads: int = 0,
                 row_stride: int | None = None) -> np.ndarray:
    from .formats import row_bytes

    raw = np.ascontiguousarray(raw, dtype=np.uint8)
    out = np.empty((N, K), dtype=np.uint16)
    lib().oracle_dequant_bf16(fmt, _ptr(raw), row_stride or row_bytes(fmt, K), _ptr(out), K, N, int(ftz), threads)
    return out


def dequant_f32(fmt: int, raw: np.ndarray, K: int, N: int, ftz: bool = False, threads: int = 0) -> np.ndarray:
    from .formats import row_bytes

    raw = np.ascontiguousarray(raw, dtype=np.uint8)
    out = np.empty((N, K), dtype=np.float32)
    lib().oracle_dequant_f32(fmt, _ptr(raw), row_bytes(fmt, K), _ptr(out), K, N, int(ftz), threads)
    return out


def mul_mat_f64(fmt: int, raw: np.ndarray, x_bits: np.ndarray, K: int, N: int, ftz: bool = False,
                threads: int = 0) -> np.ndarray:
    from .formats import row_bytes

    raw = np.ascontiguousarray(raw, dtype=np.uint8)
    x = np.ascontiguousarray(x_bits, dtype=np.uint16)
    M = x.shape[0]
    y = np.empty((M, N), dtype=np.float64)
    lib().oracle_mul_mat_f64(fmt, _ptr(raw), row_bytes(fmt, K), _ptr(x), x.shape[1], _ptr(y), M, N, K, int(ftz),
                             threads)
    return y


def mul_mat_f32(fmt: int, raw: np.ndarray, x_bits: np.ndarray, K: int, N: int, ftz: bool = False,
                threads: int = 0) -> np.ndarray:
    from .formats import row_bytes

    raw = np.ascontiguousarray(raw, dtype=np.uint8)
    x = np.ascontiguousarray(x_bits, dtype=np.uint16)
    M = x.shape[0]
    y = np.empty((M, N), dtype=np.float32)
    lib().oracle_mul_mat_f32(fmt, _ptr(raw), row_bytes(fmt, K), _ptr(x), x.shape[1], _ptr(y), M, N, K, int(ftz),
                             threads)
    return y
