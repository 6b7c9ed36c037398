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
        L.oracle_threads.argtypes = [i32]
        L.oracle_threads.restype = i32
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


def threads(n: int = 0) -> int:
    """Set the OpenMP thread count of the C oracle (n > 0) and return the
    count in effect."""
    return int(lib().oracle_threads(int(n)))


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


def _bf16_round(a: np.ndarray) -> np.ndarray:
    from ml_dtypes import bfloat16

    return a.astype(np.float32).astype(bfloat16).astype(np.float64)


def moe_ffn_f64(fmt: int, w_gate: np.ndarray, w_up: np.ndarray, w_down: np.ndarray, x_bits: np.ndarray,
                ids: np.ndarray, weights: np.ndarray, hidden: int, inter: int, n_experts_local: int,
                expert_first: int = 0, ftz: bool = False) -> np.ndarray:
    """Reference MoE FFN in float64 over bf16-dequantized experts:
    y[t] = sum_j w[t][j] * Wd_e (bf16(silu(Wg_e x_t) * (Wu_e x_t))), h rounded to
    bf16 through float32 (as the device rounds an fp32 h), local experts only,
    slots summed in order.  Dequantizes one expert at a time."""
    from .formats import bf16_bits_to_f32, row_bytes

    T, topk = ids.shape
    x = bf16_bits_to_f32(x_bits).astype(np.float64)
    y = np.zeros((T, hidden), dtype=np.float64)
    gu_bytes = inter * row_bytes(fmt, hidden)
    d_bytes = hidden * row_bytes(fmt, inter)
    contrib = {}
    for e in sorted(set(int(v) for v in ids.reshape(-1))):
        le = e - expert_first
        if le < 0 or le >= n_experts_local:
            continue
        slots = [(t, j) for t in range(T) for j in range(topk) if ids[t, j] == e]
        wg = bf16_bits_to_f32(dequant_bf16(fmt, w_gate[le * gu_bytes:(le + 1) * gu_bytes], hidden, inter, ftz)).astype(np.float64)
        wu = bf16_bits_to_f32(dequant_bf16(fmt, w_up[le * gu_bytes:(le + 1) * gu_bytes], hidden, inter, ftz)).astype(np.float64)
        wd = bf16_bits_to_f32(dequant_bf16(fmt, w_down[le * d_bytes:(le + 1) * d_bytes], inter, hidden, ftz)).astype(np.float64)
        xs = x[[t for t, _ in slots]]
        g = xs @ wg.T
        u = xs @ wu.T
        h = _bf16_round(g / (1.0 + np.exp(-g)) * u)
        out = h @ wd.T
        for (t, j), row in zip(slots, out):
            contrib[(t, j)] = float(weights[t, j]) * row
    for t in range(T):
        for j in range(topk):
            if (t, j) in contrib:
                y[t] += contrib[(t, j)]
    return y
