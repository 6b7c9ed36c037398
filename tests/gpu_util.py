"""Helpers shared by the GPU tests: host <-> device copies of raw bytes and
bf16 bit patterns (torch provides only the device memory and streams)."""

from __future__ import annotations

import numpy as np


def dev_bytes(a: np.ndarray, pad: int = 0, offset: int = 0):
    """Copy a uint8 array to the device; optional leading offset (to build
    misaligned views) and trailing padding."""
    import torch

    buf = torch.zeros(offset + a.size + pad, dtype=torch.uint8, device="cuda")
    buf[offset : offset + a.size] = torch.from_numpy(np.ascontiguousarray(a, dtype=np.uint8)).cuda()
    return buf[offset:] if offset else buf


def dev_bf16(bits: np.ndarray):
    import torch

    t = torch.from_numpy(np.ascontiguousarray(bits, dtype=np.uint16).view(np.int16)).cuda()
    return t.view(torch.bfloat16)


def host_bits(t) -> np.ndarray:
    """bf16 tensor -> numpy uint16 bit patterns."""
    import torch

    return t.contiguous().view(torch.int16).cpu().numpy().view(np.uint16)


def strided_rows(raw: np.ndarray, N: int, row_bytes: int, stride: int) -> np.ndarray:
    """Re-lay dense rows at a larger stride (padding filled with 0xA5)."""
    out = np.full(N * stride, 0xA5, dtype=np.uint8)
    out.reshape(N, stride)[:, :row_bytes] = raw.reshape(N, row_bytes)
    return out


def tolerance_ok(y: np.ndarray, ref: np.ndarray, bf16_out: bool, rel_tol: float = 1e-3):
    """The stated MUL_MAT tolerance (rel_tol = 1e-3):
         |y - ref| <= 1e-3 * |ref| + 1e-3 * rms(ref)      (fp32 output)
       plus one bf16 rounding, 2^-8 * |ref|, for bf16 output.
    ref is the float64 dequant-then-matmul oracle.  Mirrors the reference's
    allclose(rtol=1e-3, atol=1e-3) (src/quants/tests/mmul.py:121), with the
    absolute term scaled to the output's magnitude."""
    ref = np.asarray(ref, dtype=np.float64)
    err = np.abs(np.asarray(y, dtype=np.float64) - ref)
    rms = float(np.sqrt(np.mean(ref * ref))) if ref.size else 0.0
    tol = rel_tol * np.abs(ref) + rel_tol * rms
    if bf16_out:
        tol = tol + 2.0**-8 * np.abs(ref)
    ok = bool(np.all(err <= tol))
    rel = float(np.max(err / (np.abs(ref) + rms))) if ref.size else 0.0
    return ok, rel
