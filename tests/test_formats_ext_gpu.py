"""Extended GGUF formats on the GPU (Q4_K, Q5_K, IQ4_NL, IQ4_XS, F16, BF16):
spiral_dequant_bf16 bit for bit against the NumPy oracle of
oracle/formats_ext.py (ggml's published layouts; parity unpinned: the
reference has no code for these formats), with random blocks, edge scales
and strided / unaligned destinations; spiral_mul_mat within the MUL_MAT
tolerance of the float64 oracle for 1..8 vectors and for more (batched);
the ggml boundary serving the new types."""

from __future__ import annotations

import numpy as np
import pytest

import spiral_b200 as sp
from oracle import formats_ext as X

from .gpu_util import dev_bf16, dev_bytes, host_bits, tolerance_ok

pytestmark = pytest.mark.gpu

EXT = (X.Q4_K, X.Q5_K, X.IQ4_NL, X.IQ4_XS, X.F16, X.BF16)


def _edge_blocks(fmt: int, raw: np.ndarray) -> np.ndarray:
    """Overwrite a few blocks' fp16 scales with edge values: +0, -0,
    negative, subnormal, the largest finite."""
    if fmt in (X.F16, X.BF16):
        return raw
    bb = X.BLOCK_BYTES[fmt]
    out = raw.copy().reshape(-1, bb)
    edge = np.array([0x0000, 0x8000, 0xBC00, 0x0001, 0x03FF, 0x7BFF, 0xC500], dtype=np.uint16)
    n = min(len(edge), out.shape[0])
    out[:n, 0:2] = edge[:n].view(np.uint8).reshape(n, 2)
    if fmt in (X.Q4_K, X.Q5_K):  # and dmin
        out[:n, 2:4] = np.ascontiguousarray(edge[::-1][:n]).view(np.uint8).reshape(n, 2)
    return out.reshape(-1)


@pytest.mark.parametrize("fmt", EXT, ids=lambda f: X.NAMES[f])
@pytest.mark.parametrize("ftz", [False, True])
def test_ext_dequant_bit_exact(cuda, fmt, ftz):
    import torch

    K, N = 1024, 37
    raw = _edge_blocks(fmt, X.generate(fmt, K, N, seed=fmt + 100))
    want = X.dequant_bf16(fmt, raw, K, N, ftz=ftz)
    out = torch.empty((N, K), dtype=torch.bfloat16, device="cuda")
    sp.dequant_bf16(fmt, dev_bytes(raw), K, N, out, ftz=ftz)
    got = host_bits(out)
    bad = np.argwhere(got != want)
    assert bad.size == 0, (X.NAMES[fmt], bad[:5], got[tuple(bad[0])] if bad.size else None)
    assert sp.device_status() == 0


@pytest.mark.parametrize("fmt", EXT, ids=lambda f: X.NAMES[f])
def test_ext_dequant_strided_unaligned(cuda, fmt):
    """Row stride larger than the row, and an output at a 2-byte offset with
    an odd row stride (2-byte store path)."""
    import torch

    K, N = 512, 9
    rb = X.row_bytes(fmt, K)
    raw = X.generate(fmt, K, N, seed=fmt + 200)
    stride = rb + 6
    padded = np.full(N * stride, 0x5A, dtype=np.uint8)
    padded.reshape(N, stride)[:, :rb] = raw.reshape(N, rb)
    buf = torch.zeros(N * (K + 3) + 1, dtype=torch.int16, device="cuda")
    out = buf[1:].view(torch.bfloat16)
    sp.dequant_bf16(fmt, dev_bytes(padded), K, N, out, w_row_stride=stride, out_row_stride=K + 3)
    got = out.view(torch.int16).cpu().numpy().view(np.uint16)
    got = np.stack([got[n * (K + 3) : n * (K + 3) + K] for n in range(N)])
    assert np.array_equal(got, X.dequant_bf16(fmt, raw, K, N))


@pytest.mark.parametrize("fmt", EXT, ids=lambda f: X.NAMES[f])
@pytest.mark.parametrize("M", [1, 5, 8, 19])
def test_ext_mul_mat_tolerance(cuda, fmt, M):
    K, N = 2048, 300
    raw = X.generate(fmt, K, N, seed=fmt + M)
    from oracle import formats as F

    x = F.gen_activations(M, K, seed=M + 7)
    ref = X.mul_mat_f64(fmt, raw, x, K, N)
    y = sp.mul_mat(fmt, dev_bytes(raw), dev_bf16(x), N, K, y_dtype=sp.F32).cpu().numpy()
    ok, rel = tolerance_ok(y, ref, bf16_out=False)
    assert ok, (X.NAMES[fmt], rel)
    yb = sp.mul_mat(fmt, dev_bytes(raw), dev_bf16(x), N, K, y_dtype=sp.BF16).float().cpu().numpy()
    ok, rel = tolerance_ok(yb, ref, bf16_out=True)
    assert ok, (X.NAMES[fmt], rel)
    assert sp.device_status() == 0


def test_ext_ggml_boundary(cuda):
    import torch

    fmt, K, N, M = X.Q4_K, 512, 64, 3
    raw = X.generate(fmt, K, N, seed=5)
    from oracle import formats as F

    x = F.gen_activations(M, K, seed=6)
    w, xd = dev_bytes(raw), dev_bf16(x)
    y = torch.zeros((M, N), dtype=torch.float32, device="cuda")
    rb = X.row_bytes(fmt, K)
    a = sp.ggml_tensor(fmt, [K, N, 1, 1], [X.BLOCK_BYTES[fmt], rb, rb * N, rb * N], w)
    b = sp.ggml_tensor(sp.BF16, [K, M, 1, 1], [2, 2 * K, 2 * K * M, 2 * K * M], xd)
    d = sp.ggml_tensor(sp.F32, [N, M, 1, 1], [4, 4 * N, 4 * N * M, 4 * N * M], y)
    assert sp.ggml_supports_mul_mat(a, b, d)
    sp.ggml_mul_mat(a, b, d)
    ok, rel = tolerance_ok(y.cpu().numpy(), X.mul_mat_f64(fmt, raw, x, K, N), bf16_out=False)
    assert ok, rel
