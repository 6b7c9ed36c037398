"""Fused dequant-GEMM (prefill, M > 8) on the tcgen05 tensor cores.

Checked against the float64 dequant-then-matmul oracle with the stated
MUL_MAT tolerance (tests/gpu_util.tolerance_ok).  Full BASELINE config-3
shapes are checked on a seeded sample of output rows and columns (the full
float64 product of a 2048 x 14336 x 4096 GEMM is too slow for a test).
"""

from __future__ import annotations

import numpy as np
import pytest

import oracle
import spiral_b200 as sp
from oracle import formats as F

from .gpu_util import dev_bf16, dev_bytes, host_bits, tolerance_ok

pytestmark = pytest.mark.gpu
GEMM_FMTS = [F.Q4_0, F.Q8_0, F.Q6_K]


@pytest.mark.parametrize("fid", GEMM_FMTS, ids=lambda f: F.NAMES[f])
@pytest.mark.parametrize(
    "M,N,K",
    [
        (256, 128, 256),  # one tile, one K chunk
        (16, 128, 512),  # small M
        (300, 200, 768),  # partial token and feature blocks
        (512, 384, 1024),
    ],
)
def test_gemm_small_exact_shapes(cuda, fid, M, N, K):
    if K % F.BLOCK_K[fid]:
        pytest.skip("K not a block multiple")
    raw = F.generate(fid, K, N, seed=M + N + K)
    x = F.gen_activations(M, K, seed=K)
    ref = oracle.mul_mat_f64(fid, raw, x, K, N)
    y = sp.mul_mat(fid, dev_bytes(raw), dev_bf16(x), N, K, y_dtype=sp.F32).cpu().numpy()
    ok, rel = tolerance_ok(y, ref, bf16_out=False)
    assert ok, rel
    assert rel < 1e-5, rel
    yb = host_bits(sp.mul_mat(fid, dev_bytes(raw), dev_bf16(x), N, K, y_dtype=sp.BF16))
    ok, rel = tolerance_ok(F.bf16_bits_to_f32(yb), ref, bf16_out=True)
    assert ok, rel


def _sampled_reference(fid, raw, x_bits, K, N, rows, cols):
    w = oracle.dequant_bf16(fid, raw, K, N)[cols]
    wf = F.bf16_bits_to_f32(w).astype(np.float64)
    xf = F.bf16_bits_to_f32(x_bits[rows]).astype(np.float64)
    return xf @ wf.T


@pytest.mark.parametrize("fid", GEMM_FMTS, ids=lambda f: F.NAMES[f])
@pytest.mark.parametrize("M,N", [(512, 4096), (512, 14336), (2048, 4096), (2048, 14336)])
def test_gemm_baseline_config3(cuda, fid, M, N):
    K = 4096
    raw = F.generate(fid, K, N, seed=3)
    x = F.gen_activations(M, K, seed=4)
    y = host_bits(sp.mul_mat(fid, dev_bytes(raw), dev_bf16(x), N, K, y_dtype=sp.BF16))
    rng = np.random.default_rng(M + N)
    rows = np.sort(rng.choice(M, size=48, replace=False))
    cols = np.sort(rng.choice(N, size=320, replace=False))
    ref = _sampled_reference(fid, raw, x, K, N, rows, cols)
    got = F.bf16_bits_to_f32(y[np.ix_(rows, cols)])
    ok, rel = tolerance_ok(got, ref, bf16_out=True)
    assert ok, rel
    # every row and column block was written (no NaN / stale values)
    assert np.all(np.isfinite(F.bf16_bits_to_f32(y)))


def test_gemm_accumulate_and_strided_output(cuda):
    import torch

    fid, M, N, K = F.Q4_0, 96, 256, 512
    raw = F.generate(fid, K, N, seed=1)
    x = F.gen_activations(M, K, seed=2)
    y = torch.full((M, N + 16), 1.0, dtype=torch.float32, device="cuda")
    sp.mul_mat(fid, dev_bytes(raw), dev_bf16(x), N, K, y, y_dtype=sp.F32, y_row_stride=N + 16, accumulate=True)
    ref = oracle.mul_mat_f64(fid, raw, x, K, N) + 1.0
    got = y.cpu().numpy()
    ok, rel = tolerance_ok(got[:, :N], ref, bf16_out=False)
    assert ok, rel
    assert np.all(got[:, N:] == 1.0)
    assert sp.device_status() == 0


@pytest.mark.parametrize(
    "M,N,K",
    [
        (256, 128, 2048),  # one tile, 8 super-blocks per row (all 8 start phases)
        (300, 200, 4096),  # partial token and feature blocks
        (16, 130, 6144),
    ],
)
def test_gemm_q6_k_tensor_core_path(cuda, M, N, K):
    """Q6_K through the tcgen05 GEMM (K a multiple of 2048: rows of whole
    8-super-block runs), every 16-byte phase of a super-block start."""
    fid = F.Q6_K
    raw = F.generate(fid, K, N, seed=M + N + K)
    x = F.gen_activations(M, K, seed=K + 1)
    ref = oracle.mul_mat_f64(fid, raw, x, K, N)
    y = sp.mul_mat(fid, dev_bytes(raw), dev_bf16(x), N, K, y_dtype=sp.F32).cpu().numpy()
    ok, rel = tolerance_ok(y, ref, bf16_out=False)
    assert ok, rel
    assert rel < 5e-5, rel  # fp32 accumulation over K up to 6144
    assert sp.device_status() == 0


@pytest.mark.parametrize("fid", GEMM_FMTS, ids=lambda f: F.NAMES[f])
def test_gemm_is_bitwise_repeatable(cuda, fid):
    """Config 3's smallest shape (M = 512, N = 4096): repeated calls agree
    bit for bit, eagerly and as several calls inside one CUDA graph, and a
    sample of outputs is within the MUL_MAT tolerance."""
    import torch

    M, N, K = 512, 4096, 4096
    raw = F.generate(fid, K, N, seed=9)
    x = F.gen_activations(M, K, seed=10)
    w, xd = dev_bytes(raw), dev_bf16(x)
    first = sp.mul_mat(fid, w, xd, N, K, y_dtype=sp.F32).cpu().numpy()
    for _ in range(3):
        assert np.array_equal(sp.mul_mat(fid, w, xd, N, K, y_dtype=sp.F32).cpu().numpy(), first)
    ys = [torch.empty((M, N), dtype=torch.float32, device="cuda") for _ in range(3)]
    s = torch.cuda.Stream()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=s):
        for y in ys:
            sp.mul_mat(fid, w, xd, N, K, y, y_dtype=sp.F32, stream=s)
    g.replay()
    torch.cuda.synchronize()
    del g
    for y in ys:
        assert np.array_equal(y.cpu().numpy(), first)
    rng = np.random.default_rng(1)
    rows = np.sort(rng.choice(M, size=32, replace=False))
    cols = np.sort(rng.choice(N, size=256, replace=False))
    ok, rel = tolerance_ok(first[np.ix_(rows, cols)], _sampled_reference(fid, raw, x, K, N, rows, cols), bf16_out=False)
    assert ok, rel
    assert sp.device_status() == 0
