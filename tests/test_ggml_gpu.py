"""The ggml backend boundary (spiral_ggml_mul_mat / supports_mul_mat): a
GGML_OP_MUL_MAT node given as ggml tensor descriptors (type, ne, nb, data)
with src0 broadcast over the batch dims, checked per batch against
spiral_mul_mat (bit for bit) and against the float64 oracle."""

from __future__ import annotations

import numpy as np
import pytest

import oracle
import spiral_b200 as sp
from oracle import formats as F

from .gpu_util import dev_bf16, dev_bytes, tolerance_ok

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("fid", [F.Q4_0, F.Q8_0, F.Q6_K], ids=lambda f: F.NAMES[f])
def test_ggml_mul_mat_batched_broadcast(cuda, fid):
    import torch

    K, N, M = 2048, 96, 3
    ne02, ne03, ne12, ne13 = 2, 1, 4, 2  # src0 broadcast: r2 = 2, r3 = 2
    rb = F.row_bytes(fid, K)
    raws = [F.generate(fid, K, N, seed=70 + i) for i in range(ne02 * ne03)]
    w = dev_bytes(np.concatenate(raws))
    xs = F.gen_activations(ne12 * ne13 * M, K, seed=80)
    x = dev_bf16(xs)
    y = torch.zeros(ne12 * ne13 * M * N, dtype=torch.float32, device="cuda")
    src0 = sp.ggml_tensor(fid, (K, N, ne02, ne03), (F.BLOCK_BYTES[fid], rb, rb * N, rb * N * ne02), w)
    src1 = sp.ggml_tensor(sp.BF16, (K, M, ne12, ne13), (2, 2 * K, 2 * K * M, 2 * K * M * ne12), x)
    dst = sp.ggml_tensor(sp.F32, (N, M, ne12, ne13), (4, 4 * N, 4 * N * M, 4 * N * M * ne12), y)
    assert sp.ggml_supports_mul_mat(src0, src1, dst)
    sp.ggml_mul_mat(src0, src1, dst)
    got = y.cpu().numpy().reshape(ne13, ne12, M, N)
    for i3 in range(ne13):
        for i2 in range(ne12):
            a = (i3 // (ne13 // ne03)) * ne02 + i2 // (ne12 // ne02)
            xb = xs.reshape(ne13, ne12, M, K)[i3, i2]
            want = sp.mul_mat(fid, dev_bytes(raws[a]), dev_bf16(xb), N, K, y_dtype=sp.F32).cpu().numpy()
            assert np.array_equal(got[i3, i2], want), (i3, i2)
            ok, rel = tolerance_ok(got[i3, i2], oracle.mul_mat_f64(fid, raws[a], xb, K, N), bf16_out=False)
            assert ok, rel
    assert sp.device_status() == 0
