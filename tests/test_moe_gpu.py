"""MoE FFN decode layer (SwiGLU experts with Q4_0
gate/up/down, top-8 routing) on the GPU against the float64 oracle
(oracle.moe_ffn_f64).

Tolerance: the MUL_MAT rule |y - ref| <= tol*|ref| + tol*rms(ref) with
tol = 2e-3 (1e-3 for a single MUL_MAT).  The layer chains two quantized
products through a bf16 intermediate h, rounded from fp32 on the device and
from float64 in the oracle, and sums up to 8 weighted expert outputs whose
signs may cancel, so it carries about twice the single-product error."""

from __future__ import annotations

import numpy as np
import pytest

import oracle
import spiral_b200 as sp
from oracle import formats as F

from .gpu_util import dev_bf16, dev_bytes, host_bits, tolerance_ok as _tolerance_ok


def tolerance_ok(y, ref, bf16_out):
    return _tolerance_ok(y, ref, bf16_out, rel_tol=2e-3)

pytestmark = pytest.mark.gpu


def _case(fid, E, H, I, T, topk, seed):
    wg = F.gen_experts(fid, E, I, H, seed=seed)
    wu = F.gen_experts(fid, E, I, H, seed=seed + 1)
    wd = F.gen_experts(fid, E, H, I, seed=seed + 2)
    x = F.gen_activations(T, H, seed=seed + 3)
    ids, w = F.gen_routing(T, E, topk, seed=seed + 4)
    return wg, wu, wd, x, ids, w


def _run(fid, wg, wu, wd, x, ids, w, H, I, E_local, e0=0, y_dtype=sp.F32):
    import torch

    return sp.moe_ffn(fid, dev_bytes(wg), dev_bytes(wu), dev_bytes(wd), dev_bf16(x),
                      torch.from_numpy(ids).cuda(), torch.from_numpy(w).cuda(), hidden=H, inter=I,
                      n_experts_local=E_local, expert_first=e0, y_dtype=y_dtype)


@pytest.mark.parametrize("fid", [F.Q4_0, F.Q8_0], ids=lambda f: F.NAMES[f])
@pytest.mark.parametrize("E,H,I,T,topk", [(16, 256, 256, 1, 4), (16, 512, 256, 5, 4), (8, 256, 512, 17, 8),
                                          (4, 256, 256, 40, 2)])
def test_moe_small(cuda, fid, E, H, I, T, topk):
    wg, wu, wd, x, ids, w = _case(fid, E, H, I, T, topk, seed=E + H + T)
    y = _run(fid, wg, wu, wd, x, ids, w, H, I, E).cpu().numpy()
    ref = oracle.moe_ffn_f64(fid, wg, wu, wd, x, ids, w, H, I, E)
    ok, rel = tolerance_ok(y, ref, bf16_out=False)
    assert ok, rel
    assert sp.device_status() == 0


def test_moe_q6_k(cuda):
    fid, E, H, I, T, topk = F.Q6_K, 4, 2048, 2048, 3, 2
    wg, wu, wd, x, ids, w = _case(fid, E, H, I, T, topk, seed=7)
    y = _run(fid, wg, wu, wd, x, ids, w, H, I, E).cpu().numpy()
    ok, rel = tolerance_ok(y, oracle.moe_ffn_f64(fid, wg, wu, wd, x, ids, w, H, I, E), bf16_out=False)
    assert ok, rel


@pytest.mark.parametrize("T", [1, 8, 64])
def test_moe_baseline_config4(cuda, T):
    """128 experts, hidden 2048, intermediate 768, top-8, Q4_0, bf16 output;
    bitwise repeatable."""
    fid, E, H, I, topk = F.Q4_0, 128, 2048, 768, 8
    wg, wu, wd, x, ids, w = _case(fid, E, H, I, T, topk, seed=40)
    y = host_bits(_run(fid, wg, wu, wd, x, ids, w, H, I, E, y_dtype=sp.BF16))
    ref = oracle.moe_ffn_f64(fid, wg, wu, wd, x, ids, w, H, I, E)
    ok, rel = tolerance_ok(F.bf16_bits_to_f32(y), ref, bf16_out=True)
    assert ok, rel
    y2 = host_bits(_run(fid, wg, wu, wd, x, ids, w, H, I, E, y_dtype=sp.BF16))
    assert np.array_equal(y, y2)
    assert sp.device_status() == 0


def test_moe_expert_parallel_partials_sum_to_full(cuda):
    """Two expert ranges computed separately (as two ranks would) add up to
    the whole layer; ids outside a range are skipped."""
    fid, E, H, I, T, topk = F.Q4_0, 16, 512, 256, 9, 4
    wg, wu, wd, x, ids, w = _case(fid, E, H, I, T, topk, seed=3)
    full = _run(fid, wg, wu, wd, x, ids, w, H, I, E).cpu().numpy()
    gu, dd = I * F.row_bytes(fid, H), H * F.row_bytes(fid, I)
    half = E // 2
    parts = []
    for r in range(2):
        sl = slice(r * half, (r + 1) * half)
        parts.append(_run(fid, wg[sl.start * gu:sl.stop * gu], wu[sl.start * gu:sl.stop * gu],
                          wd[sl.start * dd:sl.stop * dd], x, ids, w, H, I, half, e0=r * half).cpu().numpy())
        ref_r = oracle.moe_ffn_f64(fid, wg[sl.start * gu:sl.stop * gu], wu[sl.start * gu:sl.stop * gu],
                                   wd[sl.start * dd:sl.stop * dd], x, ids, w, H, I, half, expert_first=r * half)
        ok, rel = tolerance_ok(parts[-1], ref_r, bf16_out=False)
        assert ok, rel
    ok, rel = tolerance_ok(parts[0] + parts[1], full, bf16_out=False)
    assert ok, rel


@pytest.mark.parametrize("fid", [F.Q4_0, F.Q8_0], ids=lambda f: F.NAMES[f])
@pytest.mark.parametrize("e0", [0, 4])
def test_moe_few_pairs_repeated_and_foreign_experts(cuda, fid, e0):
    """T * topk <= 16 pairs (each pair its own problem, no routing kernel):
    an expert picked twice by one token and by both tokens, ids outside the
    local range (skipped), a local range that starts past expert 0, and a
    token with no local expert (its output is the empty sum); bitwise
    repeatable."""
    E, H, I, T, topk = 12, 2048, 768, 2, 8
    wg, wu, wd, x, _, w = _case(fid, E, H, I, T, topk, seed=61)
    ids = np.array([[5, 5, 7, 9, 4, 11, 6, 8],
                    [7, -1, 15, 5, 9, 100, 10, 4]], dtype=np.int32)
    if e0:
        ids[1] = [0, 1, 2, 3, -1, 20, 1, 0]  # no expert of [e0, e0 + E_local)
    E_local = E - e0
    gu, dd = I * F.row_bytes(fid, H), H * F.row_bytes(fid, I)
    wgl, wul, wdl = wg[e0 * gu:], wu[e0 * gu:], wd[e0 * dd:]
    y = _run(fid, wgl, wul, wdl, x, ids, w, H, I, E_local, e0=e0).cpu().numpy()
    ref = oracle.moe_ffn_f64(fid, wgl, wul, wdl, x, ids, w, H, I, E_local, expert_first=e0)
    ok, rel = tolerance_ok(y, ref, bf16_out=False)
    assert ok, rel
    if e0:
        assert not y[1].any()
    y2 = _run(fid, wgl, wul, wdl, x, ids, w, H, I, E_local, e0=e0).cpu().numpy()
    assert np.array_equal(y, y2)
    assert sp.device_status() == 0
