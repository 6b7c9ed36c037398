"""Pin the CPU oracle (NumPy and C restatements) to the reference's own oracle.

Every expectation here was produced by the reference's NumPy oracle
(src/quants/tests/formats/*.py, mmul.py) via tests/golden/make_golden.py.
"""

from __future__ import annotations

import hashlib
import json
import re

import numpy as np
import pytest
from ml_dtypes import bfloat16

import oracle
from oracle import formats as F

from .conftest import GOLDEN, load_golden

FMTS = [F.Q4_0, F.Q8_0, F.Q6_K]


@pytest.mark.parametrize("fid", FMTS, ids=lambda f: F.NAMES[f])
@pytest.mark.parametrize("seed", [1, 2, 3])
def test_numpy_restatement_matches_reference_default_cases(fid, seed):
    g = load_golden(f"ref_default_{F.NAMES[fid]}_s{seed}.npz")
    K, N = int(g["K"]), int(g["N"])
    rows = F.dequant_bf16(fid, g["raw"], K, N)
    assert np.array_equal(F.to_reference_order(rows), g["expected_weights"])


@pytest.mark.parametrize("fid", FMTS, ids=lambda f: F.NAMES[f])
def test_c_oracle_matches_reference_default_cases(fid):
    for seed in (1, 2, 3):
        g = load_golden(f"ref_default_{F.NAMES[fid]}_s{seed}.npz")
        K, N = int(g["K"]), int(g["N"])
        rows = oracle.dequant_bf16(fid, g["raw"], K, N)
        assert np.array_equal(F.to_reference_order(rows), g["expected_weights"])


@pytest.mark.parametrize("fid", FMTS, ids=lambda f: F.NAMES[f])
def test_baseline_generators_match_reference_oracle(fid):
    g = load_golden(f"baseline_small_{F.NAMES[fid]}.npz")
    K, N = int(g["K"]), int(g["N"])
    # the generator is deterministic: regenerate and compare bytes too
    assert np.array_equal(F.generate(fid, K, N, seed=0), g["raw"])
    assert np.array_equal(F.dequant_bf16(fid, g["raw"], K, N), g["expected"])
    assert np.array_equal(oracle.dequant_bf16(fid, g["raw"], K, N), g["expected"])


@pytest.mark.parametrize("fid", FMTS, ids=lambda f: F.NAMES[f])
def test_edge_cases_and_flush_to_zero(fid):
    g = load_golden(f"edge_{F.NAMES[fid]}.npz")
    K, N = int(g["K"]), int(g["N"])
    for ftz, key in ((False, "expected"), (True, "expected_ftz")):
        assert np.array_equal(F.dequant_bf16(fid, g["raw"], K, N, ftz=ftz), g[key]), (ftz, "numpy")
        assert np.array_equal(oracle.dequant_bf16(fid, g["raw"], K, N, ftz=ftz), g[key]), (ftz, "C")


@pytest.mark.parametrize("key", sorted(json.loads((GOLDEN / "hashes.json").read_text())))
def test_c_oracle_full_size_digests(key):
    """Full BASELINE sizes: the C oracle reproduces the reference oracle's
    output digest (computed by the reference's per-block NumPy loop)."""
    ref = json.loads((GOLDEN / "hashes.json").read_text())[key]
    m = re.fullmatch(r"(\w+?)_K(\d+)_N(\d+)_seed0", key)
    name, K, N = m.group(1), int(m.group(2)), int(m.group(3))
    fid = F.BY_NAME[name]
    raw = F.generate(fid, K, N, seed=0)
    assert hashlib.sha256(raw.tobytes()).hexdigest() == ref["raw_sha256"]
    out = oracle.dequant_bf16(fid, raw, K, N)
    assert hashlib.sha256(out.tobytes()).hexdigest() == ref["bf16_rows_sha256"]


@pytest.mark.parametrize("fid", FMTS, ids=lambda f: F.NAMES[f])
def test_mmul_expectation_matches_reference(fid):
    """The reference's fused-mmul expectation (mmul.py:104-121) equals our
    matmul oracle on the same bf16 weights; the tiled input layout
    [K/8][4][8] is decoded correctly."""
    g = load_golden(f"ref_default_{F.NAMES[fid]}_s1.npz")
    K, N = int(g["K"]), int(g["N"])
    tiled = g["inputs_tiled"].reshape(K // 8, 4, 8)
    x_bits = np.ascontiguousarray(tiled.transpose(1, 0, 2)).reshape(4, K)
    assert np.array_equal(F.bf16_bits_to_f32(x_bits), g["inputs_rows"])
    y64 = oracle.mul_mat_f64(fid, g["raw"], x_bits, K, N)
    np.testing.assert_allclose(y64, g["expected_outputs"], rtol=1e-6, atol=1e-6)
    y32 = oracle.mul_mat_f32(fid, g["raw"], x_bits, K, N)
    np.testing.assert_allclose(y32, g["expected_outputs"], rtol=1e-5, atol=1e-5)


def test_f32_to_bf16_is_ml_dtypes_rne():
    rng = np.random.default_rng(0)
    bits = rng.integers(0, 2**32, size=200_000, dtype=np.uint64).astype(np.uint32)
    # force many exact ties and near-ties
    bits[:50_000] = (bits[:50_000] & 0xFFFF0000) | 0x8000
    bits[50_000:60_000] = (bits[50_000:60_000] & 0xFFFF0000) | 0x7FFF
    f = bits.view(np.float32)
    want = f.astype(bfloat16).view(np.uint16)
    L = oracle.lib()
    got = np.array([L.oracle_f32_to_bf16(float(v)) for v in f[:20_000]], dtype=np.uint16)
    finite = np.isfinite(f[:20_000])
    assert np.array_equal(got[finite], want[:20_000][finite])
    nan = np.isnan(f[:20_000])
    assert np.all(np.isnan(got[nan].view(bfloat16).astype(np.float32)))


def test_fp16_decode_exhaustive():
    L = oracle.lib()
    h = np.arange(65536, dtype=np.uint32).astype(np.uint16)
    want = h.view(np.float16).astype(np.float32)
    got = np.array([L.oracle_fp16_to_f32(int(v), 0) for v in h], dtype=np.float32)
    fin = np.isfinite(want)
    assert np.array_equal(got[fin].view(np.uint32), want[fin].view(np.uint32))
    assert np.array_equal(np.isnan(got), np.isnan(want))
    ftz = np.array([L.oracle_fp16_to_f32(int(v), 1) for v in h], dtype=np.float32)
    sub = ((h & 0x7C00) == 0) & ((h & 0x03FF) != 0)
    assert np.all(ftz[sub].view(np.uint32) == 0)  # subnormal -> +0
    assert np.array_equal(ftz[~sub & fin].view(np.uint32), want[~sub & fin].view(np.uint32))


def test_q6_k_encoder_roundtrip():
    rng = np.random.default_rng(3)
    q6 = rng.integers(0, 64, size=(5, 256), dtype=np.uint8)
    sc = rng.integers(-128, 128, size=(5, 16), dtype=np.int16).astype(np.int8)
    d = np.ones(5, dtype=np.float16)
    raw = F.encode_q6_k(q6, sc, d).reshape(-1)
    vals = F.dequant_f32(F.Q6_K, raw, 256, 5)
    expect = (q6.astype(np.int32) - 32) * np.repeat(sc.astype(np.int32), 16, axis=1)
    assert np.array_equal(vals, expect.astype(np.float32))


def test_moe_oracle_matches_a_plain_loop():
    """oracle.moe_ffn_f64 (C dequant, per-expert batching) against a per-slot
    loop over the NumPy restatement."""
    fid, E, H, I, T, topk = F.Q4_0, 6, 64, 32, 5, 3
    wg = F.gen_experts(fid, E, I, H, seed=1)
    wu = F.gen_experts(fid, E, I, H, seed=2)
    wd = F.gen_experts(fid, E, H, I, seed=3)
    x = F.gen_activations(T, H, seed=4)
    ids, w = F.gen_routing(T, E, topk, seed=5)
    got = oracle.moe_ffn_f64(fid, wg, wu, wd, x, ids, w, H, I, E)
    gu, dd = I * F.row_bytes(fid, H), H * F.row_bytes(fid, I)
    xf = F.bf16_bits_to_f32(x).astype(np.float64)
    want = np.zeros((T, H))
    for t in range(T):
        for j in range(topk):
            e = int(ids[t, j])
            Wg = F.bf16_bits_to_f32(F.dequant_bf16(fid, wg[e * gu:(e + 1) * gu], H, I)).astype(np.float64)
            Wu = F.bf16_bits_to_f32(F.dequant_bf16(fid, wu[e * gu:(e + 1) * gu], H, I)).astype(np.float64)
            Wd = F.bf16_bits_to_f32(F.dequant_bf16(fid, wd[e * dd:(e + 1) * dd], I, H)).astype(np.float64)
            g, u = Wg @ xf[t], Wu @ xf[t]
            h = (g / (1 + np.exp(-g)) * u).astype(np.float32).astype(bfloat16).astype(np.float64)
            want[t] += float(w[t, j]) * (Wd @ h)
    np.testing.assert_allclose(got, want, rtol=1e-12, atol=1e-12)
