"""NumPy restatement of the reference's GGUF format oracle, plus generators.

TEST INFRASTRUCTURE ONLY: the checker for the CUDA library and the source of
seeded synthetic inputs.  Nothing on the product path imports this module.

Restated from the reference's NumPy oracle (read, not copied; vectorised over
blocks instead of the reference's per-block Python loop):

* Q4_0  src/quants/tests/formats/q4_0.py:42-62   value = (q - 8) * d
* Q8_0  src/quants/tests/formats/q8_0.py:43-60   value = q * d
* Q6_K  src/quants/tests/formats/q6_k.py:55-112  value = d * sc * (q - 32)
* bf16  reference_weights(...).astype(ml_dtypes.bfloat16)  (RNE)
* order reference_weights' [cols_tile][rows_record][chunk][rows][8] stream,
        which flattens to [N/8][K][8]   (q4_0.py:65-79)

Layouts here are ggml row-major: `values[n, k]` for output feature n.  The
generators draw the BASELINE distributions (seeded PCG64, numpy
default_rng):

* Q4_0  d = fp16(|N(0,1)| * 0.02), q ~ U{0..15}
* Q8_0  d = fp16(|N(0,1)| * 0.01), q ~ U{-127..127}
* Q6_K  d = fp16(|N(0,1)| * 0.001), 6-bit q ~ U{0..63}, sc ~ U{-64..63}
"""

from __future__ import annotations

import numpy as np
from ml_dtypes import bfloat16

Q4_0, Q8_0, Q6_K = 2, 8, 14
NAMES = {Q4_0: "q4_0", Q8_0: "q8_0", Q6_K: "q6_k"}
BY_NAME = {v: k for k, v in NAMES.items()}
BLOCK_K = {Q4_0: 32, Q8_0: 32, Q6_K: 256}
BLOCK_BYTES = {Q4_0: 18, Q8_0: 34, Q6_K: 210}


def fmt_id(fmt) -> int:
    return BY_NAME[fmt] if isinstance(fmt, str) else int(fmt)


def row_bytes(fmt, K: int) -> int:
    f = fmt_id(fmt)
    return (K // BLOCK_K[f]) * BLOCK_BYTES[f]


# --------------------------------------------------------------- generators


def _fp16_abs_normal(rng, n: int, scale: float) -> np.ndarray:
    return (np.abs(rng.standard_normal(n)) * scale).astype(np.float16)


def gen_q4_0(K: int, N: int, seed: int) -> np.ndarray:
    """Canonical Q4_0 bytes, N rows of K/32 blocks."""
    assert K % 32 == 0
    rng = np.random.default_rng(seed)
    nb = N * (K // 32)
    d = _fp16_abs_normal(rng, nb, 0.02)
    q = rng.integers(0, 16, size=(nb, 32), dtype=np.uint8)
    blk = np.empty((nb, 18), dtype=np.uint8)
    blk[:, 0:2] = d.view(np.uint8).reshape(nb, 2)
    blk[:, 2:] = q[:, :16] | (q[:, 16:] << 4)
    return blk.reshape(-1)


def gen_q8_0(K: int, N: int, seed: int) -> np.ndarray:
    """Canonical Q8_0 bytes."""
    assert K % 32 == 0
    rng = np.random.default_rng(seed)
    nb = N * (K // 32)
    d = _fp16_abs_normal(rng, nb, 0.01)
    q = rng.integers(-127, 128, size=(nb, 32), dtype=np.int8)
    blk = np.empty((nb, 34), dtype=np.uint8)
    blk[:, 0:2] = d.view(np.uint8).reshape(nb, 2)
    blk[:, 2:] = q.view(np.uint8)
    return blk.reshape(-1)


def encode_q6_k(q6: np.ndarray, sc: np.ndarray, d: np.ndarray) -> np.ndarray:
    """Pack 6-bit quants [nsb,256] (0..63), int8 scales [nsb,16] and fp16 d
    [nsb] into canonical 210-byte super-blocks (inverse of q6_k.py:55-97)."""
    nsb = q6.shape[0]
    blk = np.zeros((nsb, 210), dtype=np.uint8)
    q6 = q6.astype(np.uint8)
    for h in range(2):
        q1 = q6[:, 128 * h + 0 : 128 * h + 32]
        q2 = q6[:, 128 * h + 32 : 128 * h + 64]
        q3 = q6[:, 128 * h + 64 : 128 * h + 96]
        q4 = q6[:, 128 * h + 96 : 128 * h + 128]
        blk[:, 64 * h : 64 * h + 32] = (q1 & 15) | ((q3 & 15) << 4)
        blk[:, 64 * h + 32 : 64 * h + 64] = (q2 & 15) | ((q4 & 15) << 4)
        blk[:, 128 + 32 * h : 128 + 32 * h + 32] = (
            (q1 >> 4) | ((q2 >> 4) << 2) | ((q3 >> 4) << 4) | ((q4 >> 4) << 6)
        )
    blk[:, 192:208] = sc.astype(np.int8).view(np.uint8)
    blk[:, 208:210] = d.astype(np.float16).view(np.uint8).reshape(nsb, 2)
    return blk


def gen_q6_k(K: int, N: int, seed: int) -> np.ndarray:
    """Canonical Q6_K bytes."""
    assert K % 256 == 0
    rng = np.random.default_rng(seed)
    nsb = N * (K // 256)
    q6 = rng.integers(0, 64, size=(nsb, 256), dtype=np.uint8)
    sc = rng.integers(-64, 64, size=(nsb, 16), dtype=np.int8)
    d = _fp16_abs_normal(rng, nsb, 0.001)
    return encode_q6_k(q6, sc, d).reshape(-1)


GENERATORS = {Q4_0: gen_q4_0, Q8_0: gen_q8_0, Q6_K: gen_q6_k}


def generate(fmt, K: int, N: int, seed: int) -> np.ndarray:
    return GENERATORS[fmt_id(fmt)](K, N, seed)


def gen_activations(M: int, K: int, seed: int) -> np.ndarray:
    """bf16 N(0,1) activations [M][K] as uint16 bits."""
    rng = np.random.default_rng(seed)
    return rng.standard_normal((M, K)).astype(np.float32).astype(bfloat16).view(np.uint16)


# ---------------------------------------------------------------- dequant


def _fp16_to_f32(bits: np.ndarray, ftz: bool) -> np.ndarray:
    d = bits.view(np.float16).astype(np.float32)
    if ftz:  # subnormal -> +0, as the reference repack stores it (repack.h:29-34)
        d = np.where(((bits & 0x7C00) == 0) & ((bits & 0x03FF) != 0), np.float32(0.0), d)
    return d


def dequant_f32(fmt, raw: np.ndarray, K: int, N: int, ftz: bool = False, row_stride: int | None = None):
    """values[n, k] in float32 (exact products)."""
    f = fmt_id(fmt)
    bk, bb = BLOCK_K[f], BLOCK_BYTES[f]
    rb = row_bytes(f, K)
    raw = np.asarray(raw, dtype=np.uint8)
    if row_stride is not None and row_stride != rb:
        raw = raw[: N * row_stride].reshape(N, row_stride)[:, :rb]
    blk = np.ascontiguousarray(raw[: N * rb]).reshape(N * (K // bk), bb)
    if f == Q4_0:
        d = _fp16_to_f32(blk[:, 0:2].copy().view(np.uint16).reshape(-1), ftz)
        qs = blk[:, 2:18]
        q = np.concatenate([qs & 15, qs >> 4], axis=1).astype(np.float32)
        vals = (q - np.float32(8.0)) * d[:, None]
    elif f == Q8_0:
        d = _fp16_to_f32(blk[:, 0:2].copy().view(np.uint16).reshape(-1), ftz)
        vals = blk[:, 2:34].view(np.int8).astype(np.float32) * d[:, None]
    else:
        ql = blk[:, 0:128].astype(np.int32)
        qh = blk[:, 128:192].astype(np.int32)
        sc = blk[:, 192:208].view(np.int8).astype(np.int32)
        d = _fp16_to_f32(blk[:, 208:210].copy().view(np.uint16).reshape(-1), ftz)
        vals = np.empty((blk.shape[0], 256), dtype=np.float32)
        is_ = np.arange(32) // 16
        for h in range(2):
            lo, hi, qq = ql[:, 64 * h : 64 * h + 32], ql[:, 64 * h + 32 : 64 * h + 64], qh[:, 32 * h : 32 * h + 32]
            parts = (
                (lo & 15) | ((qq & 3) << 4),
                (hi & 15) | (((qq >> 2) & 3) << 4),
                (lo >> 4) | (((qq >> 4) & 3) << 4),
                (hi >> 4) | (((qq >> 6) & 3) << 4),
            )
            for s, q in enumerate(parts):
                scale = sc[:, 8 * h + 2 * s + is_].astype(np.float32)  # [nsb, 32]
                # (d * sc) * q in that order, as the reference evaluates it:
                # exact in float32, and the order fixes the sign of a zero.
                vals[:, 128 * h + 32 * s : 128 * h + 32 * s + 32] = (d[:, None] * scale) * (q - 32).astype(np.float32)
    return vals.reshape(N, K)


def dequant_bf16(fmt, raw, K: int, N: int, ftz: bool = False, row_stride: int | None = None) -> np.ndarray:
    """bf16 bits (uint16) [N][K] — ggml row-major dequantize."""
    return dequant_f32(fmt, raw, K, N, ftz, row_stride).astype(bfloat16).view(np.uint16)


def to_reference_order(w_rows: np.ndarray) -> np.ndarray:
    """[N][K] -> the reference's weights stream [N/8][K][8] (flattened)."""
    N, K = w_rows.shape
    return np.ascontiguousarray(w_rows.reshape(N // 8, 8, K).transpose(0, 2, 1)).reshape(-1)


def bf16_bits_to_f32(bits: np.ndarray) -> np.ndarray:
    return (np.asarray(bits, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def mul_mat_f64(fmt, raw, x_bits: np.ndarray, K: int, N: int, ftz: bool = False) -> np.ndarray:
    """y[m][n] = sum_k bf16(W[n][k]) * x[m][k] in float64 (mmul.py:104-112,
    at higher precision)."""
    w = bf16_bits_to_f32(dequant_bf16(fmt, raw, K, N, ftz)).astype(np.float64)
    x = bf16_bits_to_f32(x_bits).astype(np.float64)
    return x @ w.T



def gen_routing(T: int, n_experts: int, topk: int, seed: int):
    """BASELINE config 4 routing: per token topk distinct expert ids drawn
    uniformly, weights = softmax over topk N(0,1) logits (float32)."""
    rng = np.random.default_rng(seed)
    ids = np.stack([rng.choice(n_experts, size=topk, replace=False) for _ in range(T)]).astype(np.int32)
    logits = rng.standard_normal((T, topk))
    w = np.exp(logits - logits.max(axis=1, keepdims=True))
    w = (w / w.sum(axis=1, keepdims=True)).astype(np.float32)
    return ids, w


def gen_experts(fid: int, n_experts: int, rows: int, K: int, seed: int) -> np.ndarray:
    """n_experts canonical [rows][K] tensors back to back (BASELINE
    distributions)."""
    return np.concatenate([generate(fid, K, rows, seed=seed * 1000 + e) for e in range(n_experts)])
