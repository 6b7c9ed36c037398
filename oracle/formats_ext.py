"""NumPy oracle for the GGUF formats beyond the reference's three: Q4_K,
Q5_K, IQ4_NL, IQ4_XS and the F16 / BF16 pass-through types.

TEST INFRASTRUCTURE ONLY: the checker for the CUDA library's extended
formats and the source of their seeded synthetic inputs.  Nothing on the
product path imports this module.

The reference names these formats as its next step (src/quants/TODO.md:16-22,
80-130) but has no code for them, so there are no reference golden vectors:
parity for these formats is UNPINNED.  The block layouts and the dequant
arithmetic are restated from ggml's published GGUF format definitions
(ggml-common.h block_q4_K / block_q5_K / block_iq4_nl / block_iq4_xs and
ggml-quants.c dequantize_row_q4_K / _q5_K / _iq4_nl / _iq4_xs; the reference
pins no ggml version), evaluated with one IEEE float32 rounding per
operation in ggml's order and then rounded to bf16 (RNE):

* Q4_K   144 B / 256 weights: fp16 d, fp16 dmin, 12 bytes of packed 6-bit
         (scale, min) pairs for 8 sub-blocks of 32, 128 bytes of nibbles.
         y = (d*sc)*q - (dmin*m)
* Q5_K   176 B / 256 weights: as Q4_K plus qh[32] holding the fifth bit.
* IQ4_NL 18 B / 32 weights: fp16 d, 16 bytes of nibbles indexing a fixed
         16-entry codebook.  y = d * kvalues[q]
* IQ4_XS 136 B / 256 weights: fp16 d, 6-bit sub-block scales split over
         scales_h (2 bits each) and scales_l (4 bits each), 128 bytes of
         codebook nibbles.  y = (d * (ls - 32)) * kvalues[q]
* F16 / BF16: 2 bytes per weight; bf16 = RNE(f16) / unchanged.
"""

from __future__ import annotations

import numpy as np
from ml_dtypes import bfloat16

F32, F16, Q4_K, Q5_K, IQ4_NL, IQ4_XS, BF16 = 0, 1, 12, 13, 20, 23, 30
NAMES = {F16: "f16", Q4_K: "q4_k", Q5_K: "q5_k", IQ4_NL: "iq4_nl", IQ4_XS: "iq4_xs", BF16: "bf16"}
BY_NAME = {v: k for k, v in NAMES.items()}
BLOCK_K = {F16: 1, Q4_K: 256, Q5_K: 256, IQ4_NL: 32, IQ4_XS: 256, BF16: 1}
BLOCK_BYTES = {F16: 2, Q4_K: 144, Q5_K: 176, IQ4_NL: 18, IQ4_XS: 136, BF16: 2}

# The IQ4 codebook (ggml-common.h kvalues_iq4nl): a format constant.
KVALUES_IQ4 = np.array([-127, -104, -83, -65, -49, -35, -22, -10, 1, 13, 25, 38, 53, 69, 89, 113], dtype=np.int8)


def row_bytes(fmt: int, K: int) -> int:
    return (K // BLOCK_K[fmt]) * BLOCK_BYTES[fmt]


# --------------------------------------------------------------- generators


def _fp16_abs_normal(rng, n: int, scale: float) -> np.ndarray:
    return (np.abs(rng.standard_normal(n)) * scale).astype(np.float16)


def pack_scale_min_k4(sc: np.ndarray, m: np.ndarray) -> np.ndarray:
    """[nb, 8] 6-bit scales and mins -> the 12 packed bytes of a K-quant
    super-block (inverse of get_scale_min_k4)."""
    sc = sc.astype(np.uint8)
    m = m.astype(np.uint8)
    out = np.zeros((sc.shape[0], 12), dtype=np.uint8)
    out[:, 0:4] = (sc[:, 0:4] & 63) | ((sc[:, 4:8] >> 4) << 6)
    out[:, 4:8] = (m[:, 0:4] & 63) | ((m[:, 4:8] >> 4) << 6)
    out[:, 8:12] = (sc[:, 4:8] & 15) | ((m[:, 4:8] & 15) << 4)
    return out


def unpack_scale_min_k4(scales: np.ndarray):
    """The 12 packed bytes [nb, 12] -> (sc, m) [nb, 8] (get_scale_min_k4)."""
    q = scales.astype(np.int32)
    sc = np.empty((q.shape[0], 8), dtype=np.int32)
    m = np.empty_like(sc)
    sc[:, 0:4] = q[:, 0:4] & 63
    m[:, 0:4] = q[:, 4:8] & 63
    sc[:, 4:8] = (q[:, 8:12] & 15) | ((q[:, 0:4] >> 6) << 4)
    m[:, 4:8] = (q[:, 8:12] >> 4) | ((q[:, 4:8] >> 6) << 4)
    return sc, m


def gen_q4_k(K: int, N: int, seed: int) -> np.ndarray:
    assert K % 256 == 0
    rng = np.random.default_rng(seed)
    nb = N * (K // 256)
    blk = np.empty((nb, 144), dtype=np.uint8)
    blk[:, 0:2] = _fp16_abs_normal(rng, nb, 0.01).view(np.uint8).reshape(nb, 2)
    blk[:, 2:4] = _fp16_abs_normal(rng, nb, 0.01).view(np.uint8).reshape(nb, 2)
    blk[:, 4:16] = pack_scale_min_k4(rng.integers(0, 64, (nb, 8)), rng.integers(0, 64, (nb, 8)))
    blk[:, 16:144] = rng.integers(0, 256, (nb, 128), dtype=np.uint8)
    return blk.reshape(-1)


def gen_q5_k(K: int, N: int, seed: int) -> np.ndarray:
    assert K % 256 == 0
    rng = np.random.default_rng(seed)
    nb = N * (K // 256)
    blk = np.empty((nb, 176), dtype=np.uint8)
    blk[:, 0:2] = _fp16_abs_normal(rng, nb, 0.01).view(np.uint8).reshape(nb, 2)
    blk[:, 2:4] = _fp16_abs_normal(rng, nb, 0.01).view(np.uint8).reshape(nb, 2)
    blk[:, 4:16] = pack_scale_min_k4(rng.integers(0, 64, (nb, 8)), rng.integers(0, 64, (nb, 8)))
    blk[:, 16:176] = rng.integers(0, 256, (nb, 160), dtype=np.uint8)
    return blk.reshape(-1)


def gen_iq4_nl(K: int, N: int, seed: int) -> np.ndarray:
    assert K % 32 == 0
    rng = np.random.default_rng(seed)
    nb = N * (K // 32)
    blk = np.empty((nb, 18), dtype=np.uint8)
    blk[:, 0:2] = _fp16_abs_normal(rng, nb, 0.01).view(np.uint8).reshape(nb, 2)
    blk[:, 2:18] = rng.integers(0, 256, (nb, 16), dtype=np.uint8)
    return blk.reshape(-1)


def gen_iq4_xs(K: int, N: int, seed: int) -> np.ndarray:
    assert K % 256 == 0
    rng = np.random.default_rng(seed)
    nb = N * (K // 256)
    blk = np.empty((nb, 136), dtype=np.uint8)
    blk[:, 0:2] = _fp16_abs_normal(rng, nb, 0.001).view(np.uint8).reshape(nb, 2)
    blk[:, 2:8] = rng.integers(0, 256, (nb, 6), dtype=np.uint8)  # scales_h (u16) + scales_l[4]
    blk[:, 8:136] = rng.integers(0, 256, (nb, 128), dtype=np.uint8)
    return blk.reshape(-1)


def gen_f16(K: int, N: int, seed: int) -> np.ndarray:
    rng = np.random.default_rng(seed)
    return rng.standard_normal((N, K)).astype(np.float16).view(np.uint8).reshape(-1)


def gen_bf16(K: int, N: int, seed: int) -> np.ndarray:
    rng = np.random.default_rng(seed)
    return rng.standard_normal((N, K)).astype(np.float32).astype(bfloat16).view(np.uint8).reshape(-1)


GENERATORS = {Q4_K: gen_q4_k, Q5_K: gen_q5_k, IQ4_NL: gen_iq4_nl, IQ4_XS: gen_iq4_xs, F16: gen_f16, BF16: gen_bf16}


def generate(fmt: int, K: int, N: int, seed: int) -> np.ndarray:
    return GENERATORS[fmt](K, N, seed)


# ---------------------------------------------------------------- dequant


def _fp16(bits: np.ndarray, ftz: bool) -> np.ndarray:
    """fp16 bits -> float32; with ftz, subnormals become +0 (as the library's
    FTZ flag does for every fp16 scale)."""
    bits = np.ascontiguousarray(bits).view(np.uint16).reshape(-1)
    d = bits.view(np.float16).astype(np.float32)
    if ftz:
        d = np.where(((bits & 0x7C00) == 0) & ((bits & 0x03FF) != 0), np.float32(0.0), d)
    return d


def dequant_f32(fmt: int, raw: np.ndarray, K: int, N: int, ftz: bool = False) -> np.ndarray:
    """values[n, k] in float32, evaluated as ggml's dequantize_row_* does."""
    raw = np.ascontiguousarray(np.asarray(raw, dtype=np.uint8)[: N * row_bytes(fmt, K)])
    if fmt == F16:
        return raw.view(np.float16).astype(np.float32).reshape(N, K)
    if fmt == BF16:
        return raw.view(bfloat16).astype(np.float32).reshape(N, K)
    bk, bb = BLOCK_K[fmt], BLOCK_BYTES[fmt]
    blk = raw.reshape(-1, bb)
    nb = blk.shape[0]
    f32 = np.float32
    if fmt in (Q4_K, Q5_K):
        d = _fp16(blk[:, 0:2].copy(), ftz)
        dmin = _fp16(blk[:, 2:4].copy(), ftz)
        sc, m = unpack_scale_min_k4(blk[:, 4:16])
        qs = blk[:, 16:144] if fmt == Q4_K else blk[:, 48:176]
        qh = blk[:, 16:48] if fmt == Q5_K else None
        out = np.empty((nb, 256), dtype=np.float32)
        for i in range(4):  # 64-weight chunk i: sub-blocks 2i (low nibbles) and 2i + 1 (high)
            q = qs[:, 32 * i : 32 * i + 32].astype(np.int32)
            for h in range(2):
                j = 2 * i + h
                v = (q >> (4 * h)) & 15
                if qh is not None:
                    v = v + (((qh.astype(np.int32) >> j) & 1) << 4)
                d1 = (d * sc[:, j].astype(f32)).astype(f32)  # exact
                m1 = (dmin * m[:, j].astype(f32)).astype(f32)  # exact
                out[:, 64 * i + 32 * h : 64 * i + 32 * h + 32] = (d1[:, None] * v.astype(f32)) - m1[:, None]
        return out.reshape(N, K)
    kv = KVALUES_IQ4.astype(f32)
    if fmt == IQ4_NL:
        d = _fp16(blk[:, 0:2].copy(), ftz)
        qs = blk[:, 2:18]
        q = np.concatenate([qs & 15, qs >> 4], axis=1)
        return (d[:, None] * kv[q]).reshape(N, K)
    if fmt == IQ4_XS:
        d = _fp16(blk[:, 0:2].copy(), ftz)
        sh = blk[:, 2:4].copy().view(np.uint16).reshape(-1).astype(np.int32)
        sl = blk[:, 4:8].astype(np.int32)
        qs = blk[:, 8:136]
        out = np.empty((nb, 256), dtype=np.float32)
        for ib in range(8):
            ls = ((sl[:, ib // 2] >> (4 * (ib % 2))) & 15) | (((sh >> (2 * ib)) & 3) << 4)
            dl = (d * (ls - 32).astype(f32)).astype(f32)  # exact
            q = qs[:, 16 * ib : 16 * ib + 16]
            out[:, 32 * ib : 32 * ib + 16] = dl[:, None] * kv[q & 15]
            out[:, 32 * ib + 16 : 32 * ib + 32] = dl[:, None] * kv[q >> 4]
        return out.reshape(N, K)
    raise ValueError(f"format {fmt}")


def dequant_bf16(fmt: int, raw, K: int, N: int, ftz: bool = False) -> np.ndarray:
    """bf16 bits (uint16) [N][K]."""
    return dequant_f32(fmt, raw, K, N, ftz).astype(bfloat16).view(np.uint16)


def mul_mat_f64(fmt: int, raw, x_bits: np.ndarray, K: int, N: int, ftz: bool = False) -> np.ndarray:
    """y[m][n] = sum_k bf16(W[n][k]) * x[m][k] in float64."""
    w = (dequant_bf16(fmt, raw, K, N, ftz).astype(np.uint32) << 16).view(np.float32).astype(np.float64)
    x = (np.asarray(x_bits, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32).astype(np.float64)
    return x @ w.T


# ------------------------------------------------- per-block restatement
# A second, literal per-block restatement of the same published loops (one
# weight at a time, ggml's loop order), used by the CPU tests to check the
# vectorised oracle above.


def dequant_block_loop(fmt: int, blk: bytes) -> np.ndarray:
    b = np.frombuffer(bytes(blk), dtype=np.uint8)
    f32 = np.float32
    half = lambda o: np.frombuffer(b[o : o + 2].tobytes(), dtype=np.float16)[0].astype(f32)
    if fmt in (Q4_K, Q5_K):
        d, dmin = half(0), half(2)
        scales = b[4:16]

        def get_scale_min(j):
            if j < 4:
                return int(scales[j]) & 63, int(scales[j + 4]) & 63
            return ((int(scales[j + 4]) & 0xF) | ((int(scales[j - 4]) >> 6) << 4),
                    (int(scales[j + 4]) >> 4) | ((int(scales[j]) >> 6) << 4))

        ql = b[16:144] if fmt == Q4_K else b[48:176]
        qh = b[16:48] if fmt == Q5_K else None
        y = np.empty(256, dtype=f32)
        u1, u2, is_, qo = 1, 2, 0, 0
        for j in range(0, 256, 64):
            sc, m = get_scale_min(is_)
            d1, m1 = f32(d * f32(sc)), f32(dmin * f32(m))
            sc, m = get_scale_min(is_ + 1)
            d2, m2 = f32(d * f32(sc)), f32(dmin * f32(m))
            for l in range(32):
                q = int(ql[qo + l]) & 0xF
                if qh is not None and int(qh[l]) & u1:
                    q += 16
                y[j + l] = f32(f32(d1 * f32(q)) - m1)
            for l in range(32):
                q = int(ql[qo + l]) >> 4
                if qh is not None and int(qh[l]) & u2:
                    q += 16
                y[j + 32 + l] = f32(f32(d2 * f32(q)) - m2)
            qo += 32
            is_ += 2
            u1 <<= 2
            u2 <<= 2
        return y
    if fmt == IQ4_NL:
        d = half(0)
        y = np.empty(32, dtype=f32)
        for j in range(16):
            y[j] = f32(d * f32(KVALUES_IQ4[int(b[2 + j]) & 0xF]))
            y[j + 16] = f32(d * f32(KVALUES_IQ4[int(b[2 + j]) >> 4]))
        return y
    if fmt == IQ4_XS:
        d = half(0)
        scales_h = int(b[2]) | (int(b[3]) << 8)
        y = np.empty(256, dtype=f32)
        for ib in range(8):
            ls = ((int(b[4 + ib // 2]) >> (4 * (ib % 2))) & 0xF) | (((scales_h >> (2 * ib)) & 3) << 4)
            dl = f32(d * f32(ls - 32))
            for j in range(16):
                q = int(b[8 + 16 * ib + j])
                y[32 * ib + j] = f32(dl * f32(KVALUES_IQ4[q & 0xF]))
                y[32 * ib + j + 16] = f32(dl * f32(KVALUES_IQ4[q >> 4]))
        return y
    raise ValueError(f"format {fmt}")
