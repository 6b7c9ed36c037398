"""CPU checks of the extended-format oracle (oracle/formats_ext.py) and of the
C-ABI's size queries for those formats.

The vectorised oracle is checked against a second, literal restatement of
ggml's per-block dequant loops (one weight at a time, ggml's loop order and
float32 roundings), on random blocks and on edge scales.  Parity with ggml
itself is unpinned: the reference has no code for these formats."""

from __future__ import annotations

import numpy as np
import pytest

from oracle import formats_ext as X

EXT_Q = (X.Q4_K, X.Q5_K, X.IQ4_NL, X.IQ4_XS)


@pytest.mark.parametrize("fmt", EXT_Q, ids=lambda f: X.NAMES[f])
def test_vectorised_oracle_equals_block_loop(fmt):
    K, N = 512, 4
    raw = X.generate(fmt, K, N, seed=fmt)
    bb = X.BLOCK_BYTES[fmt]
    # edge scales in the first blocks: +0, -0, negative, subnormal, max finite
    blk = raw.reshape(-1, bb)
    edge = np.array([0x0000, 0x8000, 0xBC00, 0x0001, 0x7BFF], dtype=np.uint16)
    blk[: len(edge), 0:2] = edge.view(np.uint8).reshape(-1, 2)
    raw = blk.reshape(-1)
    v = X.dequant_f32(fmt, raw, K, N)
    loop = np.concatenate([X.dequant_block_loop(fmt, raw[i * bb : (i + 1) * bb]) for i in range(blk.shape[0])])
    assert np.array_equal(v.reshape(-1).view(np.uint32), loop.view(np.uint32))


def test_kquant_scale_min_roundtrip():
    rng = np.random.default_rng(3)
    sc = rng.integers(0, 64, (200, 8))
    m = rng.integers(0, 64, (200, 8))
    s2, m2 = X.unpack_scale_min_k4(X.pack_scale_min_k4(sc, m))
    assert np.array_equal(s2, sc) and np.array_equal(m2, m)


def test_iq4_codebook_is_sorted_and_signed():
    kv = X.KVALUES_IQ4.astype(int)
    assert kv.tolist() == sorted(kv.tolist())
    assert kv.min() == -127 and kv.max() == 113 and len(kv) == 16


def test_pass_through_types():
    K, N = 64, 3
    raw = X.generate(X.BF16, K, N, seed=1)
    assert np.array_equal(X.dequant_bf16(X.BF16, raw, K, N).reshape(-1), raw.view(np.uint16))
    raw = X.generate(X.F16, K, N, seed=2)
    f = raw.view(np.float16).astype(np.float32)
    assert np.array_equal(X.dequant_f32(X.F16, raw, K, N).reshape(-1), f)


def test_abi_sizes_of_extended_formats():
    import spiral_b200 as sp

    L = sp.lib()
    for fmt in (X.Q4_K, X.Q5_K, X.IQ4_NL, X.IQ4_XS, X.F16, X.BF16):
        assert L.spiral_quants_block_rows(fmt) == X.BLOCK_K[fmt]
        assert L.spiral_quants_block_bytes(fmt) == X.BLOCK_BYTES[fmt]
        assert sp.row_bytes(fmt, 1024) == X.row_bytes(fmt, 1024)
    # the reference-format-only entry points refuse them
    assert L.spiral_quants_record_count(X.Q4_K, 256, 8) == 0
