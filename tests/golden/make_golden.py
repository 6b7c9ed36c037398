"""Generate the golden fixtures in tests/golden/ from the reference's own oracle.

Run here, where the reference tree is mounted (it does not exist on the GPU
box; the fixtures this writes travel instead):

    python tests/golden/make_golden.py [--reference DIR]

DIR defaults to $SPIRAL_REFERENCE_DIR, else a sibling directory `reference`
next to this repository.

Everything "expected" below is produced by the reference's NumPy oracle
(src/quants/tests/formats/{q4_0,q8_0,q6_k}.py) and its mmul harness
(src/quants/tests/mmul.py), imported unchanged.  Outputs:

* ref_default_<fmt>_s<seed>.npz — the reference's own generator
  (make_raw, seeds 1..3, default 256x64 shape) with reference_weights and
  the fused-mmul expectation (make_inputs seed+1000, 4 vectors,
  inputs_rows @ weights_matrix in float32, as mmul.py:104-121 does).
* baseline_small_<fmt>.npz — the BASELINE generators of oracle/formats.py at a
  small shape, expected = reference _dequant_values(...).astype(bfloat16).
* edge_<fmt>.npz — hand-built blocks: zero / negative-zero / subnormal /
  largest finite scales, every quant value, Q8_0 -128, extreme Q6_K
  sub-scales; plus the flush-to-zero expectation, made the way the reference
  device path makes it: subnormal scale bits replaced by 0
  (src/quants/q4_0/repack.h:75-80) before the oracle runs.
* hashes.json — SHA-256 of the reference oracle's bf16 output (ggml row-major
  [N][K]) for the full BASELINE dequant configs.
"""

from __future__ import annotations

import argparse
import os
import hashlib
import json
import sys
from pathlib import Path

import numpy as np
from ml_dtypes import bfloat16

HERE = Path(__file__).resolve().parent
REPO = HERE.parent.parent
sys.path.insert(0, str(REPO))

from oracle import formats as F  # noqa: E402

sys.dont_write_bytecode = True  # never write into the read-only reference tree


def load_reference(root: Path):
    tests = root / "src" / "quants" / "tests"
    sys.path.insert(0, str(tests))
    import importlib

    mods = {name: importlib.import_module(f"formats.{name}") for name in ("q4_0", "q8_0", "q6_k")}
    mmul = importlib.import_module("mmul")
    return mods, mmul


def ref_rows_bf16(mod, raw, K, N):
    """Reference oracle values [K][N] -> ggml row-major [N][K] bf16 bits."""
    vals = mod._dequant_values(raw, K, N)
    return np.ascontiguousarray(vals.T).astype(bfloat16).view(np.uint16)


def flush_subnormal_scales(fid, raw, K, N):
    raw = raw.copy()
    bb, bk = F.BLOCK_BYTES[fid], F.BLOCK_K[fid]
    blk = raw.reshape(N * (K // bk), bb)
    off = 208 if fid == F.Q6_K else 0
    bits = blk[:, off : off + 2].copy().view(np.uint16).reshape(-1)
    sub = ((bits & 0x7C00) == 0) & ((bits & 0x03FF) != 0)
    bits = np.where(sub, np.uint16(0), bits)
    blk[:, off : off + 2] = bits.view(np.uint8).reshape(-1, 2)
    return blk.reshape(-1)


SPECIAL_D = np.array(
    [0x0000, 0x8000, 0x0001, 0x8001, 0x03FF, 0x0400, 0x83FF, 0x3C00, 0xBC00, 0x7BFF, 0xFBFF, 0x2E66, 0x1400, 0x0200],
    dtype=np.uint16,
)


def edge_raw(fid, rng):
    """Blocks with every special scale, each paired with rich quants."""
    nd = len(SPECIAL_D)
    if fid == F.Q4_0:
        K, N = 32 * 16, nd
        nb = N * (K // 32)
        d = np.repeat(SPECIAL_D, K // 32)
        q = rng.integers(0, 16, size=(nb, 32), dtype=np.uint8)
        q[::2, :16] = np.arange(16, dtype=np.uint8)  # every nibble value
        blk = np.empty((nb, 18), np.uint8)
        blk[:, 0:2] = d.view(np.uint8).reshape(nb, 2)
        blk[:, 2:] = q[:, :16] | (q[:, 16:] << 4)
    elif fid == F.Q8_0:
        K, N = 32 * 16, nd
        nb = N * (K // 32)
        d = np.repeat(SPECIAL_D, K // 32)
        q = rng.integers(-128, 128, size=(nb, 32), dtype=np.int16).astype(np.int8)
        q[:, 0] = -128
        q[:, 1] = 127
        q[:, 2] = -127
        blk = np.empty((nb, 34), np.uint8)
        blk[:, 0:2] = d.view(np.uint8).reshape(nb, 2)
        blk[:, 2:] = q.view(np.uint8)
    else:
        K, N = 256 * 4, nd
        nsb = N * (K // 256)
        d = np.repeat(SPECIAL_D, K // 256)
        q6 = rng.integers(0, 64, size=(nsb, 256), dtype=np.uint8)
        q6[:, :64] = np.arange(64, dtype=np.uint8)
        sc = rng.integers(-128, 128, size=(nsb, 16), dtype=np.int16).astype(np.int8)
        sc[:, 0] = -128
        sc[:, 1] = 127
        sc[:, 2] = -1
        sc[:, 3] = 0
        blk = F.encode_q6_k(q6, sc, d.view(np.float16))
    return blk.reshape(-1), K, N


def main(argv=None):
    ap = argparse.ArgumentParser()
    default_ref = os.environ.get("SPIRAL_REFERENCE_DIR") or str(Path(__file__).resolve().parents[3] / "reference")
    ap.add_argument("--reference", default=default_ref)
    ap.add_argument("--skip-hashes", action="store_true")
    args = ap.parse_args(argv)
    mods, mmul = load_reference(Path(args.reference))

    # 1. the reference's own default cases (generator, order, fused mmul)
    for name, mod in mods.items():
        for seed in (1, 2, 3):
            K, N = mod.DEFAULT_ROWS, mod.DEFAULT_COLS
            raw = mod.make_raw(K, N, np.random.default_rng(seed))
            expected = mod.reference_weights(raw, K, N)
            packed_inputs, inputs_rows = mmul.make_inputs(K, seed, 4, 8)
            weights_matrix = (
                expected.reshape(N // 8, K, 8).transpose(1, 0, 2).reshape(K, N).astype(np.float32)
            )
            expected_outputs = inputs_rows @ weights_matrix
            np.savez_compressed(
                HERE / f"ref_default_{name}_s{seed}.npz",
                raw=raw,
                K=K,
                N=N,
                expected_weights=expected.view(np.uint16),
                inputs_tiled=np.asarray(packed_inputs).view(np.uint16),
                inputs_rows=inputs_rows.astype(np.float32),
                expected_outputs=expected_outputs.astype(np.float32),
            )

    # 2. BASELINE generators at a small shape, checked by the reference oracle
    small = {F.Q4_0: (1024, 64), F.Q8_0: (1024, 64), F.Q6_K: (2048, 32)}
    for fid, (K, N) in small.items():
        name = F.NAMES[fid]
        raw = F.generate(fid, K, N, seed=0)
        np.savez_compressed(
            HERE / f"baseline_small_{name}.npz", raw=raw, K=K, N=N, expected=ref_rows_bf16(mods[name], raw, K, N)
        )

    # 3. edge cases (+ flush-to-zero expectation)
    for fid in (F.Q4_0, F.Q8_0, F.Q6_K):
        name = F.NAMES[fid]
        raw, K, N = edge_raw(fid, np.random.default_rng(7))
        raw_ftz = flush_subnormal_scales(fid, raw, K, N)
        np.savez_compressed(
            HERE / f"edge_{name}.npz",
            raw=raw,
            K=K,
            N=N,
            expected=ref_rows_bf16(mods[name], raw, K, N),
            expected_ftz=ref_rows_bf16(mods[name], raw_ftz, K, N),
        )

    # 4. full-size digests of the reference oracle at the BASELINE configs
    if not args.skip_hashes:
        hashes = {}
        for fid, K, N in ((F.Q4_0, 4096, 4096), (F.Q8_0, 4096, 14336), (F.Q6_K, 4096, 14336)):
            name = F.NAMES[fid]
            raw = F.generate(fid, K, N, seed=0)
            out = ref_rows_bf16(mods[name], raw, K, N)
            key = f"{name}_K{K}_N{N}_seed0"
            hashes[key] = {
                "raw_sha256": hashlib.sha256(raw.tobytes()).hexdigest(),
                "bf16_rows_sha256": hashlib.sha256(out.tobytes()).hexdigest(),
            }
            print(key, hashes[key], flush=True)
        (HERE / "hashes.json").write_text(json.dumps(hashes, indent=1, sort_keys=True) + "\n")
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
