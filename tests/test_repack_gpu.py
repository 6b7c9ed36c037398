"""spiral_quants_repack on the GPU against the reference's repack contract
(src/quants/q4_0/repack.h:27-111, q8_0/repack.h:26-91, q6_k/repack.h:28-115,
common/repack.h:9-61): a strided canonical view becomes the dense tensor,
subnormal fp16 scales are flushed to +0, Q8_0 quants of -128 are reported,
and each call emits at most one warning line worded as the reference's,
through the caller's hook.  Where the reference's own host shim is built
(oracle/_ref), its stderr line for the same input is the expected text."""

from __future__ import annotations

import ctypes

import numpy as np
import pytest

import oracle
import spiral_b200 as sp
from oracle import formats as F

from .conftest import REPO
from .gpu_util import dev_bytes, strided_rows

pytestmark = pytest.mark.gpu
SCALE_AT = {F.Q4_0: 0, F.Q8_0: 0, F.Q6_K: 208}


def _blocks(fid, raw):
    return raw.reshape(-1, F.BLOCK_BYTES[fid])


def _plant(fid, raw, subnormal: bool, min_int8: bool):
    """Copy of raw with a subnormal scale in every 7th block and (Q8_0) a
    -128 quant in every 5th block."""
    out = raw.copy()
    b = _blocks(fid, out)
    at = SCALE_AT[fid]
    if subnormal:
        b[::7, at] = 0x05  # fp16 0x0005: exponent 0, mantissa 5
        b[::7, at + 1] = 0x00
    if min_int8:
        b[::5, 2 + 3] = 0x80
    return out


def _flush(fid, raw):
    want = raw.copy()
    b = _blocks(fid, want)
    at = SCALE_AT[fid]
    h = b[:, at].astype(np.uint16) | (b[:, at + 1].astype(np.uint16) << 8)
    sub = ((h & 0x7C00) == 0) & ((h & 0x03FF) != 0)
    b[sub, at] = 0
    b[sub, at + 1] = 0
    return want


def _reference_line(fid, raw, K, N, capfd):
    path = REPO / "oracle" / "_ref" / f"quants_host_{F.NAMES[fid]}.so"
    if not path.exists():
        return None
    L = ctypes.CDLL(str(path))
    L.quants_packed_bytes.argtypes = [ctypes.c_int64, ctypes.c_int64]
    L.quants_packed_bytes.restype = ctypes.c_int64
    L.quants_repack.argtypes = [ctypes.c_void_p, ctypes.c_int64, ctypes.c_void_p, ctypes.c_int64, ctypes.c_int64,
                                ctypes.c_int64]
    L.quants_repack.restype = ctypes.c_int64
    cap = int(L.quants_packed_bytes(K, N))
    dst = np.zeros(cap, dtype=np.uint8)
    capfd.readouterr()
    assert L.quants_repack(raw.ctypes.data, F.row_bytes(fid, K), dst.ctypes.data, cap, K, N) == cap
    return capfd.readouterr().err


@pytest.mark.parametrize("fid", [F.Q4_0, F.Q8_0, F.Q6_K], ids=lambda f: F.NAMES[f])
@pytest.mark.parametrize("subnormal,min_int8", [(False, False), (True, False), (False, True), (True, True)])
def test_repack_flushes_reports_and_warns_like_the_reference(cuda, capfd, fid, subnormal, min_int8):
    import torch

    if min_int8 and fid != F.Q8_0:
        pytest.skip("-128 is a Q8_0 report")
    K, N = 512, 40
    rb = F.row_bytes(fid, K)
    raw = F.generate(fid, K, N, seed=21)
    if fid == F.Q8_0:  # the generator draws -127..127: no -128 unless planted
        assert not np.any(_blocks(fid, raw)[:, 2:] == 0x80)
    raw = _plant(fid, raw, subnormal, min_int8)
    stride = rb + 16
    src = dev_bytes(strided_rows(raw, N, rb, stride))
    cap = sp.packed_bytes(fid, K, N)
    dst = torch.zeros(cap + 64, dtype=torch.uint8, device="cuda")
    lines = []
    sp.set_repack_warn(lines.append)
    try:
        got = sp.repack(fid, src, stride, dst, cap, K, N)
    finally:
        sp.set_repack_warn(to_stderr=True)
    assert got == cap
    out = dst.cpu().numpy()
    assert np.array_equal(out[:cap], _flush(fid, raw))
    assert not out[cap:].any()  # nothing written past the dense tensor
    name = F.NAMES[fid].upper()
    # the BASELINE generators draw some subnormal scales of their own
    subnormal = not np.array_equal(_flush(fid, raw), raw)
    min_int8 = fid == F.Q8_0 and bool(np.any(_blocks(fid, raw)[:, 2:] == 0x80))
    if subnormal and min_int8:
        want = [f"quants: {name} repack flushed subnormal fp16 scales to zero and found -128 int8 weights\n"]
    elif subnormal:
        want = [f"quants: {name} repack flushed subnormal fp16 scales to zero\n"]
    elif min_int8:
        want = [f"quants: {name} repack found -128 int8 weights\n"]
    else:
        want = []
    assert lines == want
    # the repacked tensor dequantizes like the reference's device path (ftz)
    back = sp.dequant_bf16(fid, dst[:cap], K, N)
    np.testing.assert_array_equal(back.view(torch.int16).cpu().numpy().view(np.uint16),
                                  oracle.dequant_bf16(fid, raw, K, N, ftz=True))
    # the reference's own repack prints the same line for the same input
    ref = _reference_line(fid, raw, K, N, capfd)  # the reference shim takes K % 256 == 0, N % 8 == 0
    if ref is not None:
        assert ref == "".join(want)


def test_repack_of_clean_data_is_silent(cuda):
    import torch

    fid, K, N = F.Q4_0, 256, 8
    raw = _flush(fid, F.generate(fid, K, N, seed=3))  # no subnormal scale left
    dst = torch.zeros(sp.packed_bytes(fid, K, N), dtype=torch.uint8, device="cuda")
    lines = []
    sp.set_repack_warn(lines.append)
    try:
        assert sp.repack(fid, dev_bytes(raw), F.row_bytes(fid, K), dst, dst.numel(), K, N) == dst.numel()
    finally:
        sp.set_repack_warn(to_stderr=True)
    assert lines == []
    assert np.array_equal(dst.cpu().numpy(), raw)


def test_repack_warning_can_be_suppressed(cuda, capfd):
    import torch

    fid, K, N = F.Q4_0, 256, 8
    raw = _plant(fid, F.generate(fid, K, N, seed=3), True, False)
    src = dev_bytes(raw)
    dst = torch.zeros(sp.packed_bytes(fid, K, N), dtype=torch.uint8, device="cuda")
    sp.set_repack_warn(None)
    try:
        capfd.readouterr()
        assert sp.repack(fid, src, F.row_bytes(fid, K), dst, dst.numel(), K, N) == dst.numel()
        assert capfd.readouterr().err == ""
    finally:
        sp.set_repack_warn(to_stderr=True)
