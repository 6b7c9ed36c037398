"""The C-ABI library loads, exports every declared symbol, and validates its
arguments on the host (no GPU work is launched by these tests).

The reference's contract for invalid input is "return 0" for the size queries
and the repack (src/quants/q4_0/repack.h:10-41, TODO.md:331-334); the compute
entry points return negative spiral_status codes.
"""

from __future__ import annotations

import ctypes
import re
import subprocess
from pathlib import Path

import pytest

import spiral_b200 as sp

from .conftest import REPO

HEADER = REPO / "include" / "spiral_b200.h"


def declared_symbols() -> set[str]:
    text = HEADER.read_text()
    return set(re.findall(r"^SPIRAL_API\s+[\w\s\*]+?\b(spiral_\w+)\s*\(", text, flags=re.M))


def test_library_exports_every_declared_symbol():
    syms = declared_symbols()
    assert len(syms) >= 12
    out = subprocess.run(["nm", "-D", "--defined-only", str(sp.LIB_PATH)], capture_output=True, text=True,
                         check=True).stdout
    exported = set(re.findall(r"\bT (spiral_\w+)", out))
    assert syms <= exported, syms - exported
    # the Python mirror binds exactly the declared surface
    assert set(sp._SIGNATURES) == syms
    L = sp.lib()
    for name in syms:
        assert getattr(L, name) is not None


def test_library_has_no_torch_or_oracle_dependency():
    out = subprocess.run(["ldd", str(sp.LIB_PATH)], capture_output=True, text=True).stdout
    assert "torch" not in out and "oracle" not in out and "python" not in out


def test_version_and_status_strings():
    L = sp.lib()
    assert L.spiral_version() >= 100
    assert L.spiral_status_string(0) == b"ok"
    assert L.spiral_status_string(-2) == b"invalid shape"
    assert L.spiral_status_string(12345) == b"unknown status"


@pytest.mark.parametrize("fmt,bk,bb", [(sp.Q4_0, 32, 18), (sp.Q8_0, 32, 34), (sp.Q6_K, 256, 210)])
def test_size_queries(fmt, bk, bb):
    L = sp.lib()
    assert L.spiral_quants_block_rows(fmt) == bk
    assert L.spiral_quants_block_bytes(fmt) == bb
    assert sp.record_count(fmt, 4096, 14336) == (4096 // bk) * 14336
    assert sp.packed_bytes(fmt, 4096, 14336) == (4096 // bk) * 14336 * bb
    # invalid shapes return 0 (reference contract)
    assert sp.record_count(fmt, bk + 1, 8) == 0
    assert sp.record_count(fmt, 0, 8) == 0
    assert sp.record_count(fmt, bk, 0) == 0
    assert sp.packed_bytes(fmt, -bk, 8) == 0
    assert sp.packed_bytes(99, 256, 8) == 0
    assert L.spiral_quants_block_rows(99) == 0


def _ref_shim(name):
    path = REPO / "oracle" / "_ref" / f"quants_host_{name}.so"
    if not path.exists():
        pytest.skip("reference host shim not built (make -C oracle ref)")
    L = ctypes.CDLL(str(path))
    L.quants_packed_bytes.argtypes = [ctypes.c_int64, ctypes.c_int64]
    L.quants_packed_bytes.restype = ctypes.c_int64
    return L


@pytest.mark.parametrize("name", ["q4_0", "q8_0", "q6_k"])
def test_packed_bytes_agree_with_reference_shim(name):
    """For the reference's own shape rules (rows % 256, cols % 8) the
    reference's repacked size equals the canonical size this library reads,
    so buffers sized with either query are interchangeable."""
    ref = _ref_shim(name)
    for rows, cols in ((256, 64), (4096, 4096), (4096, 14336), (768, 2048)):
        assert sp.packed_bytes(name, rows, cols) == ref.quants_packed_bytes(rows, cols)
    assert ref.quants_packed_bytes(100, 8) == 0 and sp.packed_bytes(name, 100, 8) == 0


def test_repack_rejects_invalid_input_with_zero():
    # no device memory is touched: every case fails validation first
    assert sp.repack(sp.Q4_0, 0, 2304, 0, 1 << 20, 4096, 8) == 0  # null pointers
    assert sp.repack(sp.Q4_0, 16, 2303, 32, 1 << 20, 4096, 8) == 0  # stride < row
    assert sp.repack(sp.Q4_0, 16, 2304, 32, 100, 4096, 8) == 0  # capacity
    assert sp.repack(sp.Q4_0, 16, 2304, 32, 1 << 20, 4097, 8) == 0  # shape


def _call_mul_mat(**kw):
    a = dict(fmt=sp.Q4_0, w=16, ws=2304, x=16, xs=4096, y=16, yd=sp.BF16, ys=8, M=1, N=8, K=4096, flags=0)
    a.update(kw)
    return sp.lib().spiral_mul_mat(a["fmt"], a["w"], a["ws"], a["x"], a["xs"], a["y"], a["yd"], a["ys"], a["M"],
                                   a["N"], a["K"], a["flags"], 0)


def test_mul_mat_validation_codes():
    assert _call_mul_mat(fmt=3) == -1
    assert _call_mul_mat(K=4001) == -2 and b"K=4001" in sp.lib().spiral_last_error()
    assert _call_mul_mat(K=4001) == -2
    assert _call_mul_mat(M=0) == -2
    assert _call_mul_mat(N=-1) == -2
    assert _call_mul_mat(w=0) == -3
    assert _call_mul_mat(x=0) == -3
    assert _call_mul_mat(yd=7) == -10
    assert _call_mul_mat(flags=sp.FLAG_ACCUMULATE) == -10  # accumulate needs f32
    assert _call_mul_mat(ws=100) == -2
    assert _call_mul_mat(xs=10) == -2
    assert _call_mul_mat(w=17) == -4


def test_dequant_and_unpack_validation_codes():
    L = sp.lib()
    assert L.spiral_dequant_bf16(sp.Q6_K, 16, 3360, 16, 4096, 4000, 8, 0, 0) == -2
    assert L.spiral_dequant_bf16(sp.Q6_K, 0, 3360, 16, 4096, 4096, 8, 0, 0) == -3
    assert L.spiral_dequant_bf16(sp.Q6_K, 16, 3000, 16, 4096, 4096, 8, 0, 0) == -2
    assert L.spiral_dequant_bf16(sp.Q6_K, 17, 3360, 16, 4096, 4096, 8, 0, 0) == -4
    assert L.spiral_quants_unpack_all(sp.Q8_0, 16, 16, 256, 60, 0, 0) == -2  # cols % 8
    assert L.spiral_quants_unpack_all(sp.Q8_0, 16, 18, 256, 64, 0, 0) == -4  # 16B output
    assert L.spiral_quants_unpack_mmul_all(sp.Q8_0, 16, 16, 16, 256, 64, 0, 0, 0) == -2
    assert L.spiral_quants_unpack_mmul_all(sp.Q8_0, 0, 16, 16, 256, 64, 4, 0, 0) == -3
    assert L.spiral_quants_unpack_mmul_all(sp.Q8_0, 16, 16, 18, 256, 64, 4, 0, 0) == -4


def test_python_mirror_raises_on_error():
    with pytest.raises(sp.SpiralError) as e:
        sp._check(sp.lib().spiral_dequant_bf16(sp.Q4_0, 0, 18, 16, 32, 32, 1, 0, 0))
    assert e.value.status == -3


def test_moe_validation_codes():
    L = sp.lib()
    assert sp.moe_workspace_bytes(128, 2048, 768, 64, 8) > 64 * 8 * 2048 * 4
    assert sp.moe_workspace_bytes(0, 2048, 768, 64, 8) == 0

    def call(**kw):
        a = dict(fmt=sp.Q4_0, wg=256, wu=256, wd=256, E=8, e0=0, H=2048, I=768, x=256, xs=2048, T=4, ids=256,
                 w=256, topk=8, y=256, yd=sp.BF16, ys=2048, ws=256, wsb=1 << 30, flags=0)
        a.update(kw)
        return L.spiral_moe_ffn(a["fmt"], a["wg"], a["wu"], a["wd"], a["E"], a["e0"], a["H"], a["I"], a["x"],
                                a["xs"], a["T"], a["ids"], a["w"], a["topk"], a["y"], a["yd"], a["ys"], a["ws"],
                                a["wsb"], a["flags"], 0)

    assert call(fmt=5) == -1
    assert call(H=2000) == -2  # not a multiple of 256
    assert call(I=4096) == -2  # above the staging limit
    assert call(T=0) == -2
    assert call(wg=0) == -3
    assert call(x=264) == -4  # activations must be 16-byte aligned
    assert call(xs=2052) == -4
    assert call(ws=260) == -4
    assert call(wsb=1024) == -5  # workspace too small
    assert call(yd=7) == -10


def test_mul_mat_allgather_validation_codes():
    L = sp.lib()
    assert sp.allgather_exchange_bytes(14336) == 256 + 2 * 32 * 14336
    assert sp.allgather_exchange_bytes(14332) == 0
    assert sp.allgather_exchange_bytes(0) == 0

    def call(**kw):
        a = dict(fmt=sp.Q4_0, w=256, ws=2304, x=256, xs=4096, y=256, ys=14336, off=7168, M=8, N=7168, NT=14336,
                 K=4096, xc=256, rank=1, world=2, flags=0)
        a.update(kw)
        return L.spiral_mul_mat_allgather(a["fmt"], a["w"], a["ws"], a["x"], a["xs"], a["y"], a["ys"], a["off"],
                                          a["M"], a["N"], a["NT"], a["K"], a["xc"], a["rank"], a["world"],
                                          a["flags"], 0)

    assert call(fmt=3) == -1
    assert call(K=4001) == -2
    assert call(M=9) == -2 and b"1..8" in L.spiral_last_error()
    assert call(M=0) == -2
    assert call(rank=2) == -10
    assert call(world=0) == -10
    assert call(y=0) == -3
    assert call(xc=0) == -3
    assert call(off=7176) == -2  # shard runs past the gathered width
    assert call(off=-8) == -2
    assert call(ys=14328) == -2  # row stride below the gathered width
    assert call(ws=2000) == -2
    assert call(w=264) == -4
    assert call(off=7164, N=7172) == -4  # 8-column granularity
    assert call(ys=14340) == -4
    assert call(y=264) == -4
    # the recovery reset checks its arguments before touching the device
    assert L.spiral_allgather_exchange_reset(256, 14332, 0) == -2
    assert L.spiral_allgather_exchange_reset(0, 14336, 0) == -3


def test_repack_rejects_misaligned_input_with_zero():
    # odd addresses or strides (the device repack moves 2-byte granules)
    assert sp.repack(sp.Q4_0, 17, 2304, 32, 1 << 20, 4096, 8) == 0
    assert sp.repack(sp.Q4_0, 16, 2305, 32, 1 << 20, 4096, 8) == 0
    assert sp.repack(sp.Q4_0, 16, 2304, 33, 1 << 20, 4096, 8) == 0


def test_repack_warning_hook_is_settable_without_a_gpu():
    lines = []
    sp.set_repack_warn(lines.append)
    sp.set_repack_warn(None)
    sp.set_repack_warn(to_stderr=True)
    assert lines == []


def test_moe_ep_validates_its_arguments():
    """Host-side argument checks of spiral_moe_ffn_ep (nothing is launched)."""
    L = sp.lib()
    p = 256  # never dereferenced: every case fails validation first
    H, I, E, topk = 2048, 768, 8, 8
    args = dict(fmt=sp.Q4_0, E=E, e0=0, H=H, I=I, T=4, maxT=4, topk=topk, peers=p, rank=0, world=2, ws=1 << 30)

    def call(**kw):
        a = dict(args, **kw)
        return L.spiral_moe_ffn_ep(a["fmt"], p, p, p, a["E"], a["e0"], a["H"], a["I"], p, H, a["T"], a["maxT"], p,
                                   p, a["topk"], p, sp.BF16, H, a["peers"], a["rank"], a["world"], p, a["ws"], 0, 0)

    assert call(rank=2) == -10
    assert call(world=0) == -10
    assert call(peers=0) == -3
    assert call(T=5) == -5  # more tokens than the exchange holds
    assert call(H=2048, world=3) == -2  # hidden not a multiple of world
    assert sp.moe_ep_exchange_bytes(0, 4) == 0 and sp.moe_ep_exchange_bytes(H, 4) > 0
    assert L.spiral_moe_ep_exchange_reset(p, 0, 4, 0) == -2
    assert L.spiral_moe_ep_exchange_reset(0, H, 4, 0) == -3


def test_ggml_supports_mul_mat_follows_ggml_rules():
    """supports_op for GGML_OP_MUL_MAT (host logic only; nothing launched)."""
    K, N, M = 4096, 64, 2
    p = 256

    def node(t0=sp.Q4_0, t1=sp.BF16, td=sp.F32, k1=K, ne12=1, ne02=1, nb00=None, nb10=2):
        bb, bk = sp.BLOCK_BYTES.get(t0, 18), sp.BLOCK_K.get(t0, 32)
        rb = K // bk * bb
        src0 = sp.ggml_tensor(t0, (K, N, ne02, 1), (nb00 or bb, rb, rb * N, rb * N * ne02), p)
        src1 = sp.ggml_tensor(t1, (k1, M, ne12, 1), (nb10, 2 * k1, 2 * k1 * M, 2 * k1 * M * ne12), p)
        es = 4 if td == sp.F32 else 2
        dst = sp.ggml_tensor(td, (N, M, ne12, 1), (es, es * N, es * N * M, es * N * M * ne12), p)
        return src0, src1, dst

    assert sp.ggml_supports_mul_mat(*node())
    for t0 in (sp.Q8_0, sp.Q6_K, sp.Q4_K, sp.Q5_K, sp.IQ4_NL, sp.IQ4_XS, sp.F16, sp.BF16):
        assert sp.ggml_supports_mul_mat(*node(t0=t0))
    assert sp.ggml_supports_mul_mat(*node(td=sp.BF16))
    assert sp.ggml_supports_mul_mat(*node(ne12=4, ne02=2))  # broadcast
    assert not sp.ggml_supports_mul_mat(*node(ne12=3, ne02=2))  # not a multiple
    assert not sp.ggml_supports_mul_mat(*node(t0=0))  # F32 src0: not quantized
    assert not sp.ggml_supports_mul_mat(*node(t1=0))  # F32 src1
    assert not sp.ggml_supports_mul_mat(*node(k1=K - 32))  # K mismatch
    assert not sp.ggml_supports_mul_mat(*node(nb10=4))  # non-contiguous src1 rows
    assert not sp.ggml_supports_mul_mat(*node(nb00=36))  # strided blocks
    s0, s1, d = node(t1=0)
    assert sp.lib().spiral_ggml_mul_mat(ctypes.byref(s0), ctypes.byref(s1), ctypes.byref(d), 0, 0) == -9
