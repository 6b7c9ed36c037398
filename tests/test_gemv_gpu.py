"""Fused dequant-GEMV (decode, M <= 8) on the GPU against the oracle.

Two levels, as in the reference (src/quants/NOTES.md:540-553):
* the reference's own fused-mmul cases (mmul.py, tiled I/O, accumulate into
  caller-zeroed fp32 outputs), checked with the reference's criterion
  allclose(rtol=1e-3, atol=1e-3) and a tighter bound;
* BASELINE config 2 shapes (14336 x 4096, B = 1..8) for all three formats,
  against the float64 dequant-then-matmul oracle with the stated tolerance
  (tests/gpu_util.tolerance_ok).
"""

from __future__ import annotations

import numpy as np
import pytest

import oracle
import spiral_b200 as sp
from oracle import formats as F

from .conftest import load_golden
from .gpu_util import dev_bf16, dev_bytes, host_bits, tolerance_ok

pytestmark = pytest.mark.gpu
FMTS = [F.Q4_0, F.Q8_0, F.Q6_K]


@pytest.mark.parametrize("fid", FMTS, ids=lambda f: F.NAMES[f])
@pytest.mark.parametrize("seed", [1, 2, 3])
def test_unpack_mmul_all_reference_cases(cuda, fid, seed):
    import torch

    g = load_golden(f"ref_default_{F.NAMES[fid]}_s{seed}.npz")
    K, N = int(g["K"]), int(g["N"])
    outputs = torch.zeros(N * 4, dtype=torch.float32, device="cuda")
    sp.unpack_mmul_all(fid, dev_bytes(g["raw"]), dev_bf16(g["inputs_tiled"]), outputs, K, N, 4)
    got = outputs.cpu().numpy().reshape(N // 8, 4, 8).transpose(1, 0, 2).reshape(4, N)
    want = g["expected_outputs"]
    assert np.allclose(got, want, rtol=1e-3, atol=1e-3)  # the reference's own check
    np.testing.assert_allclose(got, want, rtol=1e-5, atol=1e-5 * np.abs(want).max())
    # accumulate semantics: a second call adds the same product again
    sp.unpack_mmul_all(fid, dev_bytes(g["raw"]), dev_bf16(g["inputs_tiled"]), outputs, K, N, 4)
    got2 = outputs.cpu().numpy().reshape(N // 8, 4, 8).transpose(1, 0, 2).reshape(4, N)
    np.testing.assert_allclose(got2, 2 * want, rtol=1e-5, atol=2e-5 * np.abs(want).max())


@pytest.fixture(scope="module")
def big_weights():
    cache = {}

    def get(fid, K, N, seed=0):
        key = (fid, K, N, seed)
        if key not in cache:
            cache[key] = F.generate(fid, K, N, seed)
        return cache[key]

    return get


@pytest.mark.parametrize("fid", FMTS, ids=lambda f: F.NAMES[f])
@pytest.mark.parametrize("M", [1, 2, 3, 4, 8])
def test_gemv_baseline_config2(cuda, big_weights, fid, M):
    K, N = 4096, 14336
    raw = big_weights(fid, K, N)
    x = F.gen_activations(M, K, seed=100 + M)
    ref = oracle.mul_mat_f64(fid, raw, x, K, N)
    w = dev_bytes(raw)
    xd = dev_bf16(x)
    y32 = sp.mul_mat(fid, w, xd, N, K, y_dtype=sp.F32).cpu().numpy()
    ok, rel = tolerance_ok(y32, ref, bf16_out=False)
    assert ok, rel
    assert rel < 1e-5, rel  # fp32 accumulate: only summation order differs
    y16 = host_bits(sp.mul_mat(fid, w, xd, N, K, y_dtype=sp.BF16))
    ok, rel = tolerance_ok(F.bf16_bits_to_f32(y16), ref, bf16_out=True)
    assert ok, rel


@pytest.mark.parametrize("fid", FMTS, ids=lambda f: F.NAMES[f])
@pytest.mark.parametrize(
    "M,N,K",
    [
        (1, 1, 2048),  # one output feature
        (5, 37, 4096),  # ragged N (partial 16-row tile)
        (8, 4096, 4096),
        (2, 2048, 768),  # MoE down-projection K (partial chunk)
        (3, 96, 1536),  # Gemma K: Q6_K window copies
        (12, 64, 2048),  # M > 8: batched GEMV launches
    ],
)
def test_gemv_shapes(cuda, fid, M, N, K):
    if K % F.BLOCK_K[fid]:
        pytest.skip("K not a block multiple")
    raw = F.generate(fid, K, N, seed=N + K)
    x = F.gen_activations(M, K, seed=M * 7)
    ref = oracle.mul_mat_f64(fid, raw, x, K, N)
    y = sp.mul_mat(fid, dev_bytes(raw), dev_bf16(x), N, K, y_dtype=sp.F32).cpu().numpy()
    ok, rel = tolerance_ok(y, ref, bf16_out=False)
    assert ok, rel


@pytest.mark.parametrize("fid", FMTS, ids=lambda f: F.NAMES[f])
def test_gemv_strides_accumulate_ftz(cuda, fid):
    import torch

    K, N, M = 4096, 300, 4
    raw = F.generate(fid, K, N, seed=11)
    x = F.gen_activations(M, K, seed=12)
    # strided activations and outputs inside larger buffers
    xbig = np.zeros((M, K + 64), dtype=np.uint16)
    xbig[:, :K] = x
    y = torch.full((M, N + 8), 0.5, dtype=torch.float32, device="cuda")
    sp.mul_mat(fid, dev_bytes(raw), dev_bf16(xbig), N, K, y, y_dtype=sp.F32, x_row_stride=K + 64,
               y_row_stride=N + 8, accumulate=True, ftz=True)
    ref = oracle.mul_mat_f64(fid, raw, x, K, N, ftz=True) + 0.5
    got = y.cpu().numpy()
    ok, rel = tolerance_ok(got[:, :N], ref, bf16_out=False)
    assert ok, rel
    assert np.all(got[:, N:] == 0.5)


def test_gemv_is_deterministic(cuda, big_weights):
    K, N = 4096, 14336
    raw = big_weights(F.Q4_0, K, N)
    x = dev_bf16(F.gen_activations(8, K, seed=1))
    w = dev_bytes(raw)
    a = sp.mul_mat(F.Q4_0, w, x, N, K, y_dtype=sp.F32).cpu().numpy()
    b = sp.mul_mat(F.Q4_0, w, x, N, K, y_dtype=sp.F32).cpu().numpy()
    assert np.array_equal(a, b)
    assert sp.device_status() == 0


@pytest.mark.parametrize("fid", FMTS, ids=lambda f: F.NAMES[f])
@pytest.mark.parametrize(
    "M,N",
    [
        (1, 16),  # one tile
        (3, 1792),  # 112 tiles < SMs: the 8-way row shard of config 2
        (8, 4112),  # 257 tiles
        (2, 300),  # partial last tile
    ],
)
def test_gemv_small_and_ragged_tile_counts(cuda, fid, M, N):
    """Tile counts below, above and not a multiple of the SM count; bitwise
    repeatable, and the same bits with the early weight stream enabled."""
    K = 4096
    raw = F.generate(fid, K, N, seed=N + 3)
    x = F.gen_activations(M, K, seed=M + 5)
    ref = oracle.mul_mat_f64(fid, raw, x, K, N)
    w, xd = dev_bytes(raw), dev_bf16(x)
    a = sp.mul_mat(fid, w, xd, N, K, y_dtype=sp.F32).cpu().numpy()
    ok, rel = tolerance_ok(a, ref, bf16_out=False)
    assert ok, rel
    b = sp.mul_mat(fid, w, xd, N, K, y_dtype=sp.F32, static_weights=True).cpu().numpy()
    assert np.array_equal(a, b)
    assert sp.device_status() == 0


def test_gemv_back_to_back_shapes(cuda):
    """Consecutive GEMVs of different shapes and formats on one stream, with
    programmatic dependent launch between them, each match the oracle."""
    import torch

    K = 4096
    cases = [(F.Q4_0, 1, 4112), (F.Q8_0, 8, 16), (F.Q6_K, 2, 1792), (F.Q4_0, 5, 300)]
    data = []
    for i, (fid, M, N) in enumerate(cases):
        raw = F.generate(fid, K, N, seed=40 + i)
        x = F.gen_activations(M, K, seed=50 + i)
        y = torch.empty((M, N), dtype=torch.float32, device="cuda")
        data.append((fid, M, N, raw, x, dev_bytes(raw), dev_bf16(x), y))
    for _ in range(2):
        for fid, M, N, raw, x, w, xd, y in data:
            sp.mul_mat(fid, w, xd, N, K, y, y_dtype=sp.F32, static_weights=True)
    torch.cuda.synchronize()
    for fid, M, N, raw, x, w, xd, y in data:
        ok, rel = tolerance_ok(y.cpu().numpy(), oracle.mul_mat_f64(fid, raw, x, K, N), bf16_out=False)
        assert ok, (F.NAMES[fid], M, N, rel)
    assert sp.device_status() == 0


def test_gemv_in_cuda_graph_on_fresh_stream(cuda):
    """Captured into a CUDA graph on a fresh stream, replays match the
    oracle."""
    import torch

    fid, M, N, K = F.Q4_0, 4, 4112, 4096
    raw = F.generate(fid, K, N, seed=9)
    x = F.gen_activations(M, K, seed=10)
    w, xd = dev_bytes(raw), dev_bf16(x)
    y = torch.empty((M, N), dtype=torch.float32, device="cuda")
    s = torch.cuda.Stream()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=s):
        sp.mul_mat(fid, w, xd, N, K, y, y_dtype=sp.F32, static_weights=True, stream=s)
    for _ in range(3):
        y.zero_()
        g.replay()
    torch.cuda.synchronize()
    ok, rel = tolerance_ok(y.cpu().numpy(), oracle.mul_mat_f64(fid, raw, x, K, N), bf16_out=False)
    assert ok, rel
    del g
    assert sp.device_status() == 0


@pytest.mark.parametrize("fid", FMTS, ids=lambda f: F.NAMES[f])
@pytest.mark.parametrize("M,N,K,x_off", [(1, 300, 4096, 1), (8, 4112, 4096, 1), (3, 1792, 6144, 0), (8, 33, 8192, 0)])
def test_gemv_unaligned_activations_and_long_k(cuda, fid, M, N, K, x_off):
    """Activations only 2-byte aligned (staged by gathers) and K above the
    fast staging limit."""
    if K % F.BLOCK_K[fid]:
        pytest.skip("K not a block multiple")
    import torch

    raw = F.generate(fid, K, N, seed=K + N + x_off)
    x = F.gen_activations(M, K, seed=M + 77)
    xbuf = np.zeros(M * K + x_off, dtype=np.uint16)
    xbuf[x_off:] = x.reshape(-1)
    xd = dev_bf16(xbuf)[x_off:].view(M, K)
    y = torch.empty((M, N), dtype=torch.float32, device="cuda")
    sp.mul_mat(fid, dev_bytes(raw), xd, N, K, y, y_dtype=sp.F32, static_weights=True)
    ok, rel = tolerance_ok(y.cpu().numpy(), oracle.mul_mat_f64(fid, raw, x, K, N), bf16_out=False)
    assert ok, rel
    assert sp.device_status() == 0


@pytest.mark.parametrize("fid", FMTS, ids=lambda f: F.NAMES[f])
def test_gathered_gemv_single_rank(cuda, fid):
    """spiral_mul_mat_allgather with world = 1 on one GPU (the one shard is
    the whole width): outputs land in a strided row, the padding after the
    gathered width is left alone, the call count advances once per call (the
    exchange slots alternate), eagerly and in a replayed CUDA graph.  Shard
    offsets and the exchange between ranks are covered on 2 GPUs by
    test_multi_gpu."""
    import torch

    K, N, stride, off = 4096, 1800, 2048, 0  # 1800 rows: a ragged last tile of 8
    raw = F.generate(fid, K, N, seed=31)
    w = dev_bytes(raw)
    y_rows = torch.zeros((8, stride), dtype=torch.bfloat16, device="cuda")
    y = y_rows[:, :N]
    xchg = torch.zeros(sp.allgather_exchange_bytes(N), dtype=torch.uint8, device="cuda")
    peers = torch.tensor([xchg.data_ptr()], dtype=torch.int64, device="cuda")
    calls = 0
    for it, M in enumerate((1, 3, 8, 8)):
        x = F.gen_activations(M, K, seed=40 + it)
        sp.mul_mat_allgather(fid, w, dev_bf16(x), N, K, y, off, peers, 0, 1)
        calls += 1
        got = y_rows[:M].float().cpu().numpy()
        ok, rel = tolerance_ok(got[:, off:off + N], oracle.mul_mat_f64(fid, raw, x, K, N), bf16_out=True)
        assert ok, (M, rel)
        assert not got[:, off + N:].any()
    ctrl = xchg[:8].view(torch.int32).cpu().tolist()
    assert ctrl == [calls, 0]

    x = F.gen_activations(4, K, seed=50)
    xd = dev_bf16(x)
    s = torch.cuda.Stream()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=s):
        sp.mul_mat_allgather(fid, w, xd, N, K, y, off, peers, 0, 1, stream=s)
    y_rows.zero_()
    for _ in range(3):
        g.replay()
    torch.cuda.synchronize()
    calls += 3
    ok, rel = tolerance_ok(y_rows[:4, off:off + N].float().cpu().numpy(), oracle.mul_mat_f64(fid, raw, x, K, N),
                           bf16_out=True)
    assert ok, rel
    del g
    assert xchg[:8].view(torch.int32).cpu().tolist() == [calls, 0]
    assert sp.device_status() == 0


@pytest.mark.parametrize("M", [1, 3, 8])
@pytest.mark.parametrize("N", [4096, 4100])
def test_gemv_gemma_q6_k_output_head_shape(cuda, M, N):
    """The Gemma-style Q6_K output head (K = 1536: 1260-byte rows, not a
    16-byte multiple): N a multiple of 32 runs the six-super-block kernel
    (four-row bulk copies), other N the pipelined GEMV with window copies."""
    fid, K = F.Q6_K, 1536
    raw = F.generate(fid, K, N, seed=77)
    x = F.gen_activations(M, K, seed=78)
    w, xd = dev_bytes(raw), dev_bf16(x)
    y = sp.mul_mat(fid, w, xd, N, K, y_dtype=sp.F32).cpu().numpy()
    ok, rel = tolerance_ok(y, oracle.mul_mat_f64(fid, raw, x, K, N), bf16_out=False)
    assert ok, rel
    assert rel < 1e-5, rel
    assert np.array_equal(sp.mul_mat(fid, w, xd, N, K, y_dtype=sp.F32).cpu().numpy(), y)
    assert sp.device_status() == 0


@pytest.mark.parametrize("ftz", [False, True])
def test_gemv_gemma_head_strided_accumulate(cuda, ftz):
    """Six-super-block kernel with activations at an odd row stride (scalar
    fragment loads), an accumulating strided f32 output, subnormal scales
    flushed or kept, and bf16 output."""
    import torch

    fid, K, N, M = F.Q6_K, 1536, 1024, 5
    raw = F.generate(fid, K, N, seed=21)
    blk = raw.reshape(-1, 210).copy()
    blk[:6, 208:210] = np.array([0x0001, 0x8005, 0x03FF, 0x8000, 0x0000, 0x0200], dtype=np.uint16).view(np.uint8).reshape(-1, 2)
    raw = blk.reshape(-1)
    x = F.gen_activations(M, K, seed=22)
    xbig = np.zeros((M, K + 3), dtype=np.uint16)
    xbig[:, :K] = x
    y = torch.full((M, N + 8), 0.5, dtype=torch.float32, device="cuda")
    sp.mul_mat(fid, dev_bytes(raw), dev_bf16(xbig), N, K, y, y_dtype=sp.F32, x_row_stride=K + 3, y_row_stride=N + 8,
               accumulate=True, ftz=ftz)
    ref = oracle.mul_mat_f64(fid, raw, x, K, N, ftz=ftz)
    got = y.cpu().numpy()
    ok, rel = tolerance_ok(got[:, :N], ref + 0.5, bf16_out=False)
    assert ok, rel
    assert np.all(got[:, N:] == 0.5)
    yb = host_bits(sp.mul_mat(fid, dev_bytes(raw), dev_bf16(x), N, K, y_dtype=sp.BF16, ftz=ftz))
    ok, rel = tolerance_ok(F.bf16_bits_to_f32(yb), ref, bf16_out=True)
    assert ok, rel
    assert sp.device_status() == 0


@pytest.mark.parametrize("fid", FMTS, ids=lambda f: F.NAMES[f])
def test_gemv_rows_off_16_byte_alignment(cuda, fid):
    """Rows at a stride that is 4 mod 16 (window copies) and at a 4-byte
    offset base."""
    from .gpu_util import strided_rows

    K, N, M = 2048, 200, 3
    raw = F.generate(fid, K, N, seed=31)
    rb = F.row_bytes(fid, K)
    stride = rb + 4
    w = dev_bytes(strided_rows(raw, N, rb, stride), offset=4)
    x = F.gen_activations(M, K, seed=32)
    y = sp.mul_mat(fid, w, dev_bf16(x), N, K, y_dtype=sp.F32, w_row_stride=stride).cpu().numpy()
    ok, rel = tolerance_ok(y, oracle.mul_mat_f64(fid, raw, x, K, N), bf16_out=False)
    assert ok, rel


@pytest.mark.parametrize("fid", [F.Q4_0, F.Q8_0], ids=lambda f: F.NAMES[f])
@pytest.mark.parametrize("K", [1536, 3072])
def test_gemv_twelve_warp_shapes(cuda, fid, K):
    """K of 12 decode groups (1536 / 3072: the Gemma 4 E2B hidden size and
    twice it) run the activation-stationary GEMV with 12 decoding warps:
    within the MUL_MAT tolerance for several batch sizes and a ragged last
    tile, repeatable, and the gathered call (world = 1) equal to the plain
    call bit for bit."""
    import torch

    N = 1000
    raw = F.generate(fid, K, N, seed=K + 3)
    w = dev_bytes(raw)
    for M in (1, 5, 8):
        x = F.gen_activations(M, K, seed=M + K)
        xd = dev_bf16(x)
        y = sp.mul_mat(fid, w, xd, N, K, y_dtype=sp.F32).cpu().numpy()
        ok, rel = tolerance_ok(y, oracle.mul_mat_f64(fid, raw, x, K, N), bf16_out=False)
        assert ok, (M, rel)
        assert np.array_equal(sp.mul_mat(fid, w, xd, N, K, y_dtype=sp.F32).cpu().numpy(), y)
        yb = sp.mul_mat(fid, w, xd, N, K, y_dtype=sp.BF16)
        yg = torch.zeros((M, N), dtype=torch.bfloat16, device="cuda")
        xchg = torch.zeros(sp.allgather_exchange_bytes(N), dtype=torch.uint8, device="cuda")
        peers = torch.tensor([xchg.data_ptr()], dtype=torch.int64, device="cuda")
        sp.mul_mat_allgather(fid, w, xd, N, K, yg, 0, peers, 0, 1)
        assert torch.equal(yg.view(torch.int16), yb.view(torch.int16))
    assert sp.device_status() == 0
