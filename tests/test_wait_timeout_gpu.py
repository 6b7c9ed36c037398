"""A bounded device wait that runs out, on one GPU.

The gathered GEMV (spiral_mul_mat_allgather) waits, with a 2 s device-time
limit, for the other ranks' pieces of its output.  Here rank 0 of a world of
2 runs alone: both exchange buffers are local and nobody ever writes rank
1's pieces, so the wait must give up, set bit 8 of the device status
(SPIRAL_ERR_TIMEOUT from spiral_device_status) and end the kernel, leaving
the context usable.  The rank's own columns are still complete and correct,
and a call made while the error bit is set skips its wait instead of waiting
out the limit again; spiral_allgather_exchange_reset zeroes the exchange
for the recovery.  Nothing faults or hangs: the wait is the kernel's own
bounded poll of a flag that nothing sets.
"""

from __future__ import annotations

import time

import numpy as np
import pytest

import oracle
import spiral_b200 as sp
from oracle import formats as F

from .gpu_util import dev_bf16, dev_bytes, tolerance_ok

pytestmark = pytest.mark.gpu


def test_gathered_wait_gives_up_and_reports_timeout(cuda):
    import torch

    assert sp.device_status() == 0
    fid, K, N_total, M = F.Q4_0, 4096, 512, 2
    N_shard = N_total // 2
    raw = F.generate(fid, K, N_total, seed=41)
    x = F.gen_activations(M, K, seed=42)
    rb = F.row_bytes(fid, K)
    w_shard = dev_bytes(raw[: N_shard * rb])
    xd = dev_bf16(x)
    nbytes = sp.allgather_exchange_bytes(N_total)
    own = torch.zeros(nbytes, dtype=torch.uint8, device="cuda")
    absent = torch.zeros(nbytes, dtype=torch.uint8, device="cuda")  # "rank 1": never sends
    peers = torch.tensor([own.data_ptr(), absent.data_ptr()], dtype=torch.int64, device="cuda")
    y = torch.zeros((M, N_total), dtype=torch.bfloat16, device="cuda")

    t0 = time.perf_counter()
    sp.mul_mat_allgather(fid, w_shard, xd, N_shard, K, y, 0, peers, 0, 2)
    torch.cuda.synchronize()
    first = time.perf_counter() - t0
    assert first >= 1.5, first  # it waited (2 s limit) ...
    assert first < 30, first  # ... and gave up

    # the error bit is still set: a second call skips its wait
    t0 = time.perf_counter()
    sp.mul_mat_allgather(fid, w_shard, xd, N_shard, K, y, 0, peers, 0, 2)
    torch.cuda.synchronize()
    assert time.perf_counter() - t0 < 1.0

    L = sp.lib()
    import ctypes

    code = ctypes.c_uint32(0)
    st = L.spiral_device_status(torch.cuda.current_stream().cuda_stream, ctypes.byref(code))
    assert st == -8  # SPIRAL_ERR_TIMEOUT
    assert code.value & 8, code.value  # a rank's gathered pieces never arrived
    assert sp.device_status() == 0  # read-and-clear

    # the rank's own columns are complete and within the MUL_MAT tolerance
    ref = oracle.mul_mat_f64(fid, raw[: N_shard * rb], x, K, N_shard)
    got = y[:, :N_shard].float().cpu().numpy()
    ok, rel = tolerance_ok(got, ref, bf16_out=True)
    assert ok, rel
    # recovery: the exchange (call count, flags, pieces) is zeroed again, and
    # a call on it runs the protocol from its start (world 1: this rank
    # alone), equal bit for bit to the plain MUL_MAT
    assert bool(own.any())
    sp.allgather_exchange_reset(own, N_total)
    torch.cuda.synchronize()
    assert not bool(own.any())
    w_full = dev_bytes(raw)
    solo = torch.tensor([own.data_ptr()], dtype=torch.int64, device="cuda")
    yg = torch.zeros((M, N_total), dtype=torch.bfloat16, device="cuda")
    sp.mul_mat_allgather(fid, w_full, xd, N_total, K, yg, 0, solo, 0, 1)
    want = sp.mul_mat(fid, w_full, xd, N_total, K, y_dtype=sp.BF16)
    assert torch.equal(yg.view(torch.int16), want.view(torch.int16))
    assert sp.device_status() == 0
    # the context is still usable: an ordinary MUL_MAT right after
    y2 = sp.mul_mat(fid, w_shard, xd, N_shard, K, y_dtype=sp.F32).cpu().numpy()
    ok, rel = tolerance_ok(y2, ref, bf16_out=False)
    assert ok, rel
    assert sp.device_status() == 0
