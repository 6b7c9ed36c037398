"""The expert-parallel MoE entry point (spiral_moe_ffn_ep) on one GPU.

* world = 1: the combine kernel runs its whole exchange protocol against this
  rank's own exchange buffer; the result must equal spiral_moe_ffn bit for
  bit (same kernels, same summation order), on consecutive calls (the
  exchange's two parity slots) with bf16 and fp32 outputs.
* world = 2 with the second rank absent: the owner's bounded wait for the
  missing partials gives up after 2 s, sets bit 8 of the device status and
  ends the kernel, leaving the context usable.  Nothing faults or hangs: the
  wait is the kernel's own bounded poll of a flag that nothing sets; after
  spiral_moe_ep_exchange_reset the exchange serves a world = 1 call again.
The multi-rank combine itself is checked on 2+ GPUs in tests/test_multi_gpu.py.
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


def _layer(fid, E, H, I, T, topk, seed):
    import torch

    wg, wu, wd = (F.gen_experts(fid, E, I, H, seed=seed), F.gen_experts(fid, E, I, H, seed=seed + 1),
                  F.gen_experts(fid, E, H, I, seed=seed + 2))
    x = F.gen_activations(T, H, seed=seed + 3)
    ids, w = F.gen_routing(T, E, topk, seed=seed + 4)
    dev = (dev_bytes(wg), dev_bytes(wu), dev_bytes(wd), dev_bf16(x).view(T, H), torch.from_numpy(ids).cuda(),
           torch.from_numpy(w).cuda())
    return (wg, wu, wd, x, ids, w), dev


def test_moe_ep_world1_equals_single_gpu_layer(cuda):
    import torch

    fid, E, H, I, topk, max_tokens = F.Q4_0, 32, 2048, 768, 8, 64
    xchg = torch.zeros(sp.moe_ep_exchange_bytes(H, max_tokens), dtype=torch.uint8, device="cuda")
    peers = torch.tensor([xchg.data_ptr()], dtype=torch.int64, device="cuda")
    for call, (T, ydt) in enumerate(((9, sp.BF16), (64, sp.F32), (1, sp.BF16))):
        host, (wg, wu, wd, x, ids, w) = _layer(fid, E, H, I, T, topk, seed=30 + call)
        want = sp.moe_ffn(fid, wg, wu, wd, x, ids, w, hidden=H, inter=I, n_experts_local=E, y_dtype=ydt)
        got = sp.moe_ffn_ep(fid, wg, wu, wd, x, ids, w, hidden=H, inter=I, n_experts_local=E, expert_first=0,
                            exchange_peers_dev=peers, rank=0, world=1, max_tokens=max_tokens, y_dtype=ydt)
        torch.cuda.synchronize()
        a = got.view(torch.int16 if ydt == sp.BF16 else torch.int32).cpu().numpy()
        b = want.view(torch.int16 if ydt == sp.BF16 else torch.int32).cpu().numpy()
        assert np.array_equal(a, b), call
        if call == 0:  # and once against the float64 oracle
            ref = oracle.moe_ffn_f64(fid, *host[:3], host[3], host[4], host[5], H, I, E)
            ok, rel = tolerance_ok(got.float().cpu().numpy(), ref, bf16_out=True, rel_tol=2e-3)
            assert ok, rel
    assert sp.device_status() == 0


def test_moe_ep_absent_rank_times_out_and_reports(cuda):
    import ctypes

    import torch

    fid, E, H, I, topk, T, max_tokens = F.Q4_0, 8, 2048, 768, 8, 2, 4
    _, (wg, wu, wd, x, ids, w) = _layer(fid, E, H, I, T, topk, seed=50)
    nbytes = sp.moe_ep_exchange_bytes(H, max_tokens)
    own = torch.zeros(nbytes, dtype=torch.uint8, device="cuda")
    absent = torch.zeros(nbytes, dtype=torch.uint8, device="cuda")  # "rank 1": never sends
    peers = torch.tensor([own.data_ptr(), absent.data_ptr()], dtype=torch.int64, device="cuda")
    t0 = time.perf_counter()
    sp.moe_ffn_ep(fid, wg, wu, wd, x, ids, w, hidden=H, inter=I, n_experts_local=E, expert_first=0,
                  exchange_peers_dev=peers, rank=0, world=2, max_tokens=max_tokens)
    torch.cuda.synchronize()
    waited = time.perf_counter() - t0
    assert 1.5 <= waited < 30, waited
    code = ctypes.c_uint32(0)
    st = sp.lib().spiral_device_status(torch.cuda.current_stream().cuda_stream, ctypes.byref(code))
    assert st == -8 and code.value & 8, (st, code.value)
    # the context is still usable
    y = sp.moe_ffn(fid, wg, wu, wd, x, ids, w, hidden=H, inter=I, n_experts_local=E)
    torch.cuda.synchronize()
    assert torch.isfinite(y.float()).all()
    assert sp.device_status() == 0
    # recovery: the zeroed exchange runs the protocol from its start (world 1)
    assert bool(own.any())
    sp.moe_ep_exchange_reset(own, H, max_tokens)
    torch.cuda.synchronize()
    assert not bool(own.any())
    solo = torch.tensor([own.data_ptr()], dtype=torch.int64, device="cuda")
    got = sp.moe_ffn_ep(fid, wg, wu, wd, x, ids, w, hidden=H, inter=I, n_experts_local=E, expert_first=0,
                        exchange_peers_dev=solo, rank=0, world=1, max_tokens=max_tokens)
    torch.cuda.synchronize()
    assert torch.equal(got.view(torch.int16), y.view(torch.int16))
    assert sp.device_status() == 0
