"""The allocation-free MoE entry point (spiral_moe_ffn_noalloc).

It is for callers that cannot allocate device memory when they call in (a
plain C host handed device pointers, a serving loop that must not hit
cudaMalloc mid-step, memory owned by a caching allocator or a pre-planned
arena): its scratch is a static 8 MiB array inside the library.  Checked
through the C-ABI against the workspace entry point (spiral_moe_ffn) with the
MoE tolerance of tests/test_moe_gpu.py, on two calls in a row with different
inputs (the shared scratch keeps the first call's contents), and for the
capacity limit on both sides (107 tokens at config-4 dims fit, 108 do not);
one call is also checked straight against the float64 oracle.  Kept in its
own file, collected last.
"""

from __future__ import annotations

import ctypes

import numpy as np
import pytest

import oracle
import spiral_b200 as sp
from oracle import formats as F

from .gpu_util import dev_bf16, dev_bytes, tolerance_ok

pytestmark = pytest.mark.gpu


def _noalloc(L, fid, wg, wu, wd, E, H, I, x, ids, w, topk, y, stream):
    return L.spiral_moe_ffn_noalloc(fid, wg.data_ptr(), wu.data_ptr(), wd.data_ptr(), E, 0, H, I, x.data_ptr(),
                                    x.stride(0), ids.shape[0], ids.data_ptr(), w.data_ptr(), topk, y.data_ptr(),
                                    sp.F32, y.stride(0), 0, stream)


def test_moe_noalloc_matches_workspace_entry_point_on_two_calls(cuda):
    import torch

    L = sp.lib()
    stream = torch.cuda.current_stream().cuda_stream
    fid, E, H, I, topk = F.Q4_0, 32, 2048, 768, 8
    for call, (T, seed) in enumerate(((16, 71), (5, 72))):
        wg = dev_bytes(F.gen_experts(fid, E, I, H, seed=seed))
        wu = dev_bytes(F.gen_experts(fid, E, I, H, seed=seed + 1))
        wd = dev_bytes(F.gen_experts(fid, E, H, I, seed=seed + 2))
        x = dev_bf16(F.gen_activations(T, H, seed=seed + 3)).view(T, H)
        ids_np, w_np = F.gen_routing(T, E, topk, seed=seed + 4)
        ids, w = torch.from_numpy(ids_np).cuda(), torch.from_numpy(w_np).cuda()
        want = sp.moe_ffn(fid, wg, wu, wd, x, ids, w, hidden=H, inter=I, n_experts_local=E, y_dtype=sp.F32)
        got = torch.full((T, H), float("nan"), dtype=torch.float32, device="cuda")
        st = _noalloc(L, fid, wg, wu, wd, E, H, I, x, ids, w, topk, got, stream)
        assert st == 0, (call, L.spiral_last_error())
        torch.cuda.synchronize()
        ok, rel = tolerance_ok(got.cpu().numpy(), want.cpu().numpy().astype(np.float64), bf16_out=False,
                               rel_tol=2e-3)
        assert ok, (call, rel)
        if call == 1:  # and once straight against the float64 oracle
            ref = oracle.moe_ffn_f64(fid, F.gen_experts(fid, E, I, H, seed=seed),
                                     F.gen_experts(fid, E, I, H, seed=seed + 1),
                                     F.gen_experts(fid, E, H, I, seed=seed + 2),
                                     F.gen_activations(T, H, seed=seed + 3), ids_np, w_np, H, I, E)
            ok, rel = tolerance_ok(got.cpu().numpy(), ref, bf16_out=False, rel_tol=2e-3)
            assert ok, rel
    assert sp.device_status() == 0


def test_moe_noalloc_at_config4_dims_up_to_its_limit(cuda):
    """Config-4 dims (128 experts, hidden 2048, inter 768, top-8) at 107
    tokens, the most the static scratch holds, with bf16 output."""
    import torch

    L = sp.lib()
    stream = torch.cuda.current_stream().cuda_stream
    fid, E, H, I, topk, T = F.Q4_0, 128, 2048, 768, 8, 107
    assert sp.moe_workspace_bytes(E, H, I, T, topk) <= 8 << 20
    # 8 distinct experts repeated 16 times (the content is not what is tested)
    wg = dev_bytes(np.tile(F.gen_experts(fid, 8, I, H, seed=81), 16))
    wu = dev_bytes(np.tile(F.gen_experts(fid, 8, I, H, seed=82), 16))
    wd = dev_bytes(np.tile(F.gen_experts(fid, 8, H, I, seed=83), 16))
    x = dev_bf16(F.gen_activations(T, H, seed=84)).view(T, H)
    ids_np, w_np = F.gen_routing(T, E, topk, seed=85)
    ids, w = torch.from_numpy(ids_np).cuda(), torch.from_numpy(w_np).cuda()
    want = sp.moe_ffn(fid, wg, wu, wd, x, ids, w, hidden=H, inter=I, n_experts_local=E, y_dtype=sp.BF16)
    for _ in range(2):
        got = torch.zeros((T, H), dtype=torch.bfloat16, device="cuda")
        st = L.spiral_moe_ffn_noalloc(fid, wg.data_ptr(), wu.data_ptr(), wd.data_ptr(), E, 0, H, I, x.data_ptr(),
                                      x.stride(0), T, ids.data_ptr(), w.data_ptr(), topk, got.data_ptr(), sp.BF16,
                                      got.stride(0), 0, stream)
        assert st == 0, L.spiral_last_error()
        torch.cuda.synchronize()
        ok, rel = tolerance_ok(got.float().cpu().numpy(), want.float().cpu().numpy().astype(np.float64),
                               bf16_out=True, rel_tol=2e-3)
        assert ok, rel
    assert sp.device_status() == 0


def test_moe_noalloc_rejects_dims_beyond_its_scratch(cuda):
    import torch

    L = sp.lib()
    E, H, I, topk, T = 128, 2048, 768, 8, 108  # 8,414,208 bytes of scratch > 8 MiB
    assert sp.moe_workspace_bytes(E, H, I, T, topk) > 8 << 20
    dummy = torch.empty(1 << 16, dtype=torch.uint8, device="cuda")
    p = dummy.data_ptr()
    st = L.spiral_moe_ffn_noalloc(sp.Q4_0, p, p, p, E, 0, H, I, p, H, T, p, p, topk, p, sp.F32, H, 0, 0)
    assert st == -5  # SPIRAL_ERR_CAPACITY, before any launch
    assert b"spiral_moe_ffn with a workspace" in L.spiral_last_error()
