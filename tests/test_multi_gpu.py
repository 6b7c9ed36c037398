"""Multi-GPU paths on 2 B200s (skipped with fewer GPUs): the row-sharded
dequant-GEMV with an NCCL all-gather and with the all-gather fused into the
kernel (NVLink peer stores), and the expert-parallel MoE layer with
NCCL all-to-all dispatch and combine, each rank running libspiral_b200 on its
own GPU.  Checked against the float64 oracle of the whole operation."""

from __future__ import annotations

import os
import socket
from datetime import timedelta

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _ngpu() -> int:
    import torch

    return torch.cuda.device_count() if torch.cuda.is_available() else 0


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, q):
    import torch
    import torch.distributed as dist

    import oracle
    import spiral_b200 as sp
    from oracle import formats as F
    from spiral_b200.dist import expert_range, gather_rows, moe_dispatch_combine, row_range

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=60), device_id=dev)
    try:
        from tests.gpu_util import tolerance_ok

        # dense: Q4_0 14336 x 4096, B = 4, row-sharded
        fid, K, N, M = F.Q4_0, 4096, 1792, 4
        raw = F.generate(fid, K, N, seed=3)
        x = F.gen_activations(M, K, seed=4)
        n0, n1 = row_range(N, world, rank)
        rb = F.row_bytes(fid, K)
        w = torch.from_numpy(raw[n0 * rb:n1 * rb]).to(dev)
        xd = torch.from_numpy(x.view(np.int16)).to(dev).view(torch.bfloat16)
        y_local = sp.mul_mat(fid, w, xd, n1 - n0, K, y_dtype=sp.F32, static_weights=True)
        y = gather_rows(y_local, N).cpu().numpy()
        ok_dense, rel_dense = tolerance_ok(y, oracle.mul_mat_f64(fid, raw, x, K, N), bf16_out=False)

        # the same GEMV with the all-gather fused in (flagged units over
        # NVLink), uneven shards (113 tiles of 16 rows over 2 ranks), every
        # batch size, one output per batch size, several calls in a row
        # through one exchange
        from spiral_b200.dist import AllGatherExchange

        Ng = 1808
        rawg = F.generate(fid, K, Ng, seed=7)
        g0, g1 = row_range(Ng, world, rank)
        wg_shard = torch.from_numpy(rawg[g0 * rb:g1 * rb]).to(dev)
        xc = AllGatherExchange(Ng, dev)
        outs = {B: torch.zeros((B, Ng), dtype=torch.bfloat16, device=dev) for B in (1, 2, 5, 8)}
        ok_fused, rel_fused = True, 0.0
        for it in range(7):
            B = (1, 2, 5, 8)[it % 4]
            xb = F.gen_activations(B, K, seed=20 + it)
            xdb = torch.from_numpy(xb.view(np.int16)).to(dev).view(torch.bfloat16)
            sp.mul_mat_allgather(fid, wg_shard, xdb, g1 - g0, K, outs[B], g0, xc.peers, rank, world)
            yg = outs[B].float().cpu().numpy()
            ok, rel = tolerance_ok(yg, oracle.mul_mat_f64(fid, rawg, xb, K, Ng), bf16_out=True)
            ok_fused, rel_fused = ok_fused and ok, max(rel_fused, rel)
        torch.cuda.synchronize()
        dist.barrier()
        del xc

        # MoE: 16 Q4_0 experts, hidden 512, inter 256, top-4, tokens sharded
        E, H, I, T, topk = 16, 512, 256, 9, 4
        wg = F.gen_experts(fid, E, I, H, seed=1)
        wu = F.gen_experts(fid, E, I, H, seed=2)
        wdn = F.gen_experts(fid, E, H, I, seed=3)
        xm = F.gen_activations(T, H, seed=5)
        ids, wts = F.gen_routing(T, E, topk, seed=6)
        e0, e1 = expert_range(E, world, rank)
        gu, dd = I * F.row_bytes(fid, H), H * F.row_bytes(fid, I)
        wg_l = torch.from_numpy(wg[e0 * gu:e1 * gu]).to(dev)
        wu_l = torch.from_numpy(wu[e0 * gu:e1 * gu]).to(dev)
        wd_l = torch.from_numpy(wdn[e0 * dd:e1 * dd]).to(dev)
        t0, t1 = rank * T // world, (rank + 1) * T // world

        def compute(xr, idr, wr):
            return sp.moe_ffn(fid, wg_l, wu_l, wd_l, xr.view(torch.bfloat16), idr, wr, hidden=H, inter=I,
                              n_experts_local=e1 - e0, expert_first=e0, y_dtype=sp.F32)

        ym = moe_dispatch_combine(torch.from_numpy(xm[t0:t1].view(np.int16)).to(dev),
                                  torch.from_numpy(ids[t0:t1]).to(dev), torch.from_numpy(wts[t0:t1]).to(dev), E,
                                  compute)
        ref = oracle.moe_ffn_f64(fid, wg, wu, wdn, xm, ids, wts, H, I, E)[t0:t1]
        ok_moe, rel_moe = tolerance_ok(ym.cpu().numpy(), ref, bf16_out=False, rel_tol=2e-3)
        q.put((rank, ok_dense, rel_dense, ok_moe, rel_moe, ok_fused, rel_fused, sp.device_status()))
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(_ngpu() < 2, reason="needs 2 GPUs")
def test_two_gpu_row_shard_and_expert_parallel_moe():
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    q = ctx.SimpleQueue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
    assert [p.exitcode for p in procs] == [0, 0]
    for rank, ok_d, rel_d, ok_m, rel_m, ok_f, rel_f, status in (q.get() for _ in range(2)):
        assert ok_d, (rank, rel_d)
        assert ok_f, (rank, rel_f)
        assert ok_m, (rank, rel_m)
        assert status == 0
