"""Multi-GPU paths on min(8, visible) B200s (skipped with fewer than 2): every
rank is a process with its own GPU running libspiral_b200.

* dense row-sharded MUL_MAT (BASELINE config 2 dims, 14336 x 4096 Q4_0):
  NCCL all-gather, and the all-gather fused into the GEMV (flagged NVLink
  units): equal bit for bit to spiral_mul_mat on the whole weight, on every
  rank, for B = 1, 2, 5, 8 and several calls through one exchange, before
  and after the exchange's recovery reset; checked against the float64
  oracle once;
* expert-parallel MoE layer (BASELINE config 4 dims: 128 Q4_0 experts,
  hidden 2048, inter 768, top-8, T = 1 and 64) through spiral_moe_ffn_ep
  (combine fused over NVLink): identical on every rank and within the MoE
  tolerance of the float64 oracle of the whole layer, the last call after
  the exchange's recovery reset;
The fused exchanges wait on the device for at most 2 s, so the ranks enter
each one together (a barrier after every host-side oracle check).
* the Python NCCL all-to-all dispatch/combine (spiral_b200.dist) at toy dims.
"""

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


def _bits(t):
    import torch

    return t.contiguous().view(torch.int16 if t.element_size() == 2 else torch.int32)


def _worker(rank, world, port, q):
    import torch
    import torch.distributed as dist

    import oracle
    import spiral_b200 as sp
    from oracle import formats as F
    from spiral_b200.dist import AllGatherExchange, MoeExchange, expert_range, gather_rows, moe_dispatch_combine, row_range

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=120), device_id=dev)
    res = {"rank": rank}
    try:
        from tests.gpu_util import tolerance_ok

        fid, K = F.Q4_0, 4096
        rb = F.row_bytes(fid, K)

        # dense, NCCL all-gather after the shard GEMV
        N, M = 1792, 4
        raw = F.generate(fid, K, N, seed=3)
        x = F.gen_activations(M, K, seed=4)
        n0, n1 = row_range(N, world, rank)
        w = torch.from_numpy(raw[n0 * rb:n1 * rb]).to(dev)
        xd = torch.from_numpy(x.view(np.int16)).to(dev).view(torch.bfloat16)
        y_local = sp.mul_mat(fid, w, xd, n1 - n0, K, y_dtype=sp.F32, static_weights=True)
        y = gather_rows(y_local, N).cpu().numpy()
        res["dense_nccl"] = tolerance_ok(y, oracle.mul_mat_f64(fid, raw, x, K, N), bf16_out=False)

        # dense, all-gather fused in: config 2 dims, bitwise vs the whole weight
        Ng = 14336
        rawg = F.generate(fid, K, Ng, seed=7)
        g0, g1 = row_range(Ng, world, rank)
        wg_shard = torch.from_numpy(rawg[g0 * rb:g1 * rb]).to(dev)
        wg_full = torch.from_numpy(rawg).to(dev)
        xc = AllGatherExchange(Ng, dev)
        outs = {B: torch.zeros((B, Ng), dtype=torch.bfloat16, device=dev) for B in (1, 2, 5, 8)}
        mism, rel_max = 0, 0.0
        for it in range(7):
            B = (1, 2, 5, 8)[it % 4]
            xb = F.gen_activations(B, K, seed=20 + it)
            xdb = torch.from_numpy(xb.view(np.int16)).to(dev).view(torch.bfloat16)
            sp.mul_mat_allgather(fid, wg_shard, xdb, g1 - g0, K, outs[B], g0, xc.peers, rank, world)
            want = sp.mul_mat(fid, wg_full, xdb, Ng, K, y_dtype=sp.BF16)
            mism += int((_bits(outs[B]) != _bits(want)).sum().item())
            if it == 3:
                if rank == 0:
                    ok, rel = tolerance_ok(outs[B].float().cpu().numpy(), oracle.mul_mat_f64(fid, rawg, xb, K, Ng),
                                           bf16_out=True)
                    res["fused_oracle"] = (ok, rel)
                # the ranks enter every exchange together: its device waits
                # give up after 2 s, and the oracle above takes longer
                dist.barrier()
                # the recovery reset (collective): the calls after it start
                # from a zeroed exchange and must still match bit for bit
                xc.reset()
        res["fused_mismatch"] = mism
        torch.cuda.synchronize()
        dist.barrier()
        del xc

        # expert-parallel MoE at config 4 dims through spiral_moe_ffn_ep
        E, H, I, topk = 128, 2048, 768, 8
        e0, e1 = expert_range(E, world, rank)
        gu, dd = I * F.row_bytes(fid, H), H * F.row_bytes(fid, I)
        # experts are generated per expert id, so every rank builds only its own
        wg_l = torch.from_numpy(np.concatenate([F.generate(fid, H, I, seed=11000 + e) for e in range(e0, e1)])).to(dev)
        wu_l = torch.from_numpy(np.concatenate([F.generate(fid, H, I, seed=12000 + e) for e in range(e0, e1)])).to(dev)
        wd_l = torch.from_numpy(np.concatenate([F.generate(fid, I, H, seed=13000 + e) for e in range(e0, e1)])).to(dev)
        mx = MoeExchange(H, 64, dev)
        for i, T in enumerate((1, 64, 1)):
            if i == 2:
                mx.reset()  # the last call starts from a zeroed exchange
            xm = F.gen_activations(T, H, seed=500 + T)
            ids, wts = F.gen_routing(T, E, topk, seed=600 + T)
            xmd = torch.from_numpy(xm.view(np.int16)).to(dev).view(torch.bfloat16).view(T, H)
            y = sp.moe_ffn_ep(fid, wg_l, wu_l, wd_l, xmd, torch.from_numpy(ids).to(dev),
                              torch.from_numpy(wts).to(dev), hidden=H, inter=I, n_experts_local=e1 - e0,
                              expert_first=e0, exchange_peers_dev=mx.peers, rank=rank, world=world, max_tokens=64,
                              y_dtype=sp.F32)
            torch.cuda.synchronize()
            allys = [torch.empty_like(y) for _ in range(world)]
            dist.all_gather(allys, y)
            res[f"ep_identical_T{T}"] = all(torch.equal(_bits(allys[0]), _bits(a)) for a in allys)
            if rank == 0 and f"ep_oracle_T{T}" not in res:
                used = sorted(set(int(v) for v in ids.reshape(-1)))
                if "all_experts" not in res:  # the whole layer's experts, once (host only)
                    res["all_experts"] = tuple(np.concatenate([F.generate(fid, k, n, seed=s0 + e) for e in range(E)])
                                               for s0, k, n in ((11000, H, I), (12000, H, I), (13000, I, H)))
                ref = oracle.moe_ffn_f64(fid, *res["all_experts"], xm, ids, wts, H, I, E)
                res[f"ep_oracle_T{T}"] = tolerance_ok(y.cpu().numpy(), ref, bf16_out=False, rel_tol=2e-3)
                res[f"ep_experts_T{T}"] = len(used)
            res[f"ep_status_T{T}"] = sp.device_status()
            dist.barrier()  # rank 0's oracle runs for seconds: start the next exchange together
        res.pop("all_experts", None)
        torch.cuda.synchronize()
        dist.barrier()
        del mx

        # Python NCCL all-to-all dispatch/combine over spiral_moe_ffn (toy dims)
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
        res["a2a"] = tolerance_ok(ym.cpu().numpy(), ref, bf16_out=False, rel_tol=2e-3)
        res["status"] = sp.device_status()
        q.put(res)
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(_ngpu() < 2, reason="needs 2 GPUs")
def test_multi_gpu_row_shard_and_expert_parallel_moe():
    import torch.multiprocessing as mp

    world = min(8, _ngpu())
    ctx = mp.get_context("spawn")
    q = ctx.SimpleQueue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=600)
    assert [p.exitcode for p in procs] == [0] * world
    results = [q.get() for _ in range(world)]
    for r in results:
        assert r["dense_nccl"][0], r
        assert r["fused_mismatch"] == 0, r
        assert r["a2a"][0], r
        for T in (1, 64):
            assert r[f"ep_identical_T{T}"], r
            assert r[f"ep_status_T{T}"] == 0, r
        assert r["status"] == 0, r
    r0 = next(r for r in results if r["rank"] == 0)
    assert r0["fused_oracle"][0], r0
    for T in (1, 64):
        assert r0[f"ep_oracle_T{T}"][0], r0
