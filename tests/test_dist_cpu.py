"""Host logic of the multi-GPU paths on CPU: world_size-2 gloo process groups
run the same dispatch/combine and all-gather code the GPU ranks run, with the
float64 oracle as the per-rank compute (spiral_b200.dist)."""

from __future__ import annotations

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from spiral_b200.dist import expert_range, row_range


def test_row_range_covers_rows_in_tile_multiples():
    for n in (16, 300, 1792, 14336):
        for world in (1, 2, 3, 4, 8):
            bounds = [row_range(n, world, r) for r in range(world)]
            assert bounds[0][0] == 0 and bounds[-1][1] == n
            for (a0, a1), (b0, b1) in zip(bounds, bounds[1:]):
                assert a1 == b0
            assert all(b0 % 16 == 0 for b0, _ in bounds)


def test_expert_range_partitions_experts():
    for E in (128, 16, 5):
        for world in (1, 2, 4, 8):
            if world > E:
                continue
            got = [expert_range(E, world, r) for r in range(world)]
            assert got[0][0] == 0 and got[-1][1] == E
            assert all(a1 == b0 for (_, a1), (b0, _) in zip(got, got[1:]))


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _init(rank, world, port):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)


def _gather_worker(rank, world, port, q):
    import oracle
    from oracle import formats as F
    from spiral_b200.dist import gather_rows

    _init(rank, world, port)
    try:
        fid, K, N, M = F.Q8_0, 256, 64, 3
        raw = F.generate(fid, K, N, seed=1)
        x = F.gen_activations(M, K, seed=2)
        n0, n1 = row_range(N, world, rank)
        rb = F.row_bytes(fid, K)
        y_local = oracle.mul_mat_f64(fid, raw[n0 * rb:n1 * rb], x, K, n1 - n0)
        y = gather_rows(torch.from_numpy(y_local), N)
        full = oracle.mul_mat_f64(fid, raw, x, K, N)
        q.put((rank, float(np.abs(y.numpy() - full).max())))
    finally:
        dist.destroy_process_group()


def _moe_worker(rank, world, port, q):
    import oracle
    from oracle import formats as F
    from spiral_b200.dist import moe_dispatch_combine

    _init(rank, world, port)
    try:
        fid, E, H, I, T, topk = F.Q4_0, 8, 64, 32, 7, 3
        wg = F.gen_experts(fid, E, I, H, seed=1)
        wu = F.gen_experts(fid, E, I, H, seed=2)
        wd = F.gen_experts(fid, E, H, I, seed=3)
        x = F.gen_activations(T, H, seed=4)
        ids, w = F.gen_routing(T, E, topk, seed=5)
        e0, e1 = expert_range(E, world, rank)
        gu, dd = I * F.row_bytes(fid, H), H * F.row_bytes(fid, I)
        t0, t1 = rank * T // world, (rank + 1) * T // world  # this rank's tokens

        def compute(xr, idr, wr):
            part = oracle.moe_ffn_f64(fid, wg[e0 * gu:e1 * gu], wu[e0 * gu:e1 * gu], wd[e0 * dd:e1 * dd],
                                      xr.numpy().view(np.uint16), idr.numpy(), wr.numpy(), H, I, e1 - e0,
                                      expert_first=e0)
            return torch.from_numpy(part.astype(np.float32))

        y = moe_dispatch_combine(torch.from_numpy(x[t0:t1].view(np.int16)), torch.from_numpy(ids[t0:t1]),
                                 torch.from_numpy(w[t0:t1]), E, compute)
        full = oracle.moe_ffn_f64(fid, wg, wu, wd, x, ids, w, H, I, E)[t0:t1]
        q.put((rank, float(np.abs(y.numpy() - full).max() / max(1e-30, np.abs(full).max()))))
    finally:
        dist.destroy_process_group()


def _spawn(fn, world=2):
    ctx = mp.get_context("spawn")
    q = ctx.SimpleQueue()
    port = _free_port()
    procs = [ctx.Process(target=fn, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
    codes = [p.exitcode for p in procs]
    assert codes == [0] * world, codes
    return [q.get() for _ in range(world)]


def test_row_sharded_gather_matches_full_product():
    for rank, err in _spawn(_gather_worker):
        assert err < 1e-9, (rank, err)


def test_moe_expert_parallel_dispatch_combine_matches_full_layer():
    for rank, rel in _spawn(_moe_worker):
        assert rel < 1e-6, (rank, rel)  # float32 transport of float64 partials
