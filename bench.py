#!/usr/bin/env python
"""bench.py — throughput of the spiral_b200 hot path on B200.

Headline workload: Q4_0 dequant-GEMV decode,
W = 14336 x 4096 (out x in, 33,030,144 bytes of canonical Q4_0 blocks),
bf16 activations x = [B, 4096] ~ N(0,1), fp32 accumulate, bf16 out, for
B in {1, 2, 4, 8}.  One "step" is that sweep: four MUL_MAT calls, each one
streaming the whole weight from HBM.  The metric is weight GB/s: weight
bytes streamed per second (whole job, all ranks).

* Weights rotate over enough distinct copies that their total exceeds the
  126 MB L2 (inputs larger than L2 between timed iterations; no L2 flush).
* Steps are replayed as CUDA graphs of the C-ABI calls (launch overhead off
  the critical path); device time with CUDA events, max over ranks.
* N > 1 (torchrun): the weight is row-sharded by output feature, each rank
  runs its shard and the bf16 outputs are all-gathered over NCCL, so every
  rank ends each MUL_MAT with the full y.  Total work is fixed: strong scaling.
* e2e: the same sweep through the public C-ABI with host buffers: every step
  copies that step's activations from pinned host memory and reads every
  output back to pinned host memory inside the timed region.  Weights stay
  resident (uploaded once, as at model load).
* cpu_baseline / --impl reference: the C restatement of the reference's
  dequant-then-fp32-matmul (oracle/oracle.c, OpenMP on every host core),
  timed on a bounded sample of the same sweep.
"""

from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import time
from pathlib import Path

import numpy as np

REPO = Path(__file__).resolve().parent
sys.path.insert(0, str(REPO))

K_DIM, N_DIM = 4096, 14336
BATCHES = (1, 2, 4, 8)
L2_BYTES = 126 * 1024 * 1024


def parse_args(argv=None):
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20000)
    ap.add_argument("--warmup", type=int, default=200)
    ap.add_argument("--impl", choices=("spiral", "reference"), default="spiral")
    ap.add_argument("--fmt", default="q4_0", choices=("q4_0", "q8_0", "q6_k"))
    ap.add_argument("--no-extras", action="store_true", help="skip the per-format / per-batch extras")
    ap.add_argument("--cpu-seconds", type=float, default=10.0, help="CPU baseline sample budget")
    ap.add_argument("--profile", choices=("gemv", "dequant", "gemm"), default=None,
                    help="ncu helper: run --warmup + --steps eager launches of one kernel on one GPU "
                         "(B from --batch), nothing else")
    ap.add_argument("--batch", type=int, default=1, help="activation vectors for --profile gemv / gemm")
    ap.add_argument("--features", type=int, default=N_DIM, help="output features for --profile gemv / gemm")
    return ap.parse_args(argv)


def run_profile(args):
    """A few plain launches of one kernel for ncu (fresh weight copies per
    launch so every launch reads HBM)."""
    import torch

    import spiral_b200 as sp
    from oracle import formats as F

    torch.cuda.set_device(0)
    fid = F.BY_NAME[args.fmt]
    K = K_DIM
    N = args.features if args.profile in ("gemv", "gemm") else (N_DIM if args.fmt != "q4_0" else 4096)
    raw = F.generate(fid, K, N, seed=0)
    n = args.warmup + args.steps
    ws = [torch.from_numpy(raw).cuda() for _ in range(min(n, 8))]
    if args.profile in ("gemv", "gemm"):
        x = torch.from_numpy(F.gen_activations(args.batch, K, seed=1).view(np.int16)).cuda().view(torch.bfloat16)
        y = torch.empty((args.batch, N), dtype=torch.bfloat16, device="cuda")
        for i in range(n):
            sp.mul_mat(fid, ws[i % len(ws)], x, N, K, y, y_dtype=sp.BF16, static_weights=True)
    else:
        out = torch.empty((N, K), dtype=torch.bfloat16, device="cuda")
        for i in range(n):
            sp.dequant_bf16(fid, ws[i % len(ws)], K, N, out)
    torch.cuda.synchronize()
    print(json.dumps({"profile": args.profile, "fmt": args.fmt, "launches": n, "device_status": sp.device_status()}))
    return 0


def dist_env():
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", str(rank)))
    return rank, world, local


def measured_peaks():
    p = REPO / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return float(d["hbm_gbs"]), float(d["bf16_tflops"]), "measured"
    return 6650.0, 1590.0, "fallback"


def profile_traffic(kernel_key: str):
    """Per-launch DRAM bytes of the dominant kernel from the committed ncu
    summary (profiles/dram_traffic.txt: `<key> <bytes_per_launch>`)."""
    p = REPO / "profiles" / "dram_traffic.txt"
    if not p.exists():
        return None
    for line in p.read_text().splitlines():
        parts = line.split()
        if len(parts) >= 2 and parts[0] == kernel_key and not line.startswith("#"):
            try:
                return float(parts[1])
            except ValueError:
                return None
    return None


class ClockSampler:
    """nvidia-smi clocks + throttle reasons sampled during the timed region."""

    FIELDS = (
        "index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
        "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
        "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap"
    )

    def __init__(self, local_index: int):
        # nvidia-smi numbers GPUs physically; map through CUDA_VISIBLE_DEVICES
        vis = [v.strip() for v in os.environ.get("CUDA_VISIBLE_DEVICES", "").split(",") if v.strip()]
        self.gpu = vis[local_index] if local_index < len(vis) else str(local_index)
        self.proc = None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "100"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except (OSError, FileNotFoundError):
            self.proc = None
        time.sleep(0.3)
        return self

    def __exit__(self, *exc):
        self.out = ""
        if self.proc is not None:
            time.sleep(0.15)
            self.proc.terminate()
            try:
                self.out, _ = self.proc.communicate(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
                self.out, _ = self.proc.communicate()
        return False

    def summary(self):
        rows = []
        for line in (self.out or "").splitlines():
            f = [x.strip() for x in line.split(",")]
            if len(f) < 9:
                continue
            try:
                rows.append((float(f[1]), float(f[2]), f[5], f[6], f[7], f[8]))
            except ValueError:
                continue
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"], "samples": 0}
        names = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")
        reasons = sorted({n for r in rows for n, v in zip(names, r[2:]) if v.lower() == "active"})
        return {"sm_mhz": statistics.median(r[0] for r in rows), "sm_max_mhz": max(r[1] for r in rows),
                "reasons": reasons, "samples": len(rows)}


# --------------------------------------------------------------- reference


def cpu_sweep_rate(fid: int, raw: np.ndarray, K: int, N: int, xs: dict, budget_s: float, rows: int | None = None):
    """Time the oracle's dequant-then-fp32-matmul sweep (B = 1, 2, 4, 8) on
    the first `rows` output features; returns (weight GB/s, reps, rows)."""
    import oracle
    from oracle import formats as F

    rows = N if rows is None else max(16, min(N, rows))
    sub = raw[: rows * F.row_bytes(fid, K)]
    wbytes = rows * F.row_bytes(fid, K)
    oracle.mul_mat_f32(fid, sub, xs[1], K, min(rows, 64))  # warm the pool
    reps, t0 = 0, time.perf_counter()
    while True:
        for B in BATCHES:
            oracle.mul_mat_f32(fid, sub, xs[B], K, rows)
        reps += 1
        el = time.perf_counter() - t0
        if el >= budget_s:
            break
    return reps * len(BATCHES) * wbytes / el / 1e9, reps, rows


def run_reference(args):
    rank, world, _ = dist_env()
    if rank != 0:
        return 0
    from oracle import formats as F

    fid = F.BY_NAME[args.fmt]
    K, N = K_DIM, N_DIM
    raw = F.generate(fid, K, N, seed=0)
    xs = {B: F.gen_activations(B, K, seed=100 + B) for B in BATCHES}
    cores = os.cpu_count() or 1
    # one full step to size the bounded per-step sample
    t0 = time.perf_counter()
    cpu_sweep_rate(fid, raw, K, N, xs, budget_s=0.0)
    full = time.perf_counter() - t0
    total_budget = 120.0
    per_step = total_budget / max(1, args.steps + args.warmup)
    rows = N if full <= per_step else max(16, int(N * per_step / full) // 16 * 16)
    import oracle

    sub = raw[: rows * F.row_bytes(fid, K)]
    for _ in range(args.warmup):
        for B in BATCHES:
            oracle.mul_mat_f32(fid, sub, xs[B], K, rows)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        for B in BATCHES:
            oracle.mul_mat_f32(fid, sub, xs[B], K, rows)
    el = time.perf_counter() - t0
    wbytes = rows * F.row_bytes(fid, K) * len(BATCHES)
    value = wbytes * args.steps / el / 1e9
    sample = f"{rows} of {N} rows per step (B=1,2,4,8 sweep, K={K}), {args.steps} steps"
    line = {
        "impl": "reference",
        "metric": f"dequant-GEMV weight GB/s ({args.fmt.upper()} {N}x{K}, B=1,2,4,8)",
        "value": value,
        "unit": "GB/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": el / args.steps * 1e3,
        "higher_is_better": True,
        "scaling": "strong",
        "vs_baseline": None,
        "dtype": "f32",
        "data": "synthetic (seeded BASELINE distributions)",
        "config": {"workload": f"cfg2 {args.fmt} dequant-GEMV {N}x{K} B=1,2,4,8 (CPU oracle port)",
                   "l2": "n/a (CPU)"},
        "cpu_baseline": {"value": value, "unit": "GB/s", "cores": cores, "kind": "port", "sample": sample},
        "e2e": {"value": value, "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "gpu_launches": 0,
    }
    print(json.dumps(line), flush=True)
    return 0


# ------------------------------------------------------------------ spiral


def run_spiral(args):
    import torch
    import torch.distributed as dist

    import spiral_b200 as sp
    from oracle import formats as F  # generators only (seeded inputs)

    rank, world, local = dist_env()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta

        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=dev)
    sp.lib()

    fid = F.BY_NAME[args.fmt]
    K, N = K_DIM, N_DIM
    from spiral_b200.dist import AllGatherExchange, gather_rows, row_range

    n0, n1 = row_range(N, world, rank)
    Nr = n1 - n0
    assert Nr * world == N, "equal row shards (N a multiple of 16 * world)"
    rb = F.row_bytes(fid, K)
    raw = F.generate(fid, K, N, seed=0)
    shard = raw[n0 * rb : n1 * rb]
    shard_bytes = Nr * rb
    copies = max(2, min(256, math.ceil(2 * L2_BYTES / shard_bytes)))
    w0 = torch.from_numpy(shard).to(dev)
    weights = [w0] + [w0.clone() for _ in range(copies - 1)]
    xs = {B: torch.from_numpy(F.gen_activations(B, K, seed=100 + B).view(np.int16)).to(dev).view(torch.bfloat16)
          for B in BATCHES}
    ys = {B: torch.empty((B, Nr), dtype=torch.bfloat16, device=dev) for B in BATCHES}
    # N > 1: the GEMV sends its shard to every other rank over NVLink and
    # gathers theirs into its own full output (spiral_mul_mat_allgather)
    xc = AllGatherExchange(N, dev) if world > 1 else None
    yfull = {B: torch.empty((B, N), dtype=torch.bfloat16, device=dev) for B in BATCHES}

    def mul_mat_full(w, xb, B):
        if world > 1:
            sp.mul_mat_allgather(fid, w, xb, Nr, K, yfull[B], n0, xc.peers, rank, world)
            return yfull[B]
        sp.mul_mat(fid, w, xb, Nr, K, ys[B], y_dtype=sp.BF16, static_weights=True)
        return ys[B]

    # every MUL_MAT of the sweep reads a different weight copy, so no launch
    # finds its weights in L2 (the last use of a copy is `copies` launches ago)
    def sweep(i):
        for j, B in enumerate(BATCHES):
            mul_mat_full(weights[(i * len(BATCHES) + j) % copies], xs[B], B)

    def sweep_nccl(i):  # the same step with a separate NCCL all-gather (comparison only)
        for j, B in enumerate(BATCHES):
            w = weights[(i * len(BATCHES) + j) % copies]
            sp.mul_mat(fid, w, xs[B], Nr, K, ys[B], y_dtype=sp.BF16, static_weights=True)
            gather_rows(ys[B], N)

    stream = torch.cuda.Stream(device=dev)
    # warm-up (also configures kernel attributes and the per-stream GEMV
    # scratch before any capture; graphs are captured on `stream`)
    for i in range(3):
        sweep(i)
    # the side stream must not overlap the default stream's calls (gathered
    # calls on one exchange are strictly ordered)
    torch.cuda.synchronize()
    with torch.cuda.stream(stream):
        sweep(0)
        if world > 1:
            sweep_nccl(0)
    torch.cuda.synchronize()
    if sp.device_status() != 0:
        raise SystemExit(f"rank {rank}: a device-side wait gave up during warm-up")
    graph_steps = copies if copies <= 64 else 64

    def capture(nsteps, start, body):
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=stream):
            for j in range(nsteps):
                body(start + j)
        return g

    def run_steps(nsteps, graphs_cache, body, key):
        """Replay graphs for exactly nsteps steps of `body`."""
        full, tail = divmod(nsteps, graph_steps)
        if "main" not in graphs_cache:
            graphs_cache["main"] = capture(graph_steps, 0, body)
        if tail and ("tail", tail) not in graphs_cache:
            graphs_cache[("tail", tail)] = capture(tail, 0, body)
        for _ in range(full):
            graphs_cache["main"].replay()
        if tail:
            graphs_cache[("tail", tail)].replay()

    def timed(nsteps, warm, body, cache, sampler=None):
        run_steps(warm, cache, body, "w")
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        cs = torch.cuda.current_stream()
        s.record(cs)
        run_steps(nsteps, cache, body, "t")
        e.record(cs)
        torch.cuda.synchronize()
        ms = s.elapsed_time(e)
        if world > 1:
            t = torch.tensor([ms], device=dev)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            ms = float(t.item())
        return ms

    main_cache = {}
    with ClockSampler(local) as clk:
        ms = timed(args.steps, max(3, args.warmup), sweep, main_cache)
    ms_per_step = ms / args.steps
    wbytes_step = N * rb * len(BATCHES)  # whole job: every rank streams its shard
    value = wbytes_step / (ms_per_step * 1e-3) / 1e9

    # roofline of the dominant kernel: algorithmic bytes (weights + x + y) per
    # launch over the per-launch time.  At N=1 the timed region holds only
    # GEMV launches, so the per-launch time is the timed region / launches
    # (an upper bound: graph gaps between kernels count against the kernel).
    hbm_peak, tc_peak, peak_kind = measured_peaks()
    if world == 1:
        alg = sum(rb * Nr + B * K * 2 + B * Nr * 2 for B in BATCHES)
        achieved = alg / len(BATCHES) / (ms_per_step * 1e-3 / len(BATCHES)) / 1e9
    else:
        # kernel-only time on this rank: same graphs without the collectives
        cache_k = {}

        def sweep_local(i):
            for j, B in enumerate(BATCHES):
                w = weights[(i * len(BATCHES) + j) % copies]
                sp.mul_mat(fid, w, xs[B], Nr, K, ys[B], y_dtype=sp.BF16, static_weights=True)

        msk = timed(max(graph_steps, args.steps // 4), 3, sweep_local, cache_k)
        alg = sum(rb * Nr + B * K * 2 + B * Nr * 2 for B in BATCHES)
        achieved = alg / len(BATCHES) / (msk / max(graph_steps, args.steps // 4) * 1e-3 / len(BATCHES)) / 1e9
    traffic = profile_traffic(f"gemv_{args.fmt}_K{K}_N{Nr}_sweep")
    roofline = {"bound": "hbm", "achieved": achieved, "peak": hbm_peak, "unit": "GB/s",
                "frac": achieved / hbm_peak, "traffic": traffic, "peak_kind": peak_kind,
                "kernel": f"gemv_kernel<{args.fmt}>"}

    # e2e through the public C-ABI with host buffers (pinned), copies in the
    # timed region every step
    hx = {B: torch.from_numpy(F.gen_activations(B, K, seed=200 + B).view(np.int16)).pin_memory() for B in BATCHES}
    hy = {B: torch.empty((B, N), dtype=torch.int16).pin_memory() for B in BATCHES}
    xd = {B: torch.empty((B, K), dtype=torch.bfloat16, device=dev) for B in BATCHES}

    def sweep_e2e(i):
        for j, B in enumerate(BATCHES):
            w = weights[(i * len(BATCHES) + j) % copies]
            xd[B].view(torch.int16).copy_(hx[B], non_blocking=True)
            hy[B].copy_(mul_mat_full(w, xd[B], B).view(torch.int16), non_blocking=True)

    e2e_steps = max(graph_steps, args.steps // 4)
    ms_e2e = timed(e2e_steps, 3, sweep_e2e, {})
    e2e_value = wbytes_step / (ms_e2e / e2e_steps * 1e-3) / 1e9
    h2d = sum(B * K * 2 for B in BATCHES)
    d2h = sum(B * N * 2 for B in BATCHES)

    nccl = None
    if world > 1:
        msn = timed(e2e_steps, 3, sweep_nccl, {})
        nccl = {"value": wbytes_step / (msn / e2e_steps * 1e-3) / 1e9, "unit": "GB/s",
                "ms_per_step": msn / e2e_steps,
                "note": "same step with spiral_mul_mat + torch.distributed all_gather_into_tensor (NCCL)"}

    extras = {}
    if world == 1 and not args.no_extras:
        extras = bench_extras(sp, F, dev, K, N, timed, graph_steps, hbm_peak)

    cpu = None
    if rank == 0 and world == 1:
        from oracle import formats as Fo

        hx_np = {B: Fo.gen_activations(B, K, seed=100 + B) for B in BATCHES}
        rate, reps, rows = cpu_sweep_rate(fid, raw, K, N, hx_np, budget_s=args.cpu_seconds)
        cpu = {"value": rate, "unit": "GB/s", "cores": os.cpu_count() or 1, "kind": "port",
               "sample": f"{reps} full sweeps (B=1,2,4,8) over {rows}x{K} {args.fmt} in "
                         f"~{args.cpu_seconds:.0f} s, oracle/oracle.c OpenMP"}

    status = sp.device_status()
    if status != 0:
        raise SystemExit(f"rank {rank}: device status {status} after the timed runs")

    if rank == 0:
        line = {
            "metric": f"dequant-GEMV weight GB/s ({args.fmt.upper()} {N}x{K}, B=1,2,4,8)",
            "value": value,
            "unit": "GB/s",
            "n_gpus": world,
            "steps": args.steps,
            "warmup": max(3, args.warmup),
            "ms_per_step": ms_per_step,
            "higher_is_better": True,
            "scaling": "strong",
            "vs_baseline": None,
            "dtype": "bf16",
            "data": "synthetic (seeded BASELINE distributions; Q4_0 d=|N(0,1)|*0.02, x~N(0,1))",
            "config": {"workload": f"cfg2 {args.fmt} dequant-GEMV {N}x{K} B=1,2,4,8 (4 MUL_MAT per step)",
                       "weight_copies": copies,
                       "l2": f"inputs larger than L2: {copies} rotating weight copies "
                             f"({copies * shard_bytes / 2**20:.0f} MiB per rank > 126 MB L2)",
                       "parallelism": "single GPU" if world == 1 else
                       f"row-shard x{world}, all-gather fused into the GEMV (flagged NVLink stores)",
                       "graphs": f"CUDA graphs of {graph_steps} steps"},
            "roofline": roofline,
            "e2e": {"value": e2e_value, "unit": "GB/s", "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                    "note": "public C-ABI, pinned host x in / y out every step, weights resident"},
            "gpu_launches": args.steps * len(BATCHES),
            "clocks": clk.summary(),
        }
        if cpu is not None:
            line["cpu_baseline"] = cpu
        if extras:
            line["extras"] = extras
        if nccl is not None:
            line["nccl_allgather_baseline"] = nccl
        print(json.dumps(line), flush=True)

    del main_cache
    if world > 1:
        del xc
        dist.barrier()
        dist.destroy_process_group()
    return 0


MOE_BYTES_PER_EXPERT = 2654208  # Q4_0 gate + up (768 x 2048) and down (2048 x 768)


def bench_moe(sp, F, dev, timed, graph_steps, hbm_peak, Ts=(1, 2, 4, 8, 16, 32, 64)):
    """Config 4: MoE FFN decode layer, 128 Q4_0 experts (hidden 2048, inter
    768, SwiGLU), top-8, T tokens.  Weight GB/s = unique active experts x
    2,654,208 B per layer / time.  8 copies of the expert weights and 8
    routings rotate, so a layer's experts were last touched >= 8 layers ago
    (>= 168 MB of other weights: not in L2)."""
    import torch

    fid, E, H, I, topk, copies, routings = F.Q4_0, 128, 2048, 768, 8, 8, 8
    g0 = torch.from_numpy(F.gen_experts(fid, E, I, H, seed=11)).to(dev)
    u0 = torch.from_numpy(F.gen_experts(fid, E, I, H, seed=12)).to(dev)
    d0 = torch.from_numpy(F.gen_experts(fid, E, H, I, seed=13)).to(dev)
    wg = [g0] + [g0.clone() for _ in range(copies - 1)]
    wu = [u0] + [u0.clone() for _ in range(copies - 1)]
    wd = [d0] + [d0.clone() for _ in range(copies - 1)]
    res = {}
    for T in Ts:
        x = torch.from_numpy(F.gen_activations(T, H, seed=T).view(np.int16)).to(dev).view(torch.bfloat16)
        rts = [F.gen_routing(T, E, topk, seed=1000 * T + r) for r in range(routings)]
        uniq = [len(set(ids.reshape(-1).tolist())) for ids, _ in rts]
        ids = [torch.from_numpy(a).to(dev) for a, _ in rts]
        wts = [torch.from_numpy(b).to(dev) for _, b in rts]
        y = torch.empty((T, H), dtype=torch.bfloat16, device=dev)
        ws = torch.empty(sp.moe_workspace_bytes(E, H, I, T, topk), dtype=torch.uint8, device=dev)

        def body(i, x=x, ids=ids, wts=wts, y=y, ws=ws):
            c, r = i % copies, (i // copies) % routings
            sp.moe_ffn(fid, wg[c], wu[c], wd[c], x, ids[r], wts[r], hidden=H, inter=I, n_experts_local=E, y=y,
                       workspace=ws)

        steps = graph_steps * 4
        ms = timed(steps, 3, body, {})
        t = ms / steps * 1e-3
        # the captured graph cycles over graph_steps calls: average U over those
        u_mean = sum(uniq[(i // copies) % routings] for i in range(graph_steps)) / graph_steps
        wbytes = u_mean * MOE_BYTES_PER_EXPERT
        res[f"T{T}"] = {"us": t * 1e6, "unique_experts": u_mean, "weight_GBps": wbytes / t / 1e9,
                        "frac_hbm": (wbytes + T * H * 4) / t / 1e9 / hbm_peak}
    del wg, wu, wd
    return res


def bench_extras(sp, F, dev, K, N, timed, graph_steps, hbm_peak):
    """Per-batch and per-format GEMV GB/s, plus standalone dequant GB/s
    (config 0/1), each with its own rotating buffers and graphs."""
    import torch

    out = {"gemv": {}, "dequant": {}, "gemm": {}}
    _, tc_peak, _ = measured_peaks()
    for name in ("q4_0", "q8_0", "q6_k"):
        fid = F.BY_NAME[name]
        for Ng in (4096, N):
            rawg = F.generate(fid, K, Ng, seed=0)
            wg = torch.from_numpy(rawg).to(dev)
            for Mg in (512, 2048):
                x = torch.from_numpy(F.gen_activations(Mg, K, seed=Mg).view(np.int16)).to(dev).view(torch.bfloat16)
                y = torch.empty((Mg, Ng), dtype=torch.bfloat16, device=dev)

                def body_g(i, wg=wg, x=x, y=y, fid=fid, Ng=Ng):
                    sp.mul_mat(fid, wg, x, Ng, K, y, y_dtype=sp.BF16)

                steps = 20
                ms = timed(steps, 3, body_g, {})
                t = ms / steps * 1e-3
                fl = 2.0 * Mg * Ng * K
                out["gemm"][f"{name}_M{Mg}_N{Ng}"] = {"us": t * 1e6, "TFLOPs": fl / t / 1e12,
                                                       "frac_bf16_peak": fl / t / 1e12 / tc_peak}
            del wg
    for name in ("q4_0", "q8_0", "q6_k"):
        fid = F.BY_NAME[name]
        rb = F.row_bytes(fid, K)
        raw = F.generate(fid, K, N, seed=0)
        copies = max(2, math.ceil(2 * L2_BYTES / (rb * N)))
        w0 = torch.from_numpy(raw).to(dev)
        ws = [w0] + [w0.clone() for _ in range(copies - 1)]
        for B in BATCHES:
            x = torch.from_numpy(F.gen_activations(B, K, seed=B).view(np.int16)).to(dev).view(torch.bfloat16)
            y = torch.empty((B, N), dtype=torch.bfloat16, device=dev)

            def body(i, ws=ws, x=x, y=y, fid=fid, copies=copies):
                sp.mul_mat(fid, ws[i % copies], x, N, K, y, y_dtype=sp.BF16, static_weights=True)

            steps = graph_steps * 20
            ms = timed(steps, 3, body, {})
            t = ms / steps * 1e-3
            out["gemv"][f"{name}_B{B}"] = {
                "us": t * 1e6, "weight_GBps": rb * N / t / 1e9,
                "frac_hbm": (rb * N + B * K * 2 + B * N * 2) / t / 1e9 / hbm_peak}
        del ws
        # standalone dequant: config 0 (Q4_0 4096^2) and config 1 (Q8_0/Q6_K 14336x4096)
        Nd = 4096 if name == "q4_0" else N
        rawd = raw[: Nd * rb]
        in_b, out_b = Nd * rb, Nd * K * 2
        copies = max(2, math.ceil(2 * L2_BYTES / (in_b + out_b)))
        srcs = [torch.from_numpy(rawd).to(dev) for _ in range(copies)]
        dsts = [torch.empty((Nd, K), dtype=torch.bfloat16, device=dev) for _ in range(copies)]

        def body_d(i, srcs=srcs, dsts=dsts, fid=fid, Nd=Nd, copies=copies):
            sp.dequant_bf16(fid, srcs[i % copies], K, Nd, dsts[i % copies])

        steps = graph_steps * 10
        ms = timed(steps, 3, body_d, {})
        t = ms / steps * 1e-3
        out["dequant"][f"{name}_{Nd}x{K}"] = {"us": t * 1e6, "GBps": (in_b + out_b) / t / 1e9,
                                              "frac_hbm": (in_b + out_b) / t / 1e9 / hbm_peak}
        del srcs, dsts
    out["moe"] = bench_moe(sp, F, dev, timed, graph_steps, hbm_peak)
    return out


def main(argv=None):
    args = parse_args(argv)
    if args.profile:
        return run_profile(args)
    if args.impl == "reference":
        return run_reference(args)
    return run_spiral(args)


if __name__ == "__main__":
    sys.exit(main())
