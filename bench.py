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
* Steps are replayed as CUDA graphs of the C-ABI calls, every graph captured
  before the timed region; device time with CUDA events, max over ranks.
* N > 1 (torchrun): the weight is row-sharded by output feature and the
  all-gather is fused into the GEMV (spiral_mul_mat_allgather), so every rank
  ends each MUL_MAT with the full y.  Total work is fixed: strong scaling.
  Before timing, every rank checks its gathered outputs bitwise against
  spiral_mul_mat on the whole weight (same kernel, same per-row summation
  order) and exits non-zero on a mismatch.
* e2e: the same sweep through the public C-ABI with host buffers: every step
  copies that step's activations from pinned host memory and reads every
  output back to pinned host memory inside the timed region, as a serving
  loop does (double-buffered: the next step's upload and the previous step's
  read-back run on two copy streams while this step's MUL_MATs run).
  Weights stay resident (uploaded once, as at model load).
* extras: every other BASELINE config with its own roofline object — the
  standalone dequant (configs 0/1, row-sharded at N > 1), the prefill GEMM
  (config 3, row-sharded plus an NCCL all-gather at N > 1), the MoE layer
  (config 4, expert-parallel at N > 1) and, at N = 1, every format and batch
  of the GEMV.
* cpu_baseline / --impl reference: the C restatement of the reference's
  dequant-then-fp32-matmul (oracle/oracle.c, OpenMP on every host core),
  timed on a bounded sample of the same workload; at N = 1 the extras add the
  CPU figures of every config and of the reference's own C++ repack.
"""

from __future__ import annotations

import argparse
import json
import math
import os
import platform
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
E2E_GRAPH_STEPS = 128  # steps per CUDA graph of the end-to-end (host copies) loop
MOE_E, MOE_H, MOE_I, MOE_TOPK = 128, 2048, 768, 8
MOE_BYTES_PER_EXPERT = 2654208  # Q4_0 gate + up (768 x 2048) and down (2048 x 768)
MOE_TOKENS = (1, 2, 4, 8, 16, 32, 64)


def parse_args(argv=None):
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=2000)
    ap.add_argument("--warmup", type=int, default=50)
    ap.add_argument("--impl", choices=("spiral", "reference"), default="spiral")
    ap.add_argument("--fmt", default="q4_0", choices=("q4_0", "q8_0", "q6_k"))
    ap.add_argument("--no-extras", action="store_true", help="skip the per-config extras")
    ap.add_argument("--cpu-seconds", type=float, default=8.0, help="CPU baseline sample budget (headline)")
    ap.add_argument("--profile", choices=("gemv", "dequant", "gemm", "moe"), default=None,
                    help="ncu helper: run --warmup + --steps eager launches of one kernel on one GPU "
                         "(B from --batch), nothing else")
    ap.add_argument("--batch", type=int, default=1, help="activation vectors for --profile gemv / gemm, tokens for moe")
    ap.add_argument("--features", type=int, default=N_DIM, help="output features for --profile gemv / gemm")
    ap.add_argument("--k", type=int, default=K_DIM, help="reduction dimension for --profile gemv / gemm / dequant")
    return ap.parse_args(argv)


def headline_config(fmt: str, world: int) -> dict:
    """The `config` both arms print (the driver compares them)."""
    return {"workload": f"cfg2 {fmt} dequant-GEMV {N_DIM}x{K_DIM} B=1,2,4,8 (4 MUL_MAT per step)",
            "parallelism": "single GPU" if world == 1 else f"row-shard x{world}, all-gather fused into the GEMV",
            "l2": "inputs larger than L2 (rotating weight copies)"}


def headline_metric(fmt: str) -> str:
    return f"dequant-GEMV weight GB/s ({fmt.upper()} {N_DIM}x{K_DIM}, B=1,2,4,8)"


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
    """Per-launch DRAM bytes of a kernel from the committed ncu summary
    (profiles/dram_traffic.txt: `<key> <bytes_per_launch>`)."""
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


def host_info() -> dict:
    model = platform.processor() or ""
    try:
        for line in Path("/proc/cpuinfo").read_text().splitlines():
            if line.startswith("model name"):
                model = line.split(":", 1)[1].strip()
                break
    except OSError:
        pass
    return {"nproc": os.cpu_count() or 1, "cpu_model": model}


def roofline(bound: str, alg_units: float, seconds: float, peak: float, peak_kind: str, kernel: str,
             traffic=None) -> dict:
    """alg_units: algorithmic bytes (bound hbm) or flops (bound tensor) of
    one launch; seconds: that launch's average duration."""
    if bound == "hbm":
        achieved, unit = alg_units / seconds / 1e9, "GB/s"
    else:
        achieved, unit = alg_units / seconds / 1e12, "TFLOP/s"
    return {"bound": bound, "achieved": achieved, "peak": peak, "unit": unit, "frac": achieved / peak,
            "traffic": traffic, "peak_kind": peak_kind, "kernel": kernel, "alg_per_launch": alg_units,
            "launch_us": seconds * 1e6}


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


# --------------------------------------------------------------- CPU arms


def cpu_threads() -> int:
    """Give the C oracle every host core (torchrun sets OMP_NUM_THREADS=1)
    and return the thread count OpenMP will really use."""
    import oracle

    return oracle.threads(os.cpu_count() or 1)


def cpu_sweep_rate(fid: int, raw: np.ndarray, K: int, N: int, xs: dict, budget_s: float, rows: int | None = None):
    """Time the oracle's dequant-then-fp32-matmul sweep (B = 1, 2, 4, 8) on
    the first `rows` output features; returns (weight GB/s, reps, rows)."""
    import oracle
    from oracle import formats as F

    rows = N if rows is None else max(16, min(N, rows))
    sub = raw[: rows * F.row_bytes(fid, K)]
    wbytes = rows * F.row_bytes(fid, K)
    th = cpu_threads()
    oracle.mul_mat_f32(fid, sub, xs[1], K, min(rows, 64), threads=th)  # warm the pool
    reps, t0 = 0, time.perf_counter()
    while True:
        for B in BATCHES:
            oracle.mul_mat_f32(fid, sub, xs[B], K, rows, threads=th)
        reps += 1
        el = time.perf_counter() - t0
        if el >= budget_s:
            break
    return reps * len(BATCHES) * wbytes / el / 1e9, reps, rows


def _time_loop(fn, budget_s: float, min_reps: int = 1):
    fn()  # warm
    reps, t0 = 0, time.perf_counter()
    while True:
        fn()
        reps += 1
        el = time.perf_counter() - t0
        if reps >= min_reps and el >= budget_s:
            return el / reps, reps


def cpu_extras(budget_s: float) -> dict:
    """CPU figures of every config on the box's host cores (rank 0, N = 1):
    the C restatement (OpenMP, all cores) per config, the NumPy restatement
    of the reference's dequant, a NumPy fp32 matmul on the dequantized
    weights, and the reference's own C++ repack (oracle/_ref, one thread)."""
    import ctypes

    import oracle
    from oracle import formats as F

    th = cpu_threads()
    K = K_DIM
    out = {"host": host_info(), "omp_threads": th}
    # (iv) C restatement, dequant (configs 0 / 1): a row sample
    dq = {}
    for name, Nd in (("q4_0", 4096), ("q8_0", N_DIM), ("q6_k", N_DIM)):
        fid = F.BY_NAME[name]
        rows = 2048
        raw = F.generate(fid, K, rows, seed=0)
        sec, reps = _time_loop(lambda: oracle.dequant_bf16(fid, raw, K, rows, threads=th), budget_s)
        b = rows * (F.row_bytes(fid, K) + 2 * K)
        dq[f"{name}_{Nd}x{K}"] = {"value": b / sec / 1e9, "unit": "GB/s", "cores": th, "kind": "port",
                                  "sample": f"{rows} of {Nd} rows x {reps} reps, oracle/oracle.c OpenMP"}
    out["dequant"] = dq
    # (iv) C restatement, GEMM (config 3): dequant-then-fp32-matmul on a row sample
    gm = {}
    for name in ("q4_0", "q6_k"):
        fid = F.BY_NAME[name]
        rows = 64
        raw = F.generate(fid, K, rows, seed=0)
        for M in (512, 2048):
            x = F.gen_activations(M, K, seed=M)
            sec, reps = _time_loop(lambda: oracle.mul_mat_f32(fid, raw, x, K, rows, threads=th), budget_s / 2)
            gm[f"{name}_M{M}"] = {"value": 2.0 * M * rows * K / sec / 1e12, "unit": "TFLOP/s", "cores": th,
                                  "kind": "port", "sample": f"{rows} output features x {reps} reps "
                                                            f"(rate is per-feature, shape-independent)"}
    out["gemm"] = gm
    # (iv) MoE (config 4): float64 oracle layer at T = 1 and 8 (NumPy + C dequant)
    moe = {}
    fid = F.Q4_0
    E = 16  # experts are independent: time a 16-expert slice, routing within it
    wg = F.gen_experts(fid, E, MOE_I, MOE_H, seed=11)
    wu = F.gen_experts(fid, E, MOE_I, MOE_H, seed=12)
    wd = F.gen_experts(fid, E, MOE_H, MOE_I, seed=13)
    for T in (1, 8):
        x = F.gen_activations(T, MOE_H, seed=T)
        ids, wts = F.gen_routing(T, E, MOE_TOPK, seed=T)
        u = len(set(ids.reshape(-1).tolist()))
        sec, reps = _time_loop(lambda: oracle.moe_ffn_f64(fid, wg, wu, wd, x, ids, wts, MOE_H, MOE_I, E),
                               budget_s / 2)
        moe[f"T{T}"] = {"value": u * MOE_BYTES_PER_EXPERT / sec / 1e9, "unit": "GB/s (expert weights)",
                        "us_per_layer": sec * 1e6, "unique_experts": u, "cores": th, "kind": "port",
                        "sample": f"{E}-expert slice, top-{MOE_TOPK}, {reps} reps, oracle.moe_ffn_f64"}
    out["moe"] = moe
    # (i) NumPy restatement of the reference's dequant (the reference's own
    # per-block Python loop needs the reference tree, which does not travel)
    fid = F.Q4_0
    rows = 512
    raw = F.generate(fid, K, rows, seed=0)
    sec, reps = _time_loop(lambda: F.dequant_bf16(fid, raw, K, rows), budget_s / 2)
    out["numpy_dequant_q4_0"] = {"value": rows * (F.row_bytes(fid, K) + 2 * K) / sec / 1e9, "unit": "GB/s",
                                 "cores": 1, "kind": "port",
                                 "sample": f"{rows}x{K} Q4_0, {reps} reps, oracle.formats (vectorised NumPy "
                                           f"restatement of formats/q4_0.py)"}
    # (ii) NumPy fp32 matmul of the dequantized weights (BLAS, all cores)
    rows = 4096
    raw = F.generate(fid, K, rows, seed=0)
    w32 = F.bf16_bits_to_f32(oracle.dequant_bf16(fid, raw, K, rows, threads=th))
    for B in (8, 512):
        x32 = F.bf16_bits_to_f32(F.gen_activations(B, K, seed=B))
        sec, reps = _time_loop(lambda: x32 @ w32.T, budget_s / 2)
        out[f"numpy_matmul_f32_B{B}"] = {"value": 2.0 * B * rows * K / sec / 1e12, "unit": "TFLOP/s",
                                         "cores": os.cpu_count() or 1, "kind": "port",
                                         "sample": f"x[{B}x{K}] @ W^T[{K}x{rows}] fp32, {reps} reps"}
    # (iii) the reference's own C++ repack_weights (oracle/_ref, built from
    # src/quants/tests/repack.cc), one thread
    rep = {}
    for name in ("q4_0", "q8_0", "q6_k"):
        so = REPO / "oracle" / "_ref" / f"quants_host_{name}.so"
        if not so.exists():
            rep[name] = {"unavailable": "oracle/_ref not built (needs the reference tree at build time)"}
            continue
        L = ctypes.CDLL(str(so))
        L.quants_packed_bytes.argtypes = [ctypes.c_int64, ctypes.c_int64]
        L.quants_packed_bytes.restype = ctypes.c_int64
        L.quants_repack.argtypes = [ctypes.c_void_p, ctypes.c_int64, ctypes.c_void_p, ctypes.c_int64,
                                    ctypes.c_int64, ctypes.c_int64]
        L.quants_repack.restype = ctypes.c_int64
        fid = F.BY_NAME[name]
        rows = 2048
        raw = F.generate(fid, K, rows, seed=0)
        cap = int(L.quants_packed_bytes(K, rows))
        dst = np.empty(max(cap, 1), dtype=np.uint8)
        rb = F.row_bytes(fid, K)
        sec, reps = _time_loop(lambda: L.quants_repack(raw.ctypes.data, rb, dst.ctypes.data, cap, K, rows),
                               budget_s / 3)
        rep[name] = {"value": rows * rb / sec / 1e9, "unit": "GB/s (canonical bytes in)", "cores": 1,
                     "kind": "reference", "sample": f"{rows}x{K}, {reps} reps, quants_repack from "
                                                    f"src/quants/tests/repack.cc (adjacent step, not the path)"}
    out["reference_repack"] = rep
    return out


def run_reference(args):
    rank, world, _ = dist_env()
    if rank != 0:
        return 0
    import oracle
    from oracle import formats as F

    fid = F.BY_NAME[args.fmt]
    K, N = K_DIM, N_DIM
    raw = F.generate(fid, K, N, seed=0)
    xs = {B: F.gen_activations(B, K, seed=100 + B) for B in BATCHES}
    cores = cpu_threads()
    # one full step to size the bounded per-step sample
    t0 = time.perf_counter()
    for B in BATCHES:
        oracle.mul_mat_f32(fid, raw, xs[B], K, N, threads=cores)
    full = time.perf_counter() - t0
    total_budget = 120.0
    per_step = total_budget / max(1, args.steps + args.warmup)
    rows = N if full <= per_step else max(16, int(N * per_step / full) // 16 * 16)
    sub = raw[: rows * F.row_bytes(fid, K)]
    for _ in range(args.warmup):
        for B in BATCHES:
            oracle.mul_mat_f32(fid, sub, xs[B], K, rows, threads=cores)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        for B in BATCHES:
            oracle.mul_mat_f32(fid, sub, xs[B], K, rows, threads=cores)
    el = time.perf_counter() - t0
    wbytes = rows * F.row_bytes(fid, K) * len(BATCHES)
    value = wbytes * args.steps / el / 1e9
    sample = (f"{rows} of {N} rows per step (B=1,2,4,8 sweep, K={K}), {args.steps} steps; "
              f"oracle/oracle.c dequant-then-fp32-matmul, OpenMP")
    line = {
        "impl": "reference",
        "metric": headline_metric(args.fmt),
        "value": value,
        "unit": "GB/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": el / args.steps * 1e3,
        "ms_per_full_step": el / args.steps * 1e3 * (N / rows),
        "higher_is_better": True,
        "scaling": "strong",
        "vs_baseline": None,
        "dtype": "f32",
        "data": "synthetic (seeded BASELINE distributions; Q4_0 d=|N(0,1)|*0.02, x~N(0,1))",
        "config": headline_config(args.fmt, world),
        "cpu_baseline": {"value": value, "unit": "GB/s", "cores": cores, "kind": "port", "sample": sample,
                         "host": host_info()},
        "e2e": {"value": value, "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "gpu_launches": 0,
    }
    print(json.dumps(line), flush=True)
    return 0


# ------------------------------------------------------------------ GPU


class Timer:
    """CUDA-graph replays of `body(i)` steps, timed with CUDA events on the
    capture stream; every graph a timed run replays is captured before its
    start event, so the timed region holds replays only."""

    def __init__(self, dev, world, graph_steps, stream):
        self.dev, self.world, self.graph_steps, self.stream = dev, world, graph_steps, stream

    def _capture(self, nsteps, body, finish=None):
        import torch

        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=self.stream):
            for j in range(nsteps):
                body(j)
            if finish is not None:
                finish(nsteps)  # join side streams back into the capture stream
        return g

    def prepare(self, nsteps, cache, body, gsteps, finish=None):
        full, tail = divmod(nsteps, gsteps)
        if full and "main" not in cache:
            cache["main"] = self._capture(gsteps, body, finish)
        if tail and ("tail", tail) not in cache:
            cache[("tail", tail)] = self._capture(tail, body, finish)

    def replay(self, nsteps, cache, gsteps):
        full, tail = divmod(nsteps, gsteps)
        for _ in range(full):
            cache["main"].replay()
        if tail:
            cache[("tail", tail)].replay()

    def timed(self, nsteps, warm, body, gsteps=None, finish=None):
        """Device ms of `nsteps` steps (max over ranks).  A graph holds
        `gsteps` steps (default: the headline's); make it a whole number of
        the body's buffer-rotation cycles.  `finish(n)` runs at the end of
        each capture (to join streams the body forked)."""
        import torch
        import torch.distributed as dist

        gsteps = gsteps or self.graph_steps
        cache = {}
        self.prepare(warm, cache, body, gsteps, finish)
        self.prepare(nsteps, cache, body, gsteps, finish)
        if self.world > 1:
            # fused exchanges wait on the device for at most 2 s: ranks start
            # the warm-up together
            torch.cuda.synchronize()
            dist.barrier()
        with torch.cuda.stream(self.stream):
            self.replay(warm, cache, gsteps)
        torch.cuda.synchronize()
        if self.world > 1:
            dist.barrier()
        torch.cuda.synchronize()
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with torch.cuda.stream(self.stream):
            s.record(self.stream)
            self.replay(nsteps, cache, gsteps)
            e.record(self.stream)
        torch.cuda.synchronize()
        ms = s.elapsed_time(e)
        if self.world > 1:
            t = torch.tensor([ms], device=self.dev)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            ms = float(t.item())
        return ms


def run_profile(args):
    """A few plain launches of one kernel for ncu (fresh weight copies per
    launch so every launch reads HBM; dequant outputs rotate too)."""
    import torch

    import spiral_b200 as sp
    from oracle import formats as F

    torch.cuda.set_device(0)
    fid = F.BY_NAME[args.fmt]
    K = args.k
    n = args.warmup + args.steps
    if args.profile == "moe":
        E, H, I, T = MOE_E, MOE_H, MOE_I, args.batch
        wg = torch.from_numpy(F.gen_experts(fid, E, I, H, seed=11)).cuda()
        wu = torch.from_numpy(F.gen_experts(fid, E, I, H, seed=12)).cuda()
        wd = torch.from_numpy(F.gen_experts(fid, E, H, I, seed=13)).cuda()
        x = torch.from_numpy(F.gen_activations(T, H, seed=T).view(np.int16)).cuda().view(torch.bfloat16)
        ids, wts = F.gen_routing(T, E, MOE_TOPK, seed=T)
        ids, wts = torch.from_numpy(ids).cuda(), torch.from_numpy(wts).cuda()
        for _ in range(n):
            sp.moe_ffn(fid, wg, wu, wd, x, ids, wts, hidden=H, inter=I, n_experts_local=E)
    else:
        N = args.features if args.profile in ("gemv", "gemm") else (N_DIM if args.fmt != "q4_0" else 4096)
        raw = F.generate(fid, K, N, seed=0)
        ws = [torch.from_numpy(raw).cuda() for _ in range(min(n, 8))]
        if args.profile in ("gemv", "gemm"):
            x = torch.from_numpy(F.gen_activations(args.batch, K, seed=1).view(np.int16)).cuda().view(torch.bfloat16)
            y = torch.empty((args.batch, N), dtype=torch.bfloat16, device="cuda")
            for i in range(n):
                sp.mul_mat(fid, ws[i % len(ws)], x, N, K, y, y_dtype=sp.BF16, static_weights=True)
        else:
            outs = [torch.empty((N, K), dtype=torch.bfloat16, device="cuda") for _ in range(min(n, 4))]
            for i in range(n):
                sp.dequant_bf16(fid, ws[i % len(ws)], K, N, outs[i % len(outs)])
    torch.cuda.synchronize()
    print(json.dumps({"profile": args.profile, "fmt": args.fmt, "launches": n, "device_status": sp.device_status()}))
    return 0


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
    from spiral_b200.dist import AllGatherExchange, row_range

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

    stream = torch.cuda.Stream(device=dev)
    if world > 1:  # fused exchanges wait on the device for at most 2 s
        dist.barrier()
    # warm-up (also configures kernel attributes before any capture)
    with torch.cuda.stream(stream):
        for i in range(3):
            sweep(i)
    torch.cuda.synchronize()
    if sp.device_status() != 0:
        raise SystemExit(f"rank {rank}: a device-side wait gave up during warm-up")

    parity = {"check": "none"}
    if world > 1:
        # bitwise: the gathered output equals spiral_mul_mat over the whole
        # weight on this rank (same kernel and per-row summation order)
        wfull = torch.from_numpy(raw).to(dev)
        bad = 0
        with torch.cuda.stream(stream):
            for B in BATCHES:
                got = mul_mat_full(weights[0], xs[B], B).clone()
                want = sp.mul_mat(fid, wfull, xs[B], N, K, y_dtype=sp.BF16)
                bad += int((got.view(torch.int16) != want.view(torch.int16)).sum().item())
        torch.cuda.synchronize()
        del wfull
        t = torch.tensor([bad], device=dev)
        dist.all_reduce(t)
        bad = int(t.item())
        parity = {"check": "bitwise vs spiral_mul_mat on the whole weight, every rank, B=1,2,4,8",
                  "mismatches": bad, "status": "ok" if bad == 0 else "FAIL"}
        if bad:
            raise SystemExit(f"rank {rank}: gathered GEMV differs from the single-GPU result in {bad} outputs")
        if sp.device_status() != 0:
            raise SystemExit(f"rank {rank}: a device-side wait gave up during the parity check")

    # whole weight-rotation cycles, at least 32 steps (128 launches) per graph:
    # a graph boundary costs the next launch its overlap with the previous one
    graph_steps = copies * max(1, math.ceil(32 / copies)) if copies <= 64 else 64
    timer = Timer(dev, world, graph_steps, stream)
    warm = max(3, args.warmup)
    with ClockSampler(local) as clk:
        ms = timer.timed(args.steps, warm, sweep)
    ms_per_step = ms / args.steps
    wbytes_step = N * rb * len(BATCHES)  # whole job: every rank streams its shard
    value = wbytes_step / (ms_per_step * 1e-3) / 1e9

    # roofline of the dominant kernel: algorithmic bytes (weights + x + y) per
    # launch over the per-launch time.  At N=1 the timed region holds only
    # GEMV launches, so the per-launch time is the timed region / launches
    # (an upper bound: graph gaps between kernels count against the kernel).
    hbm_peak, tc_peak, peak_kind = measured_peaks()
    alg = sum(rb * Nr + B * K * 2 + B * Nr * 2 for B in BATCHES) / len(BATCHES)
    if world == 1:
        launch_s = ms_per_step * 1e-3 / len(BATCHES)
    else:
        # kernel-only time on this rank: the same sweep on the shard without the gather

        def sweep_local(i):
            for j, B in enumerate(BATCHES):
                w = weights[(i * len(BATCHES) + j) % copies]
                sp.mul_mat(fid, w, xs[B], Nr, K, ys[B], y_dtype=sp.BF16, static_weights=True)

        nk = max(graph_steps, args.steps // 4)
        launch_s = timer.timed(nk, 3, sweep_local) / nk * 1e-3 / len(BATCHES)
    head_roof = roofline("hbm", alg, launch_s, hbm_peak, peak_kind, f"gemv_xs_kernel<{args.fmt}>",
                         profile_traffic(f"gemv_{args.fmt}_K{K}_N{Nr}_sweep"))

    # e2e through the public C-ABI with host buffers (pinned), copies in the
    # timed region every step: the step's activations (B = 1, 2, 4, 8 stacked
    # in one pinned buffer) go up in one copy, the four MUL_MATs write their
    # outputs into one device buffer, which comes back in one copy.  Serving
    # pipeline: device and host buffers alternate between steps, uploads run
    # on one copy stream and read-backs on another, so step i + 1's upload and
    # step i - 1's read-back overlap step i's MUL_MATs; event waits keep each
    # buffer's upload, MUL_MATs and read-back in order.
    offs = np.cumsum([0] + list(BATCHES))
    rows = int(offs[-1])
    hx_all = torch.from_numpy(np.concatenate([F.gen_activations(B, K, seed=200 + B) for B in BATCHES]).view(np.int16))
    hx_all = hx_all.pin_memory()
    hy_all = [torch.empty((rows, N), dtype=torch.int16).pin_memory() for _ in range(2)]
    xd_all = [torch.empty((rows, K), dtype=torch.bfloat16, device=dev) for _ in range(2)]
    yd_all = [torch.empty((rows, N), dtype=torch.bfloat16, device=dev) for _ in range(2)]
    s_up, s_down = torch.cuda.Stream(device=dev), torch.cuda.Stream(device=dev)
    ev_in = [torch.cuda.Event() for _ in range(2)]
    ev_comp = [torch.cuda.Event() for _ in range(2)]
    ev_out = [torch.cuda.Event() for _ in range(2)]

    def sweep_e2e(i):
        b = i % 2
        cap = torch.cuda.current_stream()
        # upload: buffer b is free once step i - 2's MUL_MATs are done
        s_up.wait_stream(cap) if i < 2 else s_up.wait_event(ev_comp[b])
        with torch.cuda.stream(s_up):
            xd_all[b].view(torch.int16).copy_(hx_all, non_blocking=True)
            ev_in[b].record(s_up)
        cap.wait_event(ev_in[b])
        if i >= 2:
            cap.wait_event(ev_out[b])  # step i - 2's read-back of yd[b] is done
        for j, B in enumerate(BATCHES):
            w = weights[(i * len(BATCHES) + j) % copies]
            xb, yb = xd_all[b][offs[j] : offs[j] + B], yd_all[b][offs[j] : offs[j] + B]
            if world > 1:
                sp.mul_mat_allgather(fid, w, xb, Nr, K, yb, n0, xc.peers, rank, world)
            else:
                sp.mul_mat(fid, w, xb, Nr, K, yb, y_dtype=sp.BF16, static_weights=True)
        ev_comp[b].record(cap)
        s_down.wait_event(ev_comp[b])
        with torch.cuda.stream(s_down):
            hy_all[b].copy_(yd_all[b].view(torch.int16), non_blocking=True)
            ev_out[b].record(s_down)

    def join_e2e(n):
        cap = torch.cuda.current_stream()
        for b in range(min(n, 2)):
            cap.wait_event(ev_out[b])
        cap.wait_stream(s_up)

    e2e_steps = max(graph_steps, args.steps // 4)
    # A serving loop keeps its graphs long: each graph boundary drains both
    # copy streams and restarts the launch overlap, about 35 us on a B200
    # (e2e 2271 GB/s with graphs of 8 steps, 2417 with 32, 2441 with 64).
    e2e_gsteps = max(graph_steps, E2E_GRAPH_STEPS)
    e2e_timed = max(e2e_steps, e2e_gsteps)
    ms_e2e = timer.timed(e2e_timed, 3, sweep_e2e, gsteps=e2e_gsteps, finish=join_e2e)
    e2e_value = wbytes_step / (ms_e2e / e2e_timed * 1e-3) / 1e9
    h2d = sum(B * K * 2 for B in BATCHES)
    d2h = sum(B * N * 2 for B in BATCHES)

    nccl = None
    if world > 1:
        from spiral_b200.dist import gather_rows

        def sweep_nccl(i):  # the same step with a separate NCCL all-gather (comparison only)
            for j, B in enumerate(BATCHES):
                w = weights[(i * len(BATCHES) + j) % copies]
                sp.mul_mat(fid, w, xs[B], Nr, K, ys[B], y_dtype=sp.BF16, static_weights=True)
                gather_rows(ys[B], N)

        msn = timer.timed(e2e_steps, 3, sweep_nccl)
        nccl = {"value": wbytes_step / (msn / e2e_steps * 1e-3) / 1e9, "unit": "GB/s",
                "ms_per_step": msn / e2e_steps,
                "note": "same step with spiral_mul_mat + torch.distributed all_gather_into_tensor (NCCL)"}
    del weights

    extras = {}
    if not args.no_extras:
        extras = bench_extras(sp, F, dev, rank, world, timer, graph_steps, hbm_peak, tc_peak, peak_kind)

    cpu = None
    if rank == 0 and world == 1:
        hx_np = {B: F.gen_activations(B, K, seed=100 + B) for B in BATCHES}
        rate, reps, rows = cpu_sweep_rate(fid, raw, K, N, hx_np, budget_s=args.cpu_seconds)
        cpu = {"value": rate, "unit": "GB/s", "cores": cpu_threads(), "kind": "port", "host": host_info(),
               "sample": f"{reps} full sweeps (B=1,2,4,8) over {rows}x{K} {args.fmt} in "
                         f"~{args.cpu_seconds:.0f} s, oracle/oracle.c dequant-then-fp32-matmul, OpenMP"}
        if not args.no_extras:
            extras["cpu"] = cpu_extras(budget_s=max(0.5, args.cpu_seconds / 8))

    status = sp.device_status()
    if status != 0:
        raise SystemExit(f"rank {rank}: device status {status} after the timed runs")

    if rank == 0:
        cfg = headline_config(args.fmt, world)
        line = {
            "metric": headline_metric(args.fmt),
            "value": value,
            "unit": "GB/s",
            "n_gpus": world,
            "steps": args.steps,
            "warmup": warm,
            "ms_per_step": ms_per_step,
            "higher_is_better": True,
            "scaling": "strong",
            "vs_baseline": None,
            "dtype": "bf16",
            "data": "synthetic (seeded BASELINE distributions; Q4_0 d=|N(0,1)|*0.02, x~N(0,1))",
            "config": cfg,
            "setup": {"weight_copies": copies,
                      "l2": f"{copies} rotating weight copies ({copies * shard_bytes / 2**20:.0f} MiB per rank "
                            f"> 126 MB L2)",
                      "graphs": f"CUDA graphs of {graph_steps} steps, captured before the timed region"},
            "parity": parity,
            "per_launch_us": {
                "step": ms_per_step * 1e3 / len(BATCHES),
                "kernel": launch_s * 1e6,
                "gather": max(0.0, ms_per_step * 1e3 / len(BATCHES) - launch_s * 1e6) if world > 1 else 0.0,
                "note": ("one MUL_MAT: the timed step per launch; at N > 1 the same sweep on the shard without the "
                         "all-gather (kernel) and the difference (the fused gather's share)"),
            },
            "roofline": head_roof,
            "e2e": {"value": e2e_value, "unit": "GB/s", "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                    "steps": e2e_timed, "graph_steps": e2e_gsteps,
                    "note": "public C-ABI; every step one pinned-host copy of the step's activations in and one of its outputs out "
                            "(double-buffered: uploads and read-backs on two copy streams overlap the neighbouring steps' "
                            "MUL_MATs); weights resident"},
            "gpu_launches": args.steps * len(BATCHES),
            "clocks": clk.summary(),
        }
        if cpu is not None:
            line["cpu_baseline"] = cpu
        if nccl is not None:
            line["nccl_allgather_baseline"] = nccl
        if extras:
            line["extras"] = extras
        print(json.dumps(line), flush=True)

    if world > 1:
        del xc
        torch.cuda.synchronize()
        dist.barrier()
        dist.destroy_process_group()
    return 0


# ----------------------------------------------------------------- extras


def bench_dequant(sp, F, dev, rank, world, timer, graph_steps, hbm_peak, peak_kind):
    """Configs 0 and 1: standalone dequant to bf16.  At N > 1 each rank
    dequantizes its contiguous row shard (no collective); value is the whole
    job's bytes over the max-over-ranks time."""
    import torch

    from spiral_b200.dist import row_range

    K = K_DIM
    out = {}
    for name, Nt in (("q4_0", 4096), ("q8_0", N_DIM), ("q6_k", N_DIM)):
        fid = F.BY_NAME[name]
        rb = F.row_bytes(fid, K)
        r0, r1 = row_range(Nt, world, rank)
        Nd = r1 - r0
        raw = F.generate(fid, K, Nt, seed=0)[r0 * rb : r1 * rb]
        in_b, out_b = Nd * rb, Nd * K * 2
        copies = max(2, math.ceil(2 * L2_BYTES / (in_b + out_b)))
        srcs = [torch.from_numpy(raw).to(dev) for _ in range(copies)]
        dsts = [torch.empty((Nd, K), dtype=torch.bfloat16, device=dev) for _ in range(copies)]

        def body(i, srcs=srcs, dsts=dsts, fid=fid, Nd=Nd, copies=copies):
            sp.dequant_bf16(fid, srcs[i % copies], K, Nd, dsts[i % copies])

        steps = copies * max(1, 80 // copies)
        ms = timer.timed(steps, 3, body, gsteps=copies)
        t = ms / steps * 1e-3
        tot = Nt * (rb + 2 * K)
        out[f"{name}_{Nt}x{K}"] = {
            "us": t * 1e6, "GBps": tot / t / 1e9, "rows_per_rank": Nd,
            "roofline": roofline("hbm", in_b + out_b, t, hbm_peak, peak_kind, f"dequant_rows_unit<{name}>" if name == "q6_k" else f"dequant_rows_pipe<{name}>",
                                 profile_traffic(f"dequant_{name}_K{K}_N{Nd}")),
            "l2": f"{copies} rotating input/output pairs ({copies * (in_b + out_b) / 2**20:.0f} MiB > L2)"}
        del srcs, dsts
    return out


def bench_gemm(sp, F, dev, rank, world, timer, hbm_peak, tc_peak, peak_kind):
    """Config 3: prefill dequant-GEMM, Q4_0 and Q6_K, M in {512, 2048},
    N in {4096, 14336}.  At N > 1 the weight is row-sharded by output feature
    and y all-gathered over NCCL (spiral_b200.dist.gather_rows)."""
    import torch

    from spiral_b200.dist import gather_rows, row_range

    K = K_DIM
    out = {}
    for name in ("q4_0", "q8_0", "q6_k"):
        fid = F.BY_NAME[name]
        rb = F.row_bytes(fid, K)
        for Nt in (4096, N_DIM):
            if name == "q8_0" and Nt != N_DIM:
                continue
            r0, r1 = row_range(Nt, world, rank, align=128)
            Ng = r1 - r0
            wg = torch.from_numpy(F.generate(fid, K, Nt, seed=0)[r0 * rb : r1 * rb]).to(dev)
            for Mg in (512, 2048):
                x = torch.from_numpy(F.gen_activations(Mg, K, seed=Mg).view(np.int16)).to(dev).view(torch.bfloat16)
                y = torch.empty((Mg, Ng), dtype=torch.bfloat16, device=dev)

                def body(i, wg=wg, x=x, y=y, fid=fid, Ng=Ng):
                    sp.mul_mat(fid, wg, x, Ng, K, y, y_dtype=sp.BF16)

                steps = 20
                t = timer.timed(steps, 3, body) / steps * 1e-3
                fl = 2.0 * Mg * Ng * K
                ent = {"us": t * 1e6, "TFLOPs": 2.0 * Mg * Nt * K / t / 1e12, "rows_per_rank": Ng,
                       "roofline": roofline("tensor", fl, t, tc_peak, peak_kind, f"gemm_kernel<{name}>",
                                            profile_traffic(f"gemm_{name}_M{Mg}_N{Ng}"))}
                if world > 1 and Ng * world == Nt:

                    def body_g(i, wg=wg, x=x, y=y, fid=fid, Ng=Ng, Nt=Nt):
                        sp.mul_mat(fid, wg, x, Ng, K, y, y_dtype=sp.BF16)
                        gather_rows(y, Nt)

                    tg = timer.timed(steps, 3, body_g) / steps * 1e-3
                    ent["with_allgather_us"] = tg * 1e6
                    ent["TFLOPs_with_allgather"] = 2.0 * Mg * Nt * K / tg / 1e12
                out[f"{name}_M{Mg}_N{Nt}"] = ent
            del wg
    return out


def bench_moe(sp, F, dev, rank, world, timer, graph_steps, hbm_peak, peak_kind, Ts=MOE_TOKENS):
    """Config 4: MoE FFN decode layer, 128 Q4_0 experts (hidden 2048, inter
    768, SwiGLU), top-8, T tokens.  Weight GB/s = unique active experts x
    2,654,208 B per layer / time.  8 copies of the expert weights and 8
    routings rotate, so a layer's experts were last touched >= 8 layers ago
    (>= 168 MB of other weights: not in L2).  At N > 1 the experts are
    sharded (rank r owns 128/N of them), every rank holds the T tokens and
    spiral_moe_ffn_ep runs its experts and combines the ranks' partials in
    one kernel over NVLink (reduce-scatter + all-gather of fp32 units); U per
    rank is reported."""
    import torch

    from spiral_b200.dist import MoeExchange, expert_range

    fid, E, H, I, topk, routings = F.Q4_0, MOE_E, MOE_H, MOE_I, MOE_TOPK, 8
    e0, e1 = expert_range(E, world, rank)
    El = e1 - e0
    gu_b, d_b = I * F.row_bytes(fid, H), H * F.row_bytes(fid, I)
    g_all = F.gen_experts(fid, E, I, H, seed=11)
    u_all = F.gen_experts(fid, E, I, H, seed=12)
    d_all = F.gen_experts(fid, E, H, I, seed=13)
    g0 = torch.from_numpy(g_all[e0 * gu_b : e1 * gu_b]).to(dev)
    u0 = torch.from_numpy(u_all[e0 * gu_b : e1 * gu_b]).to(dev)
    d0 = torch.from_numpy(d_all[e0 * d_b : e1 * d_b]).to(dev)
    copies = max(2, min(64, math.ceil(2 * L2_BYTES / max(1, El * MOE_BYTES_PER_EXPERT // 4))))
    wg = [g0] + [g0.clone() for _ in range(copies - 1)]
    wu = [u0] + [u0.clone() for _ in range(copies - 1)]
    wd = [d0] + [d0.clone() for _ in range(copies - 1)]
    mx = MoeExchange(H, max(Ts), dev) if world > 1 else None
    res = {}
    parity = None
    if world > 1:
        # every T once: the expert-parallel layer is identical on every rank
        # and within the MoE tolerance of spiral_moe_ffn over all 128 experts
        # on this rank (a different summation order, so not bitwise)
        import torch.distributed as dist

        ga, ua, da = (torch.from_numpy(a).to(dev) for a in (g_all, u_all, d_all))
        worst, differ = 0.0, 0
        for T in Ts:
            x = torch.from_numpy(F.gen_activations(T, H, seed=T).view(np.int16)).to(dev).view(torch.bfloat16)
            ids, wts = (torch.from_numpy(a).to(dev) for a in F.gen_routing(T, E, topk, seed=1000 * T))
            dist.barrier()
            y_ep = sp.moe_ffn_ep(fid, g0, u0, d0, x, ids, wts, hidden=H, inter=I, n_experts_local=El,
                                 expert_first=e0, exchange_peers_dev=mx.peers, rank=rank, world=world,
                                 max_tokens=mx.max_tokens, y_dtype=sp.F32)
            y_1 = sp.moe_ffn(fid, ga, ua, da, x, ids, wts, hidden=H, inter=I, n_experts_local=E, y_dtype=sp.F32)
            torch.cuda.synchronize()
            ys = [torch.empty_like(y_ep) for _ in range(world)]
            dist.all_gather(ys, y_ep)
            differ += sum(int((a.view(torch.int32) != y_ep.view(torch.int32)).sum().item()) for a in ys)
            rms = float(y_1.square().mean().sqrt())
            worst = max(worst, float(((y_ep - y_1).abs() / (y_1.abs() + rms)).max()))
        del ga, ua, da
        st = sp.device_status()
        t = torch.tensor([differ, st, worst], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        differ, st, worst = int(t[0]), int(t[1]), float(t[2])
        ok = differ == 0 and st == 0 and worst <= 2e-3
        parity = {"check": "identical on every rank; vs spiral_moe_ffn over all experts on one GPU, "
                           "|d| <= 2e-3 (|y| + rms(y)), every T", "rank_mismatches": differ,
                  "max_rel": worst, "device_status": st, "status": "ok" if ok else "FAIL"}
        if not ok:
            raise SystemExit(f"rank {rank}: expert-parallel MoE parity failed: {parity}")
    for T in Ts:
        x = torch.from_numpy(F.gen_activations(T, H, seed=T).view(np.int16)).to(dev).view(torch.bfloat16)
        rts = [F.gen_routing(T, E, topk, seed=1000 * T + r) for r in range(routings)]
        uniq = [len(set(ids.reshape(-1).tolist())) for ids, _ in rts]
        uloc = [len({int(v) for v in ids.reshape(-1) if e0 <= v < e1}) for ids, _ in rts]
        ids = [torch.from_numpy(a).to(dev) for a, _ in rts]
        wts = [torch.from_numpy(b).to(dev) for _, b in rts]
        y = torch.empty((T, H), dtype=torch.bfloat16, device=dev)
        ws = torch.empty(sp.moe_workspace_bytes(El, H, I, T, topk), dtype=torch.uint8, device=dev)

        def body(i, x=x, ids=ids, wts=wts, y=y, ws=ws):
            c, r = i % copies, (i // copies) % routings
            if world == 1:
                sp.moe_ffn(fid, wg[c], wu[c], wd[c], x, ids[r], wts[r], hidden=H, inter=I, n_experts_local=El,
                           expert_first=e0, y=y, workspace=ws)
            else:
                sp.moe_ffn_ep(fid, wg[c], wu[c], wd[c], x, ids[r], wts[r], hidden=H, inter=I, n_experts_local=El,
                              expert_first=e0, exchange_peers_dev=mx.peers, rank=rank, world=world,
                              max_tokens=mx.max_tokens, y=y, workspace=ws)

        steps = copies * routings  # one graph: every (copy, routing) pair once
        t = timer.timed(steps, 3, body, gsteps=steps) / steps * 1e-3
        cyc = [(i // copies) % routings for i in range(steps)]
        u_mean = sum(uniq[r] for r in cyc) / steps
        ul_mean = sum(uloc[r] for r in cyc) / steps
        wbytes = u_mean * MOE_BYTES_PER_EXPERT
        # roofline: the rank's own expert bytes (+ activations) over the layer time
        alg = ul_mean * MOE_BYTES_PER_EXPERT + T * H * 4
        res[f"T{T}"] = {"us": t * 1e6, "unique_experts": u_mean, "unique_experts_per_rank": ul_mean,
                        "weight_GBps": wbytes / t / 1e9,
                        "roofline": roofline("hbm", alg, t, hbm_peak, peak_kind, ("moe layer: gate/up, down, combine" if T * topk <= 16 else
                                              "moe layer: route, gate/up, down, combine")
                                             if world == 1 else "moe layer, combine fused over NVLink",
                                             profile_traffic(f"moe_T{T}_E{El}"))}
    del wg, wu, wd
    if mx is not None:
        torch.cuda.synchronize()
        del mx
    if parity is not None:
        res["parity"] = parity
    return res


def bench_extras(sp, F, dev, rank, world, timer, graph_steps, hbm_peak, tc_peak, peak_kind):
    """Every other BASELINE config, each with its own rotating buffers,
    graphs and roofline object; per-format / per-batch GEMV at N = 1."""
    import torch

    K, N = K_DIM, N_DIM
    out = {}
    if world == 1:
        out["gemv"] = {}
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

                steps = copies * max(1, 160 // copies)
                t = timer.timed(steps, 3, body, gsteps=copies) / steps * 1e-3
                alg = rb * N + B * K * 2 + B * N * 2
                out["gemv"][f"{name}_B{B}"] = {
                    "us": t * 1e6, "weight_GBps": rb * N / t / 1e9,
                    "roofline": roofline("hbm", alg, t, hbm_peak, peak_kind, f"gemv_xs_kernel<{name}>",
                                         profile_traffic(f"gemv_{name}_K{K}_N{N}_B{B}"))}
            del ws, w0
        # model shape (Gemma-style Q6_K output head, K = 1536, 262,144 rows:
        # 330 MB, larger than L2 on its own)
        fid, Kh, Nh = F.Q6_K, 1536, 262144
        rbh = F.row_bytes(fid, Kh)
        wh = torch.from_numpy(F.generate(fid, Kh, Nh, seed=0)).to(dev)
        for B in (1, 8):
            x = torch.from_numpy(F.gen_activations(B, Kh, seed=B).view(np.int16)).to(dev).view(torch.bfloat16)
            y = torch.empty((B, Nh), dtype=torch.bfloat16, device=dev)

            def body_h(i, x=x, y=y):
                sp.mul_mat(fid, wh, x, Nh, Kh, y, y_dtype=sp.BF16, static_weights=True)

            t = timer.timed(8, 3, body_h, gsteps=4) / 8 * 1e-3
            alg = rbh * Nh + B * Kh * 2 + B * Nh * 2
            out["gemv"][f"q6_k_K{Kh}_N{Nh}_B{B}"] = {
                "us": t * 1e6, "weight_GBps": rbh * Nh / t / 1e9,
                "roofline": roofline("hbm", alg, t, hbm_peak, peak_kind, "gemv_xs6_kernel<q6_k> (six-super-block rows)",
                                     profile_traffic(f"gemv_q6_k_K{Kh}_N{Nh}_B{B}"))}
        del wh
        # Gemma 4 E2B Q4_0 projections the reference lists for its first
        # end-to-end target (K = 1536 / 2048; N = 256 .. 12288): small
        # matrices, so a launch's fixed cost weighs in
        fid = F.Q4_0
        for Ke, Ne in ((1536, 256), (1536, 2048), (1536, 6144), (1536, 12288), (2048, 1536)):
            rbe = F.row_bytes(fid, Ke)
            raw = F.generate(fid, Ke, Ne, seed=0)
            copies = min(2048, max(8, math.ceil(2 * L2_BYTES / (rbe * Ne))))  # > 2x L2 in all
            w0 = torch.from_numpy(raw).to(dev)
            ws = [w0] + [w0.clone() for _ in range(copies - 1)]
            for B in (1, 8):
                x = torch.from_numpy(F.gen_activations(B, Ke, seed=B).view(np.int16)).to(dev).view(torch.bfloat16)
                y = torch.empty((B, Ne), dtype=torch.bfloat16, device=dev)

                def body_e(i, ws=ws, x=x, y=y, Ke=Ke, Ne=Ne, copies=copies):
                    sp.mul_mat(fid, ws[i % copies], x, Ne, Ke, y, y_dtype=sp.BF16, static_weights=True)

                t = timer.timed(copies, 3, body_e, gsteps=copies) / copies * 1e-3
                alg = rbe * Ne + B * Ke * 2 + B * Ne * 2
                out["gemv"][f"q4_0_K{Ke}_N{Ne}_B{B}"] = {
                    "us": t * 1e6, "weight_GBps": rbe * Ne / t / 1e9,
                    "roofline": roofline("hbm", alg, t, hbm_peak, peak_kind, "gemv_xs_kernel<q4_0> (Gemma 4 E2B shape)",
                                         profile_traffic(f"gemv_q4_0_K{Ke}_N{Ne}_B{B}"))}
            del ws, w0
    out["dequant"] = bench_dequant(sp, F, dev, rank, world, timer, graph_steps, hbm_peak, peak_kind)
    out["gemm"] = bench_gemm(sp, F, dev, rank, world, timer, hbm_peak, tc_peak, peak_kind)
    out["moe"] = bench_moe(sp, F, dev, rank, world, timer, graph_steps, hbm_peak, peak_kind)
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
