"""The bench's JSON contract on the CPU: the reference arm (the oracle port
timed on host cores) prints one line with the keys the driver reads, and
under torchrun only rank 0 prints.  The GPU arm's line is produced on a
B200; its keys are the same set plus roofline, clocks and extras."""

from __future__ import annotations

import json
import os
import subprocess
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]
KEYS = {"metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better", "scaling",
        "vs_baseline", "dtype", "data", "config", "cpu_baseline", "e2e", "gpu_launches"}


def _run(env_extra: dict) -> subprocess.CompletedProcess:
    env = dict(os.environ, **env_extra)
    return subprocess.run([sys.executable, "bench.py", "--impl", "reference", "--steps", "1", "--warmup", "1"],
                          cwd=ROOT, env=env, capture_output=True, text=True, timeout=600)


def test_reference_arm_prints_one_contract_line():
    r = _run({"RANK": "0", "WORLD_SIZE": "1"})
    assert r.returncode == 0, r.stderr[-2000:]
    lines = [ln for ln in r.stdout.splitlines() if ln.startswith("{")]
    assert len(lines) == 1
    line = json.loads(lines[0])
    assert KEYS <= set(line)
    assert line["impl"] == "reference"
    assert line["unit"] == "GB/s" and line["higher_is_better"] is True and line["value"] > 0
    assert line["config"]["workload"].startswith("cfg2 q4_0")
    assert line["cpu_baseline"]["kind"] == "port" and line["cpu_baseline"]["cores"] >= 1
    assert line["e2e"]["h2d_bytes_per_step"] == 0 and line["e2e"]["d2h_bytes_per_step"] == 0
    assert line["gpu_launches"] == 0


def test_reference_arm_uses_every_core_under_torchrun():
    """torchrun exports OMP_NUM_THREADS=1; the CPU arm must still run (and
    report) one thread per host core, with the GPU arm's config."""
    sys.path.insert(0, str(ROOT))
    import bench

    r = _run({"RANK": "0", "WORLD_SIZE": "2", "LOCAL_RANK": "0", "OMP_NUM_THREADS": "1"})
    assert r.returncode == 0, r.stderr[-2000:]
    line = json.loads([ln for ln in r.stdout.splitlines() if ln.startswith("{")][0])
    assert line["cpu_baseline"]["cores"] == (os.cpu_count() or 1)
    assert line["config"] == bench.headline_config("q4_0", 2)


def test_cpu_extras_cover_every_config():
    """The per-config CPU figures the GPU arm adds at N = 1 (C restatement
    per config, NumPy dequant and matmul, the reference's own repack)."""
    sys.path.insert(0, str(ROOT))
    import bench

    out = bench.cpu_extras(budget_s=0.05)
    assert set(out["dequant"]) == {"q4_0_4096x4096", "q8_0_14336x4096", "q6_k_14336x4096"}
    assert set(out["gemm"]) == {"q4_0_M512", "q4_0_M2048", "q6_k_M512", "q6_k_M2048"}
    assert set(out["moe"]) == {"T1", "T8"}
    for group in ("dequant", "gemm", "moe"):
        for v in out[group].values():
            assert v["value"] > 0 and v["cores"] >= 1
    assert out["numpy_dequant_q4_0"]["value"] > 0
    assert out["numpy_matmul_f32_B8"]["value"] > 0
    for v in out["reference_repack"].values():
        assert "unavailable" in v or (v["value"] > 0 and v["kind"] == "reference")


def test_reference_arm_other_ranks_exit_quietly():
    r = _run({"RANK": "1", "WORLD_SIZE": "2", "LOCAL_RANK": "1"})
    assert r.returncode == 0, r.stderr[-2000:]
    assert not [ln for ln in r.stdout.splitlines() if ln.startswith("{")]
