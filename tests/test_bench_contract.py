"""CPU: the bench's reference arm (the oracle's C4 training step on the host
cores) prints one JSON line with the keys the bench contract asks for, only
rank 0 prints under a multi-rank launch, and the roofline traffic lookup
returns the committed ncu figure only for the workload it was captured on."""
import json
import os
import subprocess
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent


def _run(env_extra):
    env = dict(os.environ, MALUS_BENCH_CPU_BATCH="1", **env_extra)
    return subprocess.run([sys.executable, str(ROOT / "bench.py"), "--impl", "reference", "--steps", "1",
                           "--warmup", "3"], cwd=ROOT, env=env, capture_output=True, text=True, timeout=600)


def test_reference_arm_line():
    r = _run({"RANK": "0", "WORLD_SIZE": "1"})
    assert r.returncode == 0, r.stderr
    lines = [l for l in r.stdout.splitlines() if l.startswith("{")]
    assert len(lines) == 1
    d = json.loads(lines[0])
    assert d["impl"] == "reference"
    assert d["metric"] == "nanoGPT f32 train tokens/s" and d["unit"] == "tokens/s"
    assert d["value"] > 0 and d["higher_is_better"] is True
    assert d["steps"] == 1 and d["warmup"] == 3
    cb = d["cpu_baseline"]
    assert cb["kind"] == "port" and cb["cores"] >= 1 and cb["value"] == d["value"] and cb["sample"]
    st = cb["single_thread"]
    assert st["cores"] == 1 and st["value"] > 0 and st["unit"] == "tokens/s"
    sys.path.insert(0, str(ROOT))
    try:
        import bench
    finally:
        sys.path.pop(0)
    assert d["config"] == bench.workload_config("c4", 1)   # the same config object as the GPU arm
    assert d["e2e"] == {"value": d["value"], "unit": "tokens/s", "h2d_bytes_per_step": 0,
                        "d2h_bytes_per_step": 0}


def test_reference_arm_other_ranks_silent():
    r = _run({"RANK": "1", "WORLD_SIZE": "2"})
    assert r.returncode == 0, r.stderr
    assert not [l for l in r.stdout.splitlines() if l.startswith("{")]


def test_traffic_lookup_only_for_captured_workload():
    sys.path.insert(0, str(ROOT))
    try:
        import bench
    finally:
        sys.path.pop(0)
    committed = json.loads((ROOT / "profiles" / "roofline_traffic.json").read_text())
    assert bench.traffic_from_profiles("k_gemm_tc", "c4", 1) == committed["k_gemm_tc"]["bytes_per_launch"]
    assert bench.traffic_from_profiles("k_gemm_tc", "c5", 1) is None
    assert bench.traffic_from_profiles("k_gemm_tc", "c4", 0) is None
