"""bench.py's contract on the CPU: the reference arm (the reference's own kernel library built from its sources,
or the oracle port where it is absent) prints one JSON line with the keys the driver reads; the GPU arms' flags
parse.  No GPU is used."""

from __future__ import annotations

import json
import os
import subprocess
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))


def test_reference_arm_prints_one_contract_line():
    env = dict(os.environ, WORLD_SIZE="1", RANK="0", LOCAL_RANK="0")
    p = subprocess.run([sys.executable, "bench.py", "--impl", "reference", "--steps", "2", "--warmup", "1"],
                       cwd=ROOT, capture_output=True, text=True, timeout=600, env=env)
    assert p.returncode == 0, p.stderr[-2000:]
    lines = [ln for ln in p.stdout.splitlines() if ln.strip()]
    assert len(lines) == 1
    d = json.loads(lines[0])
    for key in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better", "scaling",
                "vs_baseline", "dtype", "data", "config", "cpu_baseline", "e2e"):
        assert key in d, key
    assert d["impl"] == "reference" and d["value"] > 0 and d["steps"] == 2
    assert d["cpu_baseline"]["kind"] in ("reference", "port") and d["cpu_baseline"]["cores"] >= 1
    assert d["e2e"]["h2d_bytes_per_step"] == 0 and d["e2e"]["value"] == d["value"]
    # the driver divides the two arms' values only when metric, unit and direction agree
    import bench
    assert d["metric"] == bench.metric_name("adamw", "bf16")
    assert d["config"]["workload"] == bench.workload_name(bench.LLAMA7B, "adamw", "bf16", None)
    assert d["unit"] == "Gparams/s" and d["higher_is_better"] is True


def test_reference_arm_other_modes():
    env = dict(os.environ, WORLD_SIZE="1", RANK="0", LOCAL_RANK="0")
    p = subprocess.run([sys.executable, "bench.py", "--impl", "reference", "--steps", "1", "--warmup", "1",
                        "--algorithm", "lion", "--precision", "fp8"],
                       cwd=ROOT, capture_output=True, text=True, timeout=600, env=env)
    assert p.returncode == 0, p.stderr[-2000:]
    d = json.loads(p.stdout.strip().splitlines()[-1])
    import bench
    assert d["metric"] == bench.metric_name("lion", "fp8") and d["value"] > 0
    assert "lion fp8 moments" in d["cpu_baseline"]["sample"]


def test_cpu_baseline_variants():
    import argparse

    import bench
    args = argparse.Namespace(algorithm="adamw", precision="bf16", cpu_seconds=0.5, cpu_variant_seconds=0.2)
    block = bench.cpu_baseline_block(args)
    assert block["value"] > 0 and block["cores"] >= 1
    if block["kind"] == "reference":
        names = [v["variant"] for v in block["variants"]]
        assert names == ["reference default pool", "forced avx2", "fp8 moments", "fp8 moments, forced avx2"]
        assert block["variants"][0]["cores"] == bench.default_reference_threads()


def test_reference_arm_other_ranks_print_nothing():
    env = dict(os.environ, WORLD_SIZE="2", RANK="1", LOCAL_RANK="1")
    p = subprocess.run([sys.executable, "bench.py", "--impl", "reference", "--steps", "1", "--warmup", "1"],
                       cwd=ROOT, capture_output=True, text=True, timeout=300, env=env)
    assert p.returncode == 0 and p.stdout.strip() == ""


def test_flags_parse():
    p = subprocess.run([sys.executable, "bench.py", "--help"], cwd=ROOT, capture_output=True, text=True, timeout=120)
    assert p.returncode == 0
    for flag in ("--gpus", "--steps", "--warmup", "--impl", "--workload", "--algorithm", "--precision", "--rounds",
                 "--gather", "--clip", "--no-e2e", "--no-cpu-baseline", "--no-parity", "--cpu-variant-seconds"):
        assert flag in p.stdout, flag


def test_gather_labels_cover_every_mode():
    """Every all-gather a ZeRO optimizer can run (and none, on one GPU) has the name the bench line prints, and
    the flag offers each mode."""
    import bench
    assert set(bench.GATHER_LABELS) == {None, "p2p", "ce", "nccl"}
    p = subprocess.run([sys.executable, "bench.py", "--help"], cwd=ROOT, capture_output=True, text=True, timeout=120)
    for mode in ("auto", "p2p", "ce", "nccl"):
        assert mode in p.stdout
