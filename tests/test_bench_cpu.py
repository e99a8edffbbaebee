"""bench.py's reference arm (the CPU oracle on the host cores): one JSON line
with the contract's keys, a bounded per-step sample, and the sample sizing."""

import json
import os
import subprocess
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)

import bench  # noqa: E402


def test_sample_size_shrinks_with_steps():
    full = bench.sample_size(steps=3, warmup=1, num_points=1_000_000)
    small = bench.sample_size(steps=100, warmup=5, num_points=1_000_000)
    tiny = bench.sample_size(steps=10_000, warmup=5, num_points=1_000_000)
    assert full == (1_000_000, 256)
    assert small[0] < full[0] and small[1] == bench.MIN_SAMPLE_TILES
    assert tiny[0] == round(1_000_000 / 64)


def test_reference_arm_prints_one_contract_line():
    out = subprocess.run(
        [sys.executable, os.path.join(ROOT, "bench.py"), "--impl", "reference", "--steps", "2",
         "--warmup", "1", "--points", "20000"],
        capture_output=True, text=True, timeout=600, cwd=ROOT, check=True).stdout
    lines = [line for line in out.splitlines() if line.startswith("{")]
    assert len(lines) == 1
    d = json.loads(lines[0])
    assert d["impl"] == "reference" and d["unit"] == "views/s" and d["value"] > 0
    assert d["steps"] == 2 and d["warmup"] == 1 and d["higher_is_better"] is True
    assert d["cpu_baseline"]["kind"] == "port" and d["cpu_baseline"]["value"] == d["value"]
    assert d["e2e"] == {"value": d["value"], "unit": "views/s", "h2d_bytes_per_step": 0,
                        "d2h_bytes_per_step": 0}
