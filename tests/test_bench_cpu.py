"""bench.py's reference arm (the CPU oracle on the host cores): one JSON line
with the contract's keys, whole views timed on an explicit thread count, and
the workload description both arms share."""

import json
import os
import subprocess
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)

import bench  # noqa: E402


def test_both_arms_describe_the_workload_alike():
    from gaussian_splats_b200 import scenes

    scene = scenes.config2(num_points=64)
    config = bench.workload_config(2, scene)
    assert config["workload"].startswith("config2") and config["gaussians"] == 64
    assert config["image"] == [1920, 1080] and config["tile_size"] == 16
    # nothing about ranks or launch mode: that goes under "run"
    assert not {"parallelism", "step", "views_per_step"} & set(config)


def test_reference_arm_prints_one_contract_line():
    out = subprocess.run(
        [sys.executable, os.path.join(ROOT, "bench.py"), "--impl", "reference", "--steps", "2",
         "--warmup", "1", "--points", "20000"],
        capture_output=True, text=True, timeout=600, cwd=ROOT, check=True,
        env=dict(os.environ, OMP_NUM_THREADS="1")).stdout
    lines = [line for line in out.splitlines() if line.startswith("{")]
    assert len(lines) == 1
    d = json.loads(lines[0])
    assert d["impl"] == "reference" and d["unit"] == "views/s" and d["value"] > 0
    assert d["steps"] == 2 and d["warmup"] == 1 and d["higher_is_better"] is True
    assert d["cpu_baseline"]["kind"] == "port" and d["cpu_baseline"]["value"] == d["value"]
    assert d["e2e"] == {"value": d["value"], "unit": "views/s", "h2d_bytes_per_step": 0,
                        "d2h_bytes_per_step": 0}
    # the whole timed region is K whole views, on every host core despite OMP_NUM_THREADS=1
    assert abs(d["ms_per_step"] * d["steps"] / 1e3 - d["steps"] / d["value"]) < 1e-6
    assert d["cpu_baseline"]["cores"] == bench.host_cores()
    assert "whole views" in d["cpu_baseline"]["sample"]
    from gaussian_splats_b200 import scenes

    assert d["config"] == bench.workload_config(2, scenes.config2(num_points=20000))


def test_launch_count_per_view():
    # 1080p at 16x16: 8160 tiles, 13 bits, two tile-sort passes.
    assert bench.sort_passes(8160) == 2 and bench.sort_passes(256) == 1
    assert bench.sort_passes(1) == 0
    # 1080p at 16x16 tiles (row/column binning): 16 forward launches, 8 more
    # for the training step's loss, plan and backward
    assert bench.launches_per_view(120, 68, backward=True) == 24
    assert bench.launches_per_view(120, 68, backward=True, peers=True) == 27
    assert bench.launches_per_view(120, 68, backward=True, peers=True, sharded=True) == 28
    # a grid too wide for the row/column tables: count scan, emit, histogram,
    # two tile-sort passes and ranges
    assert bench.launches_per_view(300, 6, backward=False) == 15
    assert bench.launches_per_view(120, 68, backward=False) == 16
    assert bench.launches_per_view(16, 16, backward=True) == 24


def test_views_split_over_ranks():
    from gaussian_splats_b200 import scenes

    multi = scenes.config4(num_points=64)
    for world in (1, 2, 4, 8):
        got = [bench.views_for_rank(multi, 4, r, world) for r in range(world)]
        assert sum(len(v) for v in got) == 64
        assert all(target is None for v in got for _, target in v)  # forward only
    single = scenes.config2(num_points=64)
    first = bench.views_for_rank(single, 2, 0, 2)
    second = bench.views_for_rank(single, 2, 1, 2)
    assert first[0][0] is single.cameras[0] and first[0][1] is single.targets[0]
    assert len(second) == 1 and second[0][1].shape == (1080, 1920, 3)
    assert not (second[0][0].position == first[0][0].position).all()


def test_reference_arm_forward_only_config():
    out = subprocess.run(
        [sys.executable, os.path.join(ROOT, "bench.py"), "--impl", "reference", "--config", "4",
         "--steps", "1", "--warmup", "0", "--points", "20000"],
        capture_output=True, text=True, timeout=600, cwd=ROOT, check=True).stdout
    d = json.loads([line for line in out.splitlines() if line.startswith("{")][0])
    assert d["value"] > 0 and d["config"]["workload"].startswith("config4")
    assert "projection backward" not in d["cpu_baseline"]["sample"]
