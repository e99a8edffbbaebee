"""Benchmark: config 2 -- one 1920x1080 view of 1M Gaussians (SH degree 3),
forward + backward with an L1 loss -- per GPU.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b200|reference]

With N > 1 (launched by torchrun, one rank per GPU) every rank renders its own
camera of the same replicated scene and the parameter gradients are summed
with one NCCL all-reduce per step (view-parallel training, weak scaling).
Rank 0 prints one JSON line. ``value`` is views/s over all ranks, timed with
CUDA events over K steps (max over ranks). Inputs exceed the 126 MB L2
(236 MB of Gaussian parameters are read every step), so no flush is needed.

``--impl reference`` times the reference algorithm on the host CPU cores: the
C restatement of the reference's rasterizer in ``oracle/`` (the reference is
Python with Triton kernels and does not travel to the GPU box). Each step is a
bounded sample of the view -- projection, binning and projection backward of
a chunk of the Gaussians, compositing forward and backward of a sample of
tiles, each scaled to the whole view -- sized so the run stays within about
two minutes whatever --steps and --warmup are.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

import numpy as np  # noqa: E402
import torch  # noqa: E402

METRIC = "fwd / fwd+bwd ms per 1080p view at 1M Gaussians; views/sec at 1/2/4/8 GPUs"
UNIT = "views/s"

# The BASELINE configs. Config 2 is the headline (the default); the others
# are measured with --config. `views`: cameras per step over all ranks (None:
# one camera per rank, weak scaling); `backward`: fwd+bwd with an L1 loss.
WORKLOADS = {
    1: dict(name="config1: 16,384 Gaussians SH0, 256x256, 16x16 tiles, fwd+bwd L1 (random "
                 "target)", views=None, backward=True),
    2: dict(name="config2: 1M Gaussians SH3, 1920x1080 (rendered 1920x1088), 16x16 tiles, "
                 "fwd+bwd L1", views=None, backward=True),
    3: dict(name="config3: 3M Gaussians SH3, 8 cameras per step split over ranks, 1600x1064 "
                 "(rendered 1600x1072), fwd+bwd L1, gradient all-reduce", views=8,
            backward=True),
    4: dict(name="config4: 6M Gaussians SH3, 3840x2160, 64-camera orbit split over ranks, "
                 "forward only", views=64, backward=False),
    5: dict(name="config5: 500k Gaussians SH1 in one dense blob, 1920x1080 (rendered "
                 "1920x1088), fwd+bwd L1", views=None, backward=True),
}
WORKLOAD = WORKLOADS[2]["name"]


# Algorithmic bytes per Gaussian with K SH coefficients: projection reads
# mean, rotation, scale, opacity (44 B) and colour (12K B) and writes
# projected mean, conic, colour, opacity, tile rectangle, count (64 B);
# projection backward reads the same parameters plus conic, the 9-float
# screen-space gradient and the count (56 B) and writes 44 + 12K B of
# gradients. K = 16: 300 B and 528 B.
def project_fwd_bytes(k):
    return 44 + 12 * k + 64


def project_bwd_bytes(k):
    return 44 + 12 * k + 56 + 44 + 12 * k


PROJECT_FWD_BYTES = project_fwd_bytes(16)
PROJECT_BWD_BYTES = project_bwd_bytes(16)
# Per evaluated (pixel, Gaussian) pair, the reference's forward arithmetic
# (composite.py:159-186): offsets 2, distance 9, exp argument 1, exp 1,
# alpha 4, activity test 3, weight 2, colour 6, transmittance 3.
COMPOSITE_FWD_FLOPS = 31
# Backward per evaluated pair (composite_bwd.py:101-195 without the dropped
# abs-gradient): distance and alpha 16, T recovery 5, weight gradient 9,
# alpha/opacity/distance gradients 6, mean/conic gradients 14, colour 4,
# suffix update 10.
COMPOSITE_BWD_FLOPS = 64


def parse_args():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=100)
    p.add_argument("--warmup", type=int, default=5)
    p.add_argument("--impl", choices=("b200", "reference"), default="b200")
    p.add_argument("--config", type=int, choices=sorted(WORKLOADS), default=2,
                   help="BASELINE config to run (2, the headline, by default)")
    p.add_argument("--points", type=int, default=None,
                   help="override the config's Gaussian count (smaller smoke runs)")
    p.add_argument("--no-cpu-baseline", action="store_true")
    p.add_argument("--no-graph", action="store_true",
                   help="launch the training step from Python instead of replaying it from "
                        "a CUDA graph")
    p.add_argument("--exchange", choices=("auto", "screen", "screen-nccl", "all-reduce"),
                   default="auto",
                   help="how ranks sum gradients with one view per rank (auto: "
                        "view_parallel.screen_exchange_pays)")
    return p.parse_args()


def load_peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        with open(path) as f:
            peaks = json.load(f)
        return float(peaks["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


class ClockSampler:
    """nvidia-smi clocks and throttle reasons sampled during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
    PERIOD_MS = 50

    def __init__(self, index):
        self.index = index
        self.proc = None
        self.path = os.path.join(ROOT, "gpurun_out", f"clocks_rank{index}.csv")

    def __enter__(self):
        try:
            os.makedirs(os.path.dirname(self.path), exist_ok=True)
            self.file = open(self.path, "w")
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-i", str(self.index), "-lms", str(self.PERIOD_MS)], stdout=self.file,
                stderr=subprocess.DEVNULL)
        except (OSError, FileNotFoundError):
            self.proc = None
            return self
        # nvidia-smi takes a moment to start; begin timing once it samples.
        deadline = time.time() + 5.0
        while time.time() < deadline and os.path.getsize(self.path) == 0:
            time.sleep(0.02)
        self.lines_before = self._line_count()
        return self

    def _line_count(self):
        with open(self.path) as f:
            return sum(1 for _ in f)

    def __exit__(self, *exc):
        if self.proc is not None:
            # Samples written up to now (plus the one in flight) cover the
            # region; later ones would be of an idle GPU.
            time.sleep(self.PERIOD_MS / 1000.0)
            self.lines_after = self._line_count()
            self.proc.terminate()
            self.proc.wait(timeout=10)
            self.file.close()

    def summary(self):
        if self.proc is None:
            return None
        rows = []
        with open(self.path) as f:
            lines = f.readlines()
        # Keep the samples taken while the timed region ran (the last one
        # before it started bounds it from below).
        first = max(0, self.lines_before - 1)
        window = lines[first:self.lines_after] or lines
        for line in window:
            parts = [x.strip() for x in line.split(",")]
            if len(parts) >= 9 and parts[1].replace(".", "").isdigit():
                rows.append(parts)
        if not rows:
            return None
        sm = [float(r[1]) for r in rows]
        reasons = set()
        names = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")
        for r in rows:
            for name, flag in zip(names, r[5:9]):
                if flag.lower() == "active":
                    reasons.add(name)
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": float(rows[0][2]),
                "samples": len(rows), "reasons": sorted(reasons)}


def fp32_peak_tflops(device):
    """FP32 CUDA-core peak measured live: cuBLAS SGEMM 8192^3 with TF32 off.
    MEASURED_PEAKS.json carries HBM and bf16 figures only."""
    prev = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    try:
        a = torch.randn(8192, 8192, device=device)
        b = torch.randn(8192, 8192, device=device)
        for _ in range(2):
            a @ b
        torch.cuda.synchronize()
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        best = float("inf")
        for _ in range(5):
            start.record()
            a @ b
            end.record()
            torch.cuda.synchronize()
            best = min(best, start.elapsed_time(end))
        return 2 * 8192 ** 3 / (best * 1e-3) / 1e12
    finally:
        torch.backends.cuda.matmul.allow_tf32 = prev


def kernel_durations(outputs, params, camera, grad_image, settings, device, repeats=5):
    """Per-launch milliseconds of the four main kernels (the two forward ones
    when `grad_image` is None), each launched through
    the C ABI right after a 1 GiB L2 flush, with CUDA events around the launch
    on the launching stream (the GPU is still busy with the flush when the
    launch is enqueued, so no host gap is timed). Returns {stage: mean ms}."""
    import ctypes

    from gaussian_splats_b200 import native

    lib = native.lib()
    (image, final_t, n_contrib, pmean, conic, pcolor, popacity, ids, ranges, counts) = outputs
    mean, rotation, scale, opacity, color = params
    n, k = mean.shape[0], color.shape[1]
    w, h = camera.image_size
    fx, fy = camera.focal_length
    cx, cy = camera.principal_point
    prm = native.make_params(fx, fy, cx, cy, w, h, settings.tile_size,
                             settings.opacity_threshold, settings.near, settings.far,
                             settings.rendering_mode, settings.confidence)
    pref = ctypes.byref(prm)
    cam_r = camera.rotation_matrix.to(device)
    cam_t = camera.translation.to(device)
    P = lambda t: ctypes.c_void_p(t.data_ptr() if t.numel() else 0)  # noqa: E731
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    out_pm, out_conic = torch.empty_like(pmean), torch.empty_like(conic)
    out_rgb, out_o = torch.empty_like(pcolor), torch.empty_like(popacity)
    bounds = torch.empty((n, 4), dtype=torch.int32, device=device)
    out_counts = torch.empty_like(counts)
    out_img, out_t = torch.empty_like(image), torch.empty_like(final_t)
    out_nc = torch.empty_like(n_contrib)
    grad_projected = torch.empty((n, 9), device=device)
    grads = [torch.empty_like(t) for t in params] if grad_image is not None else None
    launches = {
        "project_fwd": lambda: lib.gs_project_fwd(
            n, k, P(mean), P(rotation), P(scale), P(opacity), P(color), P(cam_r), P(cam_t), pref,
            P(out_pm), P(out_conic), P(out_rgb), P(out_o), P(bounds), P(out_counts), stream),
        "composite_fwd": lambda: lib.gs_composite_fwd(
            P(pmean), P(conic), P(pcolor), P(popacity), P(ids), P(ranges), pref, P(out_img),
            P(out_t), P(out_nc), stream),
    }
    if grad_image is not None:
        launches["composite_bwd"] = lambda: lib.gs_composite_bwd(
            n, P(pmean), P(conic), P(pcolor), P(popacity), P(ids), P(ranges), P(grad_image),
            P(final_t), P(n_contrib), pref, P(grad_projected), stream)
        launches["project_bwd"] = lambda: lib.gs_project_bwd(
            n, k, P(mean), P(rotation), P(scale), P(opacity), P(color), P(cam_r), P(cam_t),
            P(conic), P(grad_projected), P(counts), pref, *(P(g) for g in grads), stream)
    flush = torch.empty(1 << 28, dtype=torch.float32, device=device)  # 1 GiB > 126 MB L2
    result = {}
    for name, launch in launches.items():
        events = []
        for _ in range(repeats):
            flush.zero_()
            before, after = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            before.record()
            native.check(launch(), name)
            after.record()
            events.append((before, after))
        torch.cuda.synchronize()
        result[name] = sum(b.elapsed_time(a) for b, a in events) / repeats
    return result


def load_scene(config, points=None):
    """The config's seeded synthetic scene (CPU tensors)."""
    from gaussian_splats_b200 import scenes

    make = getattr(scenes, f"config{config}")
    return make() if points is None else make(num_points=points)


# Camera recipe (distance from the origin, vertical FOV) of the single-view
# configs, for the extra cameras of ranks > 0.
_SINGLE_VIEW_RECIPE = {1: (4.0, 60.0), 2: (5.0, 50.0), 5: (2.5, 70.0)}


def views_for_rank(scene, config, rank, world):
    """(camera, target) pairs this rank renders each step. Single-view configs:
    rank 0 renders the config's camera, other ranks a camera of the same recipe
    from a direction seeded by the rank (weak scaling). Multi-view configs: the
    config's cameras split over the ranks (strong scaling). Targets are None
    for forward-only configs; configs without targets get uniform ones."""
    from gaussian_splats_b200 import scenes
    from gaussian_splats_b200.view_parallel import shard_views

    width, height = scene.crop
    backward = WORKLOADS[config]["backward"]

    def target(i, g):
        if not backward:
            return None
        if scene.targets and i is not None:
            return scene.targets[i]
        return torch.rand(height, width, 3, generator=g)

    if WORKLOADS[config]["views"] is None:
        if rank == 0:
            return [(scene.cameras[0], target(0, torch.Generator().manual_seed(999)))]
        g = torch.Generator().manual_seed(1000 + rank)
        distance, fov = _SINGLE_VIEW_RECIPE[config]
        cam = scenes.look_at_camera(distance * scenes.random_direction(g), fovy_degrees=fov,
                                    width=width, height=height)
        return [(cam, target(None, g))]
    return [(scene.cameras[i], target(i, None))
            for i in shard_views(len(scene.cameras), world, rank)]


# Seconds of CPU work the reference arm may spend on its timed and warm-up
# steps together. A step always composites at least MIN_SAMPLE_TILES tiles
# (enough to keep every host thread busy); the chunk of Gaussians projected,
# binned and back-projected shrinks with the time left per step.
REFERENCE_BUDGET_S = 120.0
MIN_SAMPLE_TILES = 128


def sample_size(steps, warmup, num_points):
    """(Gaussians in the chunk, tiles) of one reference-arm step."""
    per_step = REFERENCE_BUDGET_S / max(1, steps + warmup)
    tiles = 256 if per_step >= 2.0 else MIN_SAMPLE_TILES
    fraction = min(1.0, max(1.0 / 64.0, (per_step - 0.6) / 4.4))
    return max(1, int(round(num_points * fraction))), tiles


def run_reference(args, rank, world):
    """CPU restatement of the reference, timed on this host's cores (rank 0).
    Each step is a bounded sample of the view, sized so warm-up plus timed
    steps stay within about REFERENCE_BUDGET_S."""
    if rank != 0:
        return
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle as O

    scene = load_scene(args.config, args.points)
    backward = WORKLOADS[args.config]["backward"]
    cores = os.cpu_count() or 1
    os.environ.setdefault("OMP_NUM_THREADS", str(cores))
    chunk, tiles = sample_size(args.steps, args.warmup, scene.num_points)
    view = cpu_view_setup(O, scene, backward)
    step_s = []
    sample = None
    for i in range(args.warmup + args.steps):
        seconds, sample = cpu_view_seconds(O, view, chunk=chunk, tiles=tiles, seed=i)
        if i >= args.warmup:
            step_s.append(seconds)
    per_view = statistics.median(step_s)
    value = 1.0 / per_view
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": per_view * 1e3,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic", "config": {"workload": WORKLOADS[args.config]["name"]},
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": cores, "kind": "port",
                         "sample": sample},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def cpu_view_setup(O, scene, backward=True):
    """The whole view's projection and binning (of the scene's first camera),
    which the sampled compositing steps read, and the per-view fixed cost of
    the compositing calls (image buffers; in the backward the [intersections,
    9] row buffer and its reduction per Gaussian), timed once with an empty
    tile list."""
    inputs, s = O.scene_inputs(scene)
    keys = ("mean", "rotation", "scale", "opacity", "color", "camera_rotation",
            "camera_translation")
    proj = O.project(*(inputs[k] for k in keys), s)
    binned = O.bin(proj["bounds"], proj["projected_mean"][:, 2], proj["counts"], s)
    width, height = scene.crop
    grad_image = np.full((s.height, s.width, 3), 1.0 / (width * height * 3), np.float32)
    view = {"scene": scene, "inputs": inputs, "settings": s, "keys": keys, "proj": proj,
            "binned": binned, "grad_image": grad_image, "backward": backward}
    none = np.zeros((0,), np.int32)
    fixed = [composite_seconds(O, view, none) for _ in range(6)][1:]  # first call warms up
    view["fixed_fwd"] = statistics.median(f[0] for f in fixed)
    view["fixed_bwd"] = statistics.median(f[1] for f in fixed)
    return view


def composite_seconds(O, view, tiles):
    """Seconds of the oracle's compositing forward and backward over `tiles`."""
    s, proj, binned = view["settings"], view["proj"], view["binned"]
    t0 = time.perf_counter()
    comp = O.composite(proj["projected_mean"], proj["inverse_covariance"],
                       proj["projected_color"], proj["projected_opacity"],
                       binned["gaussian_ids"], binned["ranges"], s, tiles=tiles)
    t1 = time.perf_counter()
    if view["backward"]:
        O.composite_bwd(dict(proj, **binned, **comp), view["grad_image"], s, tiles=tiles)
    t2 = time.perf_counter()
    return t1 - t0, t2 - t1


def cpu_view_seconds(O, view, chunk, tiles, seed):
    """Seconds for one config-2 view on the CPU oracle, from a bounded sample:
    projection, binning and projection backward of a contiguous random chunk
    of `chunk` Gaussians scaled to all of them, plus compositing forward and
    backward of `tiles` random tiles -- the per-view fixed cost once, the
    per-tile remainder scaled to all tiles by list entries."""
    s, inputs, keys = view["settings"], view["inputs"], view["keys"]
    n = view["scene"].num_points
    rng = np.random.default_rng(seed)
    first = int(rng.integers(0, n - chunk + 1))
    part = slice(first, first + chunk)
    chunk_inputs = [inputs[k][part] if k not in ("camera_rotation", "camera_translation")
                    else inputs[k] for k in keys]
    chosen = rng.choice(s.num_tiles, size=min(tiles, s.num_tiles), replace=False).astype(np.int32)
    # Longest lists first, so the host threads' dynamic schedule balances a
    # small sample as well as it balances the whole view.
    ranges = view["binned"]["ranges"]
    chosen = chosen[np.argsort(-(ranges[chosen, 1] - ranges[chosen, 0]), kind="stable")]
    t0 = time.perf_counter()
    chunk_proj = O.project(*chunk_inputs, s)
    t1 = time.perf_counter()
    O.bin(chunk_proj["bounds"], chunk_proj["projected_mean"][:, 2], chunk_proj["counts"], s)
    t2 = time.perf_counter()
    fwd_s, bwd_s = composite_seconds(O, view, chosen)
    grad_projected = np.zeros((chunk, 9), np.float32)
    t3 = time.perf_counter()
    if view["backward"]:
        O.project_bwd(*chunk_inputs, chunk_proj["inverse_covariance"], grad_projected,
                      chunk_proj["counts"], s)
    t4 = time.perf_counter()
    gaussian_scale = n / chunk
    # Ratio estimate: compositing time follows the list entries walked, so the
    # sampled tiles' time is scaled by all entries over the sampled entries.
    lengths = ranges[:, 1] - ranges[:, 0]
    tile_scale = float(lengths.sum()) / max(1.0, float(lengths[chosen].sum()))
    fixed = view["fixed_fwd"] + view["fixed_bwd"]
    per_tile = max(0.0, fwd_s + bwd_s - fixed)
    seconds = ((t1 - t0) + (t2 - t1) + (t4 - t3)) * gaussian_scale + fixed + per_tile * tile_scale
    what = "projection, binning, projection backward" if view["backward"] else \
        "projection, binning"
    sample = (f"one view: {what} of {chunk} of "
              f"{n} Gaussians scaled by {gaussian_scale:.2f}; composite "
              f"{'fwd+bwd' if view['backward'] else 'fwd'} on "
              f"{len(chosen)} of {s.num_tiles} random tiles, per-tile time scaled by "
              f"{tile_scale:.1f} (all list entries / sampled entries), per-view fixed "
              f"time ({fixed:.2f} s) counted once")
    return seconds, sample


# Algorithmic bytes per Gaussian of one fused optimizer step with K SH
# coefficients: parameter, gradient and both Adam moments read (4 x (11 + 3K)
# floats), the position noise's normal samples read (3 floats), parameter and
# moments written (3 x (11 + 3K) floats). K = 16: 1,664 B.
def optimizer_bytes(k):
    return 4 * (7 * (11 + 3 * k) + 3)


def optimizer_timings(params, grads, device, repeats=5):
    """Milliseconds of one training-loop optimizer step on these parameters
    and gradients: the fused step (FusedAdam with position noise) and, for
    comparison, what the reference runs -- torch.optim.Adam (eps 1e-15) then
    noise_splats' tensor ops (training/utils.py:50-62) -- each after a 1 GiB
    L2 flush, timed with CUDA events."""
    import torch.nn.functional as F

    from gaussian_splats_b200.optim import GROUP_NAMES, FusedAdam
    from gaussian_splats_b200.utils import quaternion_to_rotation_matrix

    lrs = (1.6e-4, 1e-3, 5e-3, 5e-2, 2.5e-3)  # training/train.py:78-83

    def copies():
        tensors = [p.detach().clone().requires_grad_() for p in params]
        for t, g in zip(tensors, grads):
            t.grad = g.clone()
        return tensors

    def noise_splats(mean, rotation, scale, opacity, noise_lr, position_lr):
        rot = quaternion_to_rotation_matrix(F.normalize(rotation, dim=-1))
        factor = rot * scale.exp()[:, None, :]
        covariance = factor @ factor.transpose(-1, -2)
        gate = torch.sigmoid(100 * (1 - opacity.sigmoid() - 0.995))
        noise = torch.randn_like(mean) * gate * noise_lr * position_lr
        mean.add_((covariance @ noise[..., None]).squeeze(-1))

    ours = copies()
    fused = FusedAdam([{"params": [t], "name": n, "lr": lr}
                       for t, n, lr in zip(ours, GROUP_NAMES, lrs)], eps=1e-15)
    theirs = copies()
    plain = torch.optim.Adam([{"params": [t], "lr": lr} for t, lr in zip(theirs, lrs)],
                             eps=1e-15)

    def reference_step():
        plain.step()
        with torch.no_grad():
            noise_splats(theirs[0], theirs[1], theirs[2], theirs[3], 5e5, lrs[0])

    flush = torch.empty(1 << 28, dtype=torch.float32, device=device)
    result = {}
    for name, fn in (("fused", lambda: fused.step(noise=(5e5, lrs[0]))),
                     ("torch", reference_step)):
        fn()  # first step allocates the moments
        events = []
        for _ in range(repeats):
            flush.zero_()
            before, after = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            before.record()
            fn()
            after.record()
            events.append((before, after))
        torch.cuda.synchronize()
        result[name] = sum(b.elapsed_time(a) for b, a in events) / repeats
    return result


DEAD_FRACTION = 0.03  # rows made dead for the relocation timing


def relocation_timings(params, device, repeats=3):
    """Milliseconds of one splat relocation as the reference's training loop
    runs it once the count has reached max_splats (density factor 1.0: dead
    rows replaced by copies of live ones sampled by opacity, the Adam moments
    of every touched row zeroed): gaussian_splats_b200.relocate with FusedAdam
    state, and for comparison the reference's tensor ops (training/utils.py:
    83-193, restated with torch) on torch.optim.Adam state. The parameters are
    these, with a seeded DEAD_FRACTION of rows given opacity logit -8. Both
    draw the same copies (same seed). CUDA events around the whole call (its
    host waits included), after a 1 GiB L2 flush; mean over ``repeats``."""
    import math

    from gaussian_splats_b200 import relocate as R
    from gaussian_splats_b200.optim import GROUP_NAMES, FusedAdam
    from gaussian_splats_b200.splats import GaussianSplat

    n = len(params[0])
    order = torch.randperm(n, generator=torch.Generator().manual_seed(77))
    dead_rows = order[: int(DEAD_FRACTION * n)].to(device)
    degree = torch.arange(1, 52, device=device)
    table = torch.tensor([[math.comb(m, d) if d <= m else 0 for d in range(1, 52)]
                          for m in range(52)], dtype=torch.float32, device=device)
    table = table * ((-1.0) ** (degree - 1) / degree.sqrt())

    def fresh(optimizer_class):
        tensors = [p.detach().clone() for p in params]
        tensors[3][dead_rows] = -8.0
        splats = GaussianSplat.from_tensors(*tensors)
        opt = optimizer_class([{"params": [getattr(splats, k)], "name": k, "lr": 1e-3}
                               for k in GROUP_NAMES], eps=1e-15)
        for k in GROUP_NAMES:
            p = getattr(splats, k)
            opt.state[p] = {"step": torch.tensor(1.0), "exp_avg": torch.full_like(p, 0.1),
                            "exp_avg_sq": torch.full_like(p, 0.01)}
        return splats, opt

    @torch.no_grad()
    def torch_relocate(splats, opt):
        opacity = splats.opacity.sigmoid().squeeze(-1)
        dead_mask = opacity < 0.005
        dead = dead_mask.nonzero().squeeze(-1)
        drawn = torch.multinomial(opacity.masked_fill(dead_mask, 0), len(dead), replacement=True)
        counts = torch.bincount(drawn, minlength=n).cpu()
        parent_rows = counts.nonzero().squeeze(-1)
        copies = counts[parent_rows].to(device)
        parent_rows = parent_rows.to(device)
        source = parent_rows.repeat_interleave(copies)
        o = opacity[parent_rows]
        total = (copies + 1).clamp(1, 51)
        o_new = 1 - (1 - o).pow(1 / total)
        series = table[total] * o_new[:, None].pow(degree) * (degree <= total[:, None])
        s_new = splats.scale[parent_rows].exp() * (o / series.sum(-1))[:, None]
        o_new = o_new.clamp(0.005, 1 - 1e-6)
        for name in ("mean", "rotation", "color", "normals"):
            value = getattr(splats, name)
            value.index_copy_(0, dead, value[source])
        splats.opacity.index_copy_(0, parent_rows, torch.logit(o_new)[:, None])
        splats.opacity.index_copy_(0, dead, torch.logit(o_new.repeat_interleave(copies))[:, None])
        splats.scale.index_copy_(0, parent_rows, s_new.log())
        splats.scale.index_copy_(0, dead, s_new.repeat_interleave(copies, dim=0).log())
        rows = torch.cat((parent_rows, dead)).unique()
        for state in opt.state.values():
            for key in ("exp_avg", "exp_avg_sq"):
                state[key][rows] = 0

    flush = torch.empty(1 << 28, dtype=torch.float32, device=device)
    result = {}
    for name, optimizer_class, fn in (
            ("fused", FusedAdam, lambda s, o: R.relocate_splats(s, o, 1.0)),
            ("torch", torch.optim.Adam, torch_relocate)):
        times = []
        for _ in range(repeats + 1):  # the first run warms up
            splats, opt = fresh(optimizer_class)
            flush.zero_()
            torch.manual_seed(2024)
            before, after = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            before.record()
            fn(splats, opt)
            after.record()
            torch.cuda.synchronize()
            times.append(before.elapsed_time(after))
            del splats, opt
        result[name] = sum(times[1:]) / repeats
    result["dead_rows"] = len(dead_rows)
    return result


BATCH_VIEWS = 16  # cameras per rasterize_batch call in forward-only multi-camera configs


def sort_passes(num_tiles):
    """8-bit radix passes of the tile sort for `num_tiles` tiles."""
    bits = max(0, (max(1, num_tiles) - 1).bit_length())
    return (bits + 7) // 8


def launches_per_view(num_tiles, backward, peers=False):
    """This library's kernel launches for one view: projection; the count
    phase (histogram, 4 depth passes, count scan); the sort phase (emit,
    histogram when the tile sort has passes, the passes, ranges);
    compositing; in a training step the L1 loss (partial sums, total,
    gradient), compositing backward and projection backward; and with the
    peer exchange its three handshake kernels."""
    passes = sort_passes(num_tiles)
    forward = 1 + 6 + (2 + (1 + passes if passes else 0)) + 1
    return forward + (5 if backward else 0) + (3 if peers else 0)


def main():
    args = parse_args()
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime

        torch.distributed.init_process_group(
            "nccl" if args.impl == "b200" else "gloo",
            timeout=datetime.timedelta(seconds=120))
    if args.impl == "reference":
        run_reference(args, rank, world)
        if world > 1:
            torch.distributed.destroy_process_group()
        return
    torch.cuda.set_device(local_rank)
    device = torch.device("cuda", local_rank)
    from gaussian_splats_b200.graphs import CapturedStep
    from gaussian_splats_b200.losses import l1_loss
    from gaussian_splats_b200.rasterize import StageTimer, rasterize_batch, rasterize_outputs
    from gaussian_splats_b200.splats import GaussianSplat
    from gaussian_splats_b200 import view_parallel
    from gaussian_splats_b200.view_parallel import screen_exchange_pays
    from gaussian_splats_b200.view_parallel import train_step as vp_train_step

    workload = WORKLOADS[args.config]
    backward = workload["backward"]
    scene = load_scene(args.config, args.points)
    views = views_for_rank(scene, args.config, rank, world)
    cameras = [camera for camera, _ in views]
    views_per_step = world * len(views) if workload["views"] is None else workload["views"]
    crop_w, crop_h = scene.crop
    host = [t.contiguous() for t in scene.tensors()]
    params = [t.to(device) for t in host]
    splats = GaussianSplat.from_tensors(*params)
    for p in splats.parameters():
        p.requires_grad_(backward and p is not splats.normals)
    # Cameras stay on the host: each 3x3 matrix is built there once per render
    # and uploaded (48 bytes), instead of ~15 tiny device kernels.
    targets_cpu = [target for _, target in views]
    targets = [t.to(device) if t is not None else None for t in targets_cpu]
    trainable = [splats.mean, splats.rotation, splats.scale, splats.opacity, splats.color]
    settings = scene.settings

    def render(s, camera):
        return rasterize_outputs(s, camera, settings.tile_size, settings.opacity_threshold,
                                 settings.near, settings.far)

    def loss_fn(image, target):
        # (image[:crop_h, :crop_w] - target).abs().mean(), fused
        return l1_loss(image, target)

    def forward_step(s=splats):
        with torch.no_grad():
            return [render(s, camera)[0] for camera in cameras]

    # Forward-only multi-camera configs render through the batched op, 16
    # cameras per call (one projection launch and one host wait per call).
    batched = not backward and workload["views"] is not None

    def batched_step(s=splats):
        images = []
        for first in range(0, len(cameras), BATCH_VIEWS):
            images += [out[0] for out in rasterize_batch(
                s, cameras[first:first + BATCH_VIEWS], settings.tile_size,
                settings.opacity_threshold, settings.near, settings.far)]
        return images

    # One view per rank: the ranks can exchange screen-space gradients, each
    # summing the projection backward over all views (view_parallel), where
    # that beats all-reducing the parameter gradients; several views per rank:
    # the parameter gradients are all-reduced once per step.
    screen = world > 1 and len(cameras) == 1 and (
        args.exchange in ("screen", "screen-nccl") or
        (args.exchange == "auto" and screen_exchange_pays(world)))
    # screen-space gradients read from peer memory (default) or all-gathered by NCCL
    view_parallel.EXCHANGE_TRANSPORT = "nccl" if args.exchange == "screen-nccl" else "p2p"
    peers = screen and view_parallel.EXCHANGE_TRANSPORT == "p2p"

    def train_step():
        return vp_train_step(splats, cameras, targets, trainable,
                             lambda s, c: render(s, c)[0], loss_fn, screen_exchange=screen)

    step = train_step if backward else (batched_step if batched else forward_step)

    def timed(fn, steps):
        if world > 1:
            torch.distributed.barrier()
        torch.cuda.synchronize()
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record()
        for _ in range(steps):
            fn()
        end.record()
        torch.cuda.synchronize()
        if world > 1:
            torch.distributed.barrier()
        ms = start.elapsed_time(end) / steps
        if world > 1:
            t = torch.tensor([ms], device=device)
            torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
            ms = float(t)
        return ms

    # Forward only.
    for _ in range(args.warmup):
        forward_step()
    fwd_ms = timed(forward_step, args.steps)

    # The headline step: forward + backward (+ the gradient exchange), or
    # forward only. The training step is replayed from a CUDA graph
    # (gaussian_splats_b200.graphs: one launch per step, the same kernels) on
    # one GPU, and on several when the ranks exchange through peer memory; the
    # per-stage times come from steps launched from Python, which the stage
    # timer's events need. A step with an NCCL collective is launched from
    # Python: no collective is captured into a graph.
    for _ in range(args.warmup):
        step()
    graphed = backward and not args.no_graph and (world == 1 or peers)
    eager_ms = None
    if graphed:
        with StageTimer() as stages:
            eager_ms = timed(step, max(3, args.steps // 5))
        stage_ms = stages.durations()
        captured = CapturedStep(step, warmup=max(1, args.warmup))
        for _ in range(args.warmup):
            captured()
        with ClockSampler(local_rank) as clocks:
            ms = timed(captured, args.steps)
        if not captured.check():
            raise RuntimeError("a timed replay overflowed its intersection buffer")
        if peers:
            view_parallel.check_exchange()
    else:
        with ClockSampler(local_rank) as clocks, StageTimer() as stages:
            ms = timed(step, args.steps)
        stage_ms = stages.durations()
    clock = clocks.summary()
    value = views_per_step * 1000.0 / ms

    # Structure of this rank's first view (for the roofline's work counts).
    camera0 = cameras[0]
    with torch.no_grad():
        out = render(splats, camera0)
        n_contrib = int(out[2].sum())
        intersections = int(out[7].numel())
        visible = int((out[9] > 0).sum())
        # Pairs the reference's compositing kernels evaluate: every pixel of a
        # tile for every list entry up to the tile's largest contributor count
        # (composite.py:148-188, composite_bwd.py:81-93).
        ts = settings.tile_size
        nc = out[2].reshape(out[2].shape[0] // ts, ts, out[2].shape[1] // ts, ts)
        tile_max = nc.permute(0, 2, 1, 3).reshape(-1, ts * ts).amax(dim=1).long()
        lengths = out[8][:, 1] - out[8][:, 0]
        num_tiles = int(lengths.numel())
        pairs = int((torch.minimum(lengths, tile_max) * ts * ts).sum())
        grad_image = None
        if backward:
            grad_image = torch.zeros_like(out[0])
            diff = out[0][:crop_h, :crop_w] - targets[0]
            grad_image[:crop_h, :crop_w] = torch.sign(diff) / diff.numel()
    kernel_ms = kernel_durations(out, params, camera0, grad_image, settings, device)
    fp32_peak = fp32_peak_tflops(device)
    optimizer_ms = None
    if backward:
        train_step()  # leaves this rank's summed, all-reduced gradients in .grad
        optimizer_ms = optimizer_timings(trainable, [p.grad for p in trainable], device)
        relocation_ms = relocation_timings(trainable, device)

    # End to end through the public API with host buffers: each step copies the
    # Gaussian parameters and this rank's targets from pinned host memory,
    # renders, and reads the result back (the loss, or for forward-only
    # configs one sum per image). Inputs are double-buffered: the copy of step
    # i+1 runs on a copy stream while step i computes (the buffer it
    # overwrites was last read by step i-1, which the read-back has already
    # waited for), so the step time is max(copy, compute).
    pinned = [t.pin_memory() for t in host] + \
        [t.pin_memory() for t in targets_cpu if t is not None]
    h2d = sum(t.numel() * t.element_size() for t in pinned)
    d2h = 4 if backward else 4 * len(cameras)
    copy_stream = torch.cuda.Stream(device)
    slots = []
    for _ in range(2):
        buffers = [torch.empty_like(t, device=device) for t in pinned]
        slot_splats = GaussianSplat.from_tensors(*buffers[:5])
        slot_trainable = [slot_splats.mean, slot_splats.rotation, slot_splats.scale,
                          slot_splats.opacity, slot_splats.color]
        for p in slot_trainable:
            p.requires_grad_(backward)
        slots.append((buffers, slot_splats, slot_trainable, torch.cuda.Event()))

    def prefetch(i):
        buffers, _, _, ready = slots[i % 2]
        with torch.no_grad(), torch.cuda.stream(copy_stream):
            for dst, src in zip(buffers, pinned):
                dst.copy_(src, non_blocking=True)
            ready.record(copy_stream)

    def slot_step(slot):
        buffers, slot_splats, slot_trainable, _ = slot
        return lambda: vp_train_step(slot_splats, cameras, buffers[5:], slot_trainable,
                                     lambda s, c: render(s, c)[0], loss_fn,
                                     screen_exchange=screen)

    slot_steps = [slot_step(slot) for slot in slots]
    if graphed:
        # one captured step per buffer slot, captured on real inputs
        prefetch(0)
        prefetch(1)
        torch.cuda.synchronize()
        slot_steps = [CapturedStep(fn, warmup=1) for fn in slot_steps]

    def e2e_run(steps):
        prefetch(0)
        for i in range(steps):
            if i + 1 < steps:
                prefetch(i + 1)
            buffers, slot_splats, slot_trainable, ready = slots[i % 2]
            torch.cuda.current_stream().wait_event(ready)
            if backward:
                loss = slot_steps[i % 2]()
                loss.item()
            else:
                images = (batched_step if batched else forward_step)(slot_splats)
                torch.stack([image.sum() for image in images]).cpu()

    e2e_run(max(1, args.warmup // 2))
    e2e_steps = max(3, args.steps // 2)
    e2e_ms = timed(lambda: e2e_run(e2e_steps), 1) / e2e_steps
    if graphed and not all(fn.check() for fn in slot_steps):
        raise RuntimeError("an end-to-end replay overflowed its intersection buffer")
    if peers:
        view_parallel.check_exchange()

    hbm_peak, peak_kind = load_peaks()
    n, k = scene.num_points, host[4].shape[1]
    traffic = {}
    profile_json = os.path.join(ROOT, "profiles", "traffic.json")
    if args.config == 2 and args.points is None and os.path.exists(profile_json):
        with open(profile_json) as f:
            traffic = json.load(f)

    def hbm(name, bytes_per_launch):
        gbs = bytes_per_launch / (kernel_ms[name] * 1e-3) / 1e9
        return {"bound": "hbm", "achieved": gbs, "peak": hbm_peak, "unit": "GB/s",
                "frac": gbs / hbm_peak, "traffic": traffic.get(name), "ms": kernel_ms[name],
                "algorithmic_bytes": bytes_per_launch,
                "note": f"peak: {peak_kind} hbm_gbs (MEASURED_PEAKS.json)"}

    def fp32(name, flops):
        tflops = flops / (kernel_ms[name] * 1e-3) / 1e12
        return {"bound": "fp32", "achieved": tflops, "peak": fp32_peak, "unit": "TFLOP/s",
                "frac": tflops / fp32_peak, "traffic": traffic.get(name), "ms": kernel_ms[name],
                "algorithmic_flops": flops,
                "note": "peak: FP32 cuBLAS SGEMM measured in this run (no FP32 figure in "
                        "MEASURED_PEAKS.json); work = reference-evaluated pairs x ops/pair"}

    rooflines = {
        "project_fwd": hbm("project_fwd", n * project_fwd_bytes(k)),
        "composite_fwd": fp32("composite_fwd", pairs * COMPOSITE_FWD_FLOPS),
    }
    if backward:
        rooflines["project_bwd"] = hbm("project_bwd", n * project_bwd_bytes(k))
        rooflines["composite_bwd"] = fp32("composite_bwd", pairs * COMPOSITE_BWD_FLOPS)
    dominant = max(kernel_ms, key=kernel_ms.get)
    main_roof = dict(rooflines[dominant], kernel=dominant)
    optimizer = None
    if optimizer_ms is not None:
        gbs = n * optimizer_bytes(k) / (optimizer_ms["fused"] * 1e-3) / 1e9
        optimizer = {
            "fused_ms": optimizer_ms["fused"], "torch_adam_and_noise_ms": optimizer_ms["torch"],
            "roofline": {"bound": "hbm", "achieved": gbs, "peak": hbm_peak, "unit": "GB/s",
                         "frac": gbs / hbm_peak, "algorithmic_bytes": n * optimizer_bytes(k),
                         "note": f"peak: {peak_kind} hbm_gbs (MEASURED_PEAKS.json)"},
            "relocation": {
                "fused_ms": relocation_ms["fused"], "torch_ms": relocation_ms["torch"],
                "dead_rows": relocation_ms["dead_rows"],
                "note": "relocate_splats at density 1.0 (dead rows replaced, moments reset), "
                        "FusedAdam state; torch = the reference's tensor ops; every 100 steps "
                        "in the reference's loop"},
            "note": "one training-loop optimizer step (Adam over the five parameter groups + "
                    "position noise), not part of the timed fwd+bwd step"}
    per_view = len(cameras)

    line = {
        "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms, "fwd_ms": fwd_ms / per_view,
        "batched_fwd_ms": ms / per_view if batched else None,
        "fwd_bwd_ms": ms / per_view if backward else None,
        "eager_ms_per_step": eager_ms,
        "higher_is_better": True,
        "scaling": "weak" if workload["views"] is None else "strong",
        "vs_baseline": None, "dtype": "f32",
        "data": f"synthetic (seeded config-{args.config} scene"
                + (", random L1 target)" if backward else ")"),
        "config": {"workload": workload["name"], "gaussians": n,
                   "image": [crop_w, crop_h], "tile_size": settings.tile_size,
                   "views_per_step": views_per_step, "views_per_rank_per_step": per_view,
                   "parallelism": (f"view-parallel x{world}" + (
                       (", projection backward summed over all ranks' views, reading their "
                        "screen-space gradients from peer memory (symmetric memory, NVLink)"
                        if peers else
                        ", NCCL all-gather of screen-space gradients + projection backward "
                        "summed over all ranks' views" if screen else
                        ", NCCL all-reduce of gradients") if backward else ", no collective"))
                   if world > 1 else "single GPU",
                   "step": "CUDA-graph replay of the captured training step (same kernels; "
                           "eager_ms_per_step is the step launched from Python)" if graphed
                   else "launched from Python",
                   "l2": "inputs larger than L2 (Gaussian parameters read every view)"
                   if n * project_fwd_bytes(k) > 126e6 else
                   "inputs smaller than L2; each view re-reads them"},
        "stage_ms": stage_ms, "kernel_ms": kernel_ms, "dominant_kernel": dominant,
        "view": {"visible": visible, "intersections": intersections, "tiles": num_tiles,
                 "active_pairs": n_contrib, "reference_pairs": pairs},
        "roofline": main_roof, "rooflines": rooflines, "optimizer": optimizer,
        "e2e": {"value": views_per_step * 1000.0 / e2e_ms, "unit": UNIT, "ms_per_step": e2e_ms,
                "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h},
        "gpu_launches": (launches_per_view(num_tiles, backward, peers) * per_view
                         if not batched else
                         (launches_per_view(num_tiles, False) - 1) * per_view
                         + -(-per_view // BATCH_VIEWS)) * args.steps,
        "clocks": clock,
    }
    if world == 1 and rank == 0 and not args.no_cpu_baseline:
        sys.path.insert(0, os.path.join(ROOT, "oracle"))
        import oracle as O

        view = cpu_view_setup(O, load_scene(args.config, args.points), backward)
        seconds, sample = cpu_view_seconds(O, view, chunk=scene.num_points, tiles=256, seed=0)
        line["cpu_baseline"] = {"value": 1.0 / seconds, "unit": UNIT,
                                "cores": os.cpu_count(), "kind": "port", "sample": sample}
    if rank == 0:
        print(json.dumps(line), flush=True)
    if world > 1:
        torch.distributed.destroy_process_group()


if __name__ == "__main__":
    main()
