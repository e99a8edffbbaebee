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
WORKLOAD = "config2: 1M Gaussians SH3, 1920x1080 (rendered 1920x1088), 16x16 tiles, fwd+bwd L1"
# Algorithmic bytes per Gaussian (K = 16 SH coefficients): projection reads
# mean, rotation, scale, opacity (44 B) and colour (192 B) and writes
# projected mean, conic, colour, opacity, tile rectangle, count (64 B);
# projection backward reads the same parameters plus conic, the 9-float
# screen-space gradient and the count (56 B) and writes 236 B of gradients.
PROJECT_FWD_BYTES = 44 + 12 * 16 + 64
PROJECT_BWD_BYTES = 44 + 12 * 16 + 56 + 44 + 12 * 16
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
    p.add_argument("--points", type=int, default=1_000_000)
    p.add_argument("--no-cpu-baseline", action="store_true")
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
    """Per-launch milliseconds of the four main kernels, each launched through
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
    grads = [torch.empty_like(t) for t in params]
    launches = {
        "project_fwd": lambda: lib.gs_project_fwd(
            n, k, P(mean), P(rotation), P(scale), P(opacity), P(color), P(cam_r), P(cam_t), pref,
            P(out_pm), P(out_conic), P(out_rgb), P(out_o), P(bounds), P(out_counts), stream),
        "composite_fwd": lambda: lib.gs_composite_fwd(
            P(pmean), P(conic), P(pcolor), P(popacity), P(ids), P(ranges), pref, P(out_img),
            P(out_t), P(out_nc), stream),
        "composite_bwd": lambda: lib.gs_composite_bwd(
            n, P(pmean), P(conic), P(pcolor), P(popacity), P(ids), P(ranges), P(grad_image),
            P(final_t), P(n_contrib), pref, P(grad_projected), stream),
        "project_bwd": lambda: lib.gs_project_bwd(
            n, k, P(mean), P(rotation), P(scale), P(opacity), P(color), P(cam_r), P(cam_t),
            P(conic), P(grad_projected), P(counts), pref, *(P(g) for g in grads), stream),
    }
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


def make_view(scene, rank):
    """Rank 0 renders config 2's camera; other ranks a camera from the same
    recipe (radius 5, random direction) seeded by rank."""
    from gaussian_splats_b200 import scenes

    if rank == 0:
        return scene.cameras[0], scene.targets[0]
    g = torch.Generator().manual_seed(1000 + rank)
    cam = scenes.look_at_camera(5.0 * scenes.random_direction(g), fovy_degrees=50.0,
                                width=1920, height=1080)
    return cam, torch.rand(1080, 1920, 3, generator=g)


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

    from gaussian_splats_b200 import scenes

    scene = scenes.config2(num_points=args.points)
    cores = os.cpu_count() or 1
    os.environ.setdefault("OMP_NUM_THREADS", str(cores))
    chunk, tiles = sample_size(args.steps, args.warmup, scene.num_points)
    view = cpu_view_setup(O, scene)
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
        "data": "synthetic", "config": {"workload": WORKLOAD},
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": cores, "kind": "port",
                         "sample": sample},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def cpu_view_setup(O, scene):
    """The whole view's projection and binning, which the sampled compositing
    steps read, and the per-view fixed cost of the compositing calls (image
    buffers; in the backward the [intersections, 9] row buffer and its
    reduction per Gaussian), timed once with an empty tile list."""
    inputs, s = O.scene_inputs(scene)
    keys = ("mean", "rotation", "scale", "opacity", "color", "camera_rotation",
            "camera_translation")
    proj = O.project(*(inputs[k] for k in keys), s)
    binned = O.bin(proj["bounds"], proj["projected_mean"][:, 2], proj["counts"], s)
    grad_image = np.full((s.height, s.width, 3), 1.0 / (1920 * 1080 * 3), np.float32)
    view = {"scene": scene, "inputs": inputs, "settings": s, "keys": keys, "proj": proj,
            "binned": binned, "grad_image": grad_image}
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
    sample = (f"one config-2 view: projection, binning, projection backward of {chunk} of "
              f"{n} Gaussians scaled by {gaussian_scale:.2f}; composite fwd+bwd on "
              f"{len(chosen)} of {s.num_tiles} random tiles, per-tile time scaled by "
              f"{tile_scale:.1f} (all list entries / sampled entries), per-view fixed "
              f"time ({fixed:.2f} s) counted once")
    return seconds, sample


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
    from gaussian_splats_b200 import scenes
    from gaussian_splats_b200.rasterize import StageTimer, rasterize_outputs
    from gaussian_splats_b200.splats import GaussianSplat
    from gaussian_splats_b200.view_parallel import train_step as vp_train_step

    scene = scenes.config2(num_points=args.points)
    camera, target_cpu = make_view(scene, rank)
    crop_w, crop_h = scene.crop
    host = [t.contiguous() for t in scene.tensors()]
    params = [t.to(device) for t in host]
    splats = GaussianSplat.from_tensors(*params)
    for p in splats.parameters():
        p.requires_grad_(p is not splats.normals)
    # The camera stays on the host: its 3x3 matrix is built there once per
    # render and uploaded (48 bytes), instead of ~15 tiny device kernels.
    target = target_cpu.to(device)
    trainable = [splats.mean, splats.rotation, splats.scale, splats.opacity, splats.color]
    settings = scene.settings

    def render(s):
        return rasterize_outputs(s, camera, settings.tile_size, settings.opacity_threshold,
                                 settings.near, settings.far)

    def train_step():
        # One view per rank; the gradients are summed over ranks with one
        # all-reduce per parameter tensor (view_parallel.train_step).
        return vp_train_step(splats, [camera], [target], trainable,
                             lambda s, c: render(s)[0],
                             lambda image, t: (image[:crop_h, :crop_w] - t).abs().mean())

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
    with torch.no_grad():
        for _ in range(args.warmup):
            render(splats)
        fwd_ms = timed(lambda: render(splats), args.steps)

    # Forward + backward (+ all-reduce): the headline.
    for _ in range(args.warmup):
        train_step()
    with ClockSampler(local_rank) as clocks, StageTimer() as stages:
        ms = timed(train_step, args.steps)
    stage_ms = stages.durations()
    clock = clocks.summary()
    value = world * 1000.0 / ms

    # Structure of the view (for the roofline's work counts).
    with torch.no_grad():
        out = render(splats)
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
        pairs = int((torch.minimum(lengths, tile_max) * ts * ts).sum())
        grad_image = torch.zeros_like(out[0])
        diff = out[0][:crop_h, :crop_w] - target
        grad_image[:crop_h, :crop_w] = torch.sign(diff) / diff.numel()
    kernel_ms = kernel_durations(out, params, camera, grad_image, settings, device)
    fp32_peak = fp32_peak_tflops(device)

    # End to end through the public API with host buffers: each step copies the
    # Gaussian parameters and the target from pinned host memory, renders
    # forward + backward, and reads the loss back. Inputs are double-buffered:
    # the copy of step i+1 runs on a copy stream while step i computes (the
    # buffer it overwrites was last read by step i-1, which the loss read-back
    # has already waited for), so the step time is max(copy, compute).
    pinned = [t.pin_memory() for t in host] + [target_cpu.pin_memory()]
    h2d = sum(t.numel() * t.element_size() for t in pinned)
    copy_stream = torch.cuda.Stream(device)
    slots = []
    for _ in range(2):
        buffers = [torch.empty_like(p) for p in params] + [torch.empty_like(target)]
        slot_splats = GaussianSplat.from_tensors(*buffers[:5])
        slot_trainable = [slot_splats.mean, slot_splats.rotation, slot_splats.scale,
                          slot_splats.opacity, slot_splats.color]
        for p in slot_trainable:
            p.requires_grad_(True)
        slots.append((buffers, slot_splats, slot_trainable, torch.cuda.Event()))

    def prefetch(i):
        buffers, _, _, ready = slots[i % 2]
        with torch.no_grad(), torch.cuda.stream(copy_stream):
            for dst, src in zip(buffers, pinned):
                dst.copy_(src, non_blocking=True)
            ready.record(copy_stream)

    def e2e_run(steps):
        prefetch(0)
        for i in range(steps):
            if i + 1 < steps:
                prefetch(i + 1)
            buffers, slot_splats, slot_trainable, ready = slots[i % 2]
            torch.cuda.current_stream().wait_event(ready)
            loss = vp_train_step(slot_splats, [camera], [buffers[-1]], slot_trainable,
                                 lambda s, c: render(s)[0],
                                 lambda image, t: (image[:crop_h, :crop_w] - t).abs().mean())
            loss.item()

    e2e_run(max(1, args.warmup // 2))
    e2e_steps = max(3, args.steps // 2)
    e2e_ms = timed(lambda: e2e_run(e2e_steps), 1) / e2e_steps

    hbm_peak, peak_kind = load_peaks()
    launches_per_step = 15  # 1 projection, 6 count-phase, 5 sort-phase, 2 composite, 1 proj bwd
    n = scene.num_points
    traffic = {}
    profile_json = os.path.join(ROOT, "profiles", "traffic.json")
    if os.path.exists(profile_json):
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
        "project_fwd": hbm("project_fwd", n * PROJECT_FWD_BYTES),
        "project_bwd": hbm("project_bwd", n * PROJECT_BWD_BYTES),
        "composite_fwd": fp32("composite_fwd", pairs * COMPOSITE_FWD_FLOPS),
        "composite_bwd": fp32("composite_bwd", pairs * COMPOSITE_BWD_FLOPS),
    }
    dominant = max(kernel_ms, key=kernel_ms.get)
    main_roof = dict(rooflines[dominant], kernel=dominant)

    line = {
        "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms, "fwd_ms": fwd_ms, "fwd_bwd_ms": ms,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic (seeded config-2 scene, random L1 target)",
        "config": {"workload": WORKLOAD, "gaussians": n, "image": [1920, 1080],
                   "tile_size": settings.tile_size, "views_per_rank_per_step": 1,
                   "parallelism": f"view-parallel x{world}, NCCL all-reduce of gradients"
                   if world > 1 else "single GPU",
                   "l2": "inputs larger than L2 (236 MB of parameters read per step)"},
        "stage_ms": stage_ms, "kernel_ms": kernel_ms, "dominant_kernel": dominant,
        "view": {"visible": visible, "intersections": intersections,
                 "active_pairs": n_contrib, "reference_pairs": pairs},
        "roofline": main_roof, "rooflines": rooflines,
        "e2e": {"value": world * 1000.0 / e2e_ms, "unit": UNIT, "ms_per_step": e2e_ms,
                "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": 4},
        "gpu_launches": launches_per_step * args.steps,
        "clocks": clock,
    }
    if world == 1 and rank == 0 and not args.no_cpu_baseline:
        sys.path.insert(0, os.path.join(ROOT, "oracle"))
        import oracle as O

        cpu_scene = scenes.config2(num_points=args.points)
        view = cpu_view_setup(O, cpu_scene)
        seconds, sample = cpu_view_seconds(O, view, chunk=cpu_scene.num_points, tiles=256,
                                           seed=0)
        line["cpu_baseline"] = {"value": 1.0 / seconds, "unit": UNIT,
                                "cores": os.cpu_count(), "kind": "port", "sample": sample}
    if rank == 0:
        print(json.dumps(line), flush=True)
    if world > 1:
        torch.distributed.destroy_process_group()


if __name__ == "__main__":
    main()
