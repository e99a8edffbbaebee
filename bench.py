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


# Binning's bytes in this build, each array read or written once: the count
# phase reads counts and depths (8 B per Gaussian) and moves 16 B per visible
# Gaussian in each of its 4 depth passes; the row pass reads each visible
# Gaussian's id and rectangle twice (40 B) and writes 4 B per row segment;
# the column pass reads each segment and its column span twice (24 B) and
# writes 4 B per intersection; the ranges are 16 B per tile.
def binning_bytes(n, visible, segments, intersections, tiles):
    return 8 * n + 104 * visible + 28 * segments + 4 * intersections + 16 * tiles


# The reference's binning (intersections.py:10-88): per Gaussian its bounds,
# depth and count (32 B); per intersection a 12-byte emit and a 64-bit key +
# 32-bit id radix sort (6 passes x 24 B) plus the 8-byte range read.
REF_BIN_BYTES_PER_GAUSSIAN = 32
REF_BIN_BYTES_PER_INTERSECTION = 164


# The projection also writes each visible Gaussian's 64-byte compositing
# record (the compositors' staged form).
RECORD_BYTES = 64
PROJECT_FWD_BYTES = project_fwd_bytes(16)
PROJECT_BWD_BYTES = project_bwd_bytes(16)
# Per evaluated (pixel, Gaussian) pair, the reference's forward arithmetic
# (composite.py:159-186): offsets 2, distance 9, exp argument 1, exp 13 (the
# FP32 operations of the deterministic exp: range reduction 5, degree-7
# polynomial 8), alpha 4, activity test 3, weight 2, colour 6, transmittance 3.
COMPOSITE_FWD_FLOPS = 43
# Backward per evaluated pair (composite_bwd.py:101-195 without the dropped
# abs-gradient): distance and alpha 28 (exp 13 as above), T recovery 5, weight
# gradient 9, alpha/opacity/distance gradients 6, mean/conic gradients 14,
# colour 4, suffix update 10.
COMPOSITE_BWD_FLOPS = 76
# Warp schedulers per SM (one instruction issued per scheduler per cycle) and
# SMs of a B200: the issue roof of the compositors.
SCHEDULERS_PER_SM, SM_COUNT = 4, 148


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
    p.add_argument("--exchange", choices=("auto", "shard", "screen", "screen-nccl", "all-reduce"),
                   default="auto",
                   help="how ranks sum gradients with one view per rank: the sharded peer "
                        "exchange, the whole-gradient peer exchange, its NCCL all-gather form, "
                        "or the parameter-gradient all-reduce (auto: view_parallel's choice "
                        "for the world size)")
    return p.parse_args()


def load_peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        with open(path) as f:
            peaks = json.load(f)
        return float(peaks["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


class ClockSampler:
    """SM clock, power and throttle reasons of this rank's GPU, sampled every
    PERIOD_S while the timed region runs, through NVML (the library behind
    nvidia-smi) from a background thread. The timed loop spends its time in
    ``torch.cuda.synchronize()``, which releases the GIL, so a millisecond-scale
    period yields a few samples per millisecond of timed GPU work."""

    PERIOD_S = 0.001
    # NVML clock-event reason bits (nvml.h: nvmlClocksEventReason*)
    REASONS = {0x4: "sw_power_cap", 0x8: "hw_slowdown", 0x20: "sw_thermal_slowdown",
               0x40: "hw_thermal_slowdown"}

    def __init__(self, device_index):
        self.device_index = device_index
        self.samples = []
        self.thread = None
        self.max_mhz = None

    def _handle(self, nvml):
        uuid = str(torch.cuda.get_device_properties(self.device_index).uuid)
        for i in range(nvml.nvmlDeviceGetCount()):
            handle = nvml.nvmlDeviceGetHandleByIndex(i)
            name = nvml.nvmlDeviceGetUUID(handle)
            name = name.decode() if isinstance(name, bytes) else name
            if name.endswith(uuid):
                return handle
        return None

    def __enter__(self):
        import threading

        try:
            import pynvml as nvml

            nvml.nvmlInit()
            handle = self._handle(nvml)
        except Exception:  # no NVML: the line carries no clock record
            return self
        if handle is None:
            return self
        self.max_mhz = float(nvml.nvmlDeviceGetMaxClockInfo(handle, nvml.NVML_CLOCK_SM))
        reasons = getattr(nvml, "nvmlDeviceGetCurrentClocksEventReasons", None) or \
            nvml.nvmlDeviceGetCurrentClocksThrottleReasons
        self.stop = threading.Event()

        def sample():
            while not self.stop.is_set():
                self.samples.append((float(nvml.nvmlDeviceGetClockInfo(handle, nvml.NVML_CLOCK_SM)),
                                     int(reasons(handle)),
                                     nvml.nvmlDeviceGetPowerUsage(handle) / 1000.0))
                time.sleep(self.PERIOD_S)

        self.thread = threading.Thread(target=sample, daemon=True)
        self.thread.start()
        deadline = time.time() + 2.0
        while not self.samples and time.time() < deadline:
            time.sleep(self.PERIOD_S)
        self.samples.clear()  # keep what the timed region saw
        return self

    def __exit__(self, *exc):
        if self.thread is not None:
            self.stop.set()
            self.thread.join(timeout=5)

    def summary(self):
        if not self.samples:
            return None
        reasons = sorted({name for _, bits, _ in self.samples
                          for bit, name in self.REASONS.items() if bits & bit})
        return {"sm_mhz": statistics.median(mhz for mhz, _, _ in self.samples),
                "sm_max_mhz": self.max_mhz, "samples": len(self.samples),
                "power_w_max": max(w for _, _, w in self.samples), "reasons": reasons,
                "source": f"NVML every {self.PERIOD_S * 1e3:g} ms during the timed region"}


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


PARITY_RTOL, PARITY_ATOL = 1e-4, 1e-6  # the parameter-gradient tolerance of the contract


def gradient_parity(step, local_view, trainable, device):
    """Checks the multi-GPU step's summed gradients on every rank.

    ``step()`` runs the timed step (graph replay or Python launch, with its
    exchange: peer memory or all-reduce) and returns the summed parameter
    gradients it produced. The check recomputes them the plain way: this
    rank's views forward and backward with no exchange (``local_view``), then
    one NCCL all-reduce per parameter. Tolerance: |a - b| <= atol + rtol |b|
    elementwise. Returns the worst figures over ranks; every rank gets the
    same answer."""
    got = [g.detach().clone() for g in step()]
    torch.cuda.synchronize()
    local_view()
    for p in trainable:
        torch.distributed.all_reduce(p.grad)
    max_abs = ratio = max_rel = 0.0
    for a, p in zip(got, trainable):
        b = p.grad
        err = (a - b).abs()
        max_abs = max(max_abs, float(err.max()))
        ratio = max(ratio, float((err / (PARITY_ATOL + PARITY_RTOL * b.abs())).max()))
        beyond_atol = err > PARITY_ATOL
        if bool(beyond_atol.any()):
            max_rel = max(max_rel, float((err[beyond_atol] / b.abs()[beyond_atol]).max()))
    worst = torch.tensor([max_abs, ratio, max_rel], device=device)
    torch.distributed.all_reduce(worst, op=torch.distributed.ReduceOp.MAX)
    max_abs, ratio, max_rel = worst.tolist()
    return {"max_abs": max_abs, "max_rel": max_rel, "max_tol_ratio": ratio,
            "rtol": PARITY_RTOL, "atol": PARITY_ATOL, "ok": ratio <= 1.0,
            "against": "rank-local backward of each rank's views + NCCL all-reduce of the "
                       "parameter gradients"}


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
    # the compositors' records of this view (what the timed projection rewrites)
    records = torch.empty((n, 16), device=device)
    native.check(lib.gs_pack_records(n, P(pmean), P(conic), P(pcolor), P(popacity), pref,
                                     P(records), stream), "gs_pack_records")
    out_records = torch.empty_like(records)
    # the compositors' heavy-first tile orders, as the operator computes them per view
    fwd_order = torch.empty((ranges.shape[0],), dtype=torch.int32, device=device)
    order_work = torch.empty((ranges.shape[0] + 128,), dtype=torch.int32, device=device)
    native.check(lib.gs_tile_order(P(ranges), None, pref, P(fwd_order), P(order_work), stream),
                 "gs_tile_order")
    bwd_plan = torch.empty((lib.gs_composite_bwd_plan_size(pref),), dtype=torch.uint8,
                           device=device)
    if grad_image is not None:
        native.check(lib.gs_composite_bwd_plan(P(ranges), P(n_contrib), pref, 0, P(bwd_plan),
                                               bwd_plan.numel(), stream),
                     "gs_composite_bwd_plan")
    launches = {
        "project_fwd": lambda: lib.gs_project_fwd(
            n, k, P(mean), P(rotation), P(scale), P(opacity), P(color), P(cam_r), P(cam_t), pref,
            P(out_pm), P(out_conic), P(out_rgb), P(out_o), P(bounds), P(out_counts),
            P(out_records), stream),
        "composite_fwd": lambda: lib.gs_composite_fwd(
            P(records), P(ids), P(ranges), pref, P(out_img), P(out_t), P(out_nc), P(fwd_order),
            stream),
    }
    if grad_image is not None:
        launches["composite_bwd"] = lambda: lib.gs_composite_bwd(
            n, P(records), P(ids), P(ranges), P(grad_image), P(final_t), P(n_contrib), pref,
            P(grad_projected), P(bwd_plan), stream)
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


def host_cores():
    """Host CPU cores this process may run on."""
    try:
        return len(os.sched_getaffinity(0))
    except (AttributeError, OSError):
        return os.cpu_count() or 1


def workload_config(config, scene):
    """The ``config`` object of the JSON line: what the workload is, the same
    for both arms and every N (how a run executes it -- ranks, graphs,
    exchange -- is reported under ``run``)."""
    n = scene.num_points
    k = scene.color.shape[1]
    return {"workload": WORKLOADS[config]["name"], "gaussians": n,
            "image": list(scene.crop), "tile_size": scene.settings.tile_size,
            "l2": "inputs larger than L2 (Gaussian parameters read every view)"
            if n * project_fwd_bytes(k) > 126e6 else
            "inputs smaller than L2; each view re-reads them"}


class ReferenceView:
    """One whole view of a config through the CPU restatement of the
    reference (``oracle/``): projection, binning and compositing of the
    config's first camera and, for the training configs, the L1 loss gradient
    against that camera's target (the one rank 0 of the GPU arm uses),
    compositing backward and projection backward. Nothing is sampled or
    extrapolated: ``run()`` times the whole view."""

    def __init__(self, O, scene, config):
        self.O = O
        self.inputs, self.settings = O.scene_inputs(scene)
        self.backward = WORKLOADS[config]["backward"]
        self.crop = scene.crop
        self.target = None
        if self.backward:
            _, target = views_for_rank(scene, config, 0, 1)[0]
            self.target = target.numpy()
        self.what = ("projection, binning, compositing, L1 loss gradient, compositing backward, "
                     "projection backward" if self.backward else
                     "projection, binning, compositing")

    def run(self):
        O, s, inputs = self.O, self.settings, self.inputs
        t0 = time.perf_counter()
        fwd = O.rasterize(*(inputs[k] for k in REFERENCE_KEYS), s)
        if self.backward:
            width, height = self.crop
            diff = fwd["image"][:height, :width] - self.target
            grad_image = np.zeros_like(fwd["image"])
            grad_image[:height, :width] = np.sign(diff) / np.float32(diff.size)
            O.backward(inputs, fwd, grad_image, s)
        return time.perf_counter() - t0


REFERENCE_KEYS = ("mean", "rotation", "scale", "opacity", "color", "camera_rotation",
                  "camera_translation")


def load_oracle(threads):
    """The CPU restatement, its parallel loops set to ``threads`` host threads
    (explicitly: torchrun exports OMP_NUM_THREADS=1). Returns (module, threads
    in effect)."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle as O

    return O, O.set_threads(threads)


def run_reference(args, rank, world):
    """The reference's algorithm on this host's cores (rank 0 only; other
    ranks exit at once): W warm-up views, then K whole views timed back to
    back. value = K / seconds."""
    if rank != 0:
        return
    O, threads = load_oracle(host_cores())
    scene = load_scene(args.config, args.points)
    view = ReferenceView(O, scene, args.config)
    for _ in range(args.warmup):
        view.run()
    seconds = sum(view.run() for _ in range(args.steps))
    value = args.steps / seconds
    sample = (f"{args.steps} whole views of the config's first camera ({view.what}), "
              f"timed back to back after {args.warmup} warm-up views; nothing sampled or scaled")
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": seconds * 1e3 / args.steps,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": f"synthetic (seeded config-{args.config} scene"
                + (", random L1 target)" if view.backward else ")"),
        "config": workload_config(args.config, scene),
        "run": {"host": "CPU restatement of the reference's kernels (oracle/gs_oracle.c, "
                        "OpenMP)", "threads": threads, "ranks_working": 1},
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": threads, "kind": "port",
                         "sample": sample},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


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


CPU_BASELINE_VIEWS = 3  # whole views timed for the GPU arm's cpu_baseline

BATCH_VIEWS = 16  # cameras per rasterize_batch call in forward-only multi-camera configs


def sort_passes(num_tiles):
    """8-bit radix passes of the tile sort for `num_tiles` tiles."""
    bits = max(0, (max(1, num_tiles) - 1).bit_length())
    return (bits + 7) // 8


def launches_per_view(tiles_w, tiles_h, backward, peers=False, sharded=False):
    """This library's kernel launches for one view: projection; the count
    phase (histogram, 4 depth passes); the sort phase (the row/column path's
    count, scan and scatter of rows and of columns, plus its row layout; or,
    for grids over 256 tile columns or 512 rows, count scan, emit, histogram,
    tile-sort passes and ranges); the forward's tile order (count, scatter);
    compositing; in a training step the L1 loss (partial sums, total,
    gradient), the backward's plan (per-tile contributor maximum, count,
    scatter), compositing backward and projection backward; and with a peer
    exchange its handshake kernels (begin, publish, finish; the sharded form
    also its shard release)."""
    if tiles_w <= 256 and tiles_h <= 512:
        sort_phase = 7
    else:
        passes = sort_passes(tiles_w * tiles_h)
        sort_phase = 2 + (1 + passes if passes else 0) + 1
    forward = 1 + 5 + sort_phase + 2 + 1
    handshakes = 4 if sharded else (3 if peers else 0)
    return forward + (8 if backward else 0) + handshakes


def main():
    args = parse_args()
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        # host CPU work on rank 0 only: no process group, no collective
        run_reference(args, rank, world)
        return
    if world > 1:
        import datetime

        torch.distributed.init_process_group("nccl", timeout=datetime.timedelta(seconds=120))
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
    transport = {"screen": "p2p", "screen-nccl": "nccl", "shard": "p2p-shard"}.get(
        args.exchange, "auto")
    screen = world > 1 and len(cameras) == 1 and (
        args.exchange in ("shard", "screen", "screen-nccl") or
        (args.exchange == "auto" and screen_exchange_pays(world, transport)))
    view_parallel.EXCHANGE_TRANSPORT = transport
    if world > 1:
        transport = view_parallel.transport_for()
    peers = screen and transport in view_parallel.PEER_TRANSPORTS

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
        rank_ms[fn] = [ms]
        if world > 1:
            every = torch.zeros(world, device=device)
            every[rank] = ms
            torch.distributed.all_reduce(every)  # each rank's own time, for the record
            rank_ms[fn] = every.tolist()
            ms = max(rank_ms[fn])
        return ms

    rank_ms = {}

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
        # the gradient tensors the graph writes on every replay (bound to .grad
        # during capture; later eager steps rebind .grad to other tensors)
        step_grads = [p.grad for p in trainable]
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
    headline_rank_ms = rank_ms[captured if graphed else step]
    parity = None
    rank_view_ms = None
    if world > 1 and backward:
        # Each rank's own view, forward + backward without any exchange
        # (launched from Python): how much of the multi-GPU step is camera
        # imbalance rather than exchange cost.
        def local_view():
            for p in trainable:
                p.grad = None
            for camera, target in zip(cameras, targets):
                loss_fn(render(splats, camera)[0], target).backward()

        for _ in range(2):
            local_view()
        timed(local_view, 5)
        rank_view_ms = rank_ms[local_view]
        if graphed:
            def replay():
                captured()
                return step_grads
        else:
            def replay():
                step()
                return [p.grad for p in trainable]
        parity = gradient_parity(replay, local_view, trainable, device)

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
        # Row segments (one per tile row a Gaussian's rectangle spans): the
        # distinct (tile row, Gaussian) pairs of the lists.
        tiles_w = out[2].shape[1] // ts
        entry_row = torch.repeat_interleave(
            torch.arange(num_tiles, device=lengths.device) // tiles_w, lengths)
        segments = int(torch.unique((entry_row << 32) | out[7][:intersections].long()).numel())
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

    pipes = {}
    pipes_json = os.path.join(ROOT, "profiles", "pipes.json")
    if args.config == 2 and args.points is None and os.path.exists(pipes_json):
        with open(pipes_json) as f:
            pipes = json.load(f)
    clock_mhz = (clock or {}).get("sm_mhz") or 1965.0

    def issue(name, flops):
        """The compositors are bound by instruction issue (no tensor work, DRAM
        a few % busy): achieved = warp instructions per launch (counted by ncu
        on this workload) / live launch time, against one instruction per
        scheduler per cycle at the clock measured during the timed region.
        The reference-work FP32 rate is kept beside it, labelled by its basis."""
        tflops = flops / (kernel_ms[name] * 1e-3) / 1e12
        work = {"basis": "reference-evaluated (pixel, Gaussian) pairs x FP32 ops per pair of the "
                         "reference's arithmetic: a rate of reference work, not pipe "
                         "utilisation (the kernel culls pairs the reference evaluates)",
                "achieved": tflops, "unit": "TFLOP/s", "fp32_sgemm_peak": fp32_peak,
                "vs_sgemm": tflops / fp32_peak, "algorithmic_flops": flops}
        entry = {"bound": "issue", "achieved": None, "peak": None, "unit": "Ginst/s",
                 "frac": None, "traffic": traffic.get(name), "ms": kernel_ms[name],
                 "reference_work": work}
        counters = pipes.get(name)
        if counters:
            inst = counters["inst_executed"]
            achieved = inst / (kernel_ms[name] * 1e-3) / 1e9
            peak = SCHEDULERS_PER_SM * SM_COUNT * clock_mhz * 1e6 / 1e9
            entry.update(
                achieved=achieved, peak=peak, frac=achieved / peak,
                inst_executed=inst, fma_pipe_pct=counters["fma_pipe_pct"],
                alu_pipe_pct=counters["alu_pipe_pct"],
                threads_per_warp_inst=counters["threads_per_warp_inst"],
                warp_inst_per_active_pair=inst / max(1, n_contrib),
                thread_inst_per_active_pair=inst * counters["threads_per_warp_inst"]
                / max(1, n_contrib),
                note="warp instructions from ncu (profiles/pipes.json, same workload); time "
                     "live (CUDA events, L2 flushed); peak = 4 schedulers x 148 SMs x the "
                     "median SM clock of the timed region")
        return entry

    rooflines = {
        "project_fwd": hbm("project_fwd", n * project_fwd_bytes(k) + visible * RECORD_BYTES),
        "composite_fwd": issue("composite_fwd", pairs * COMPOSITE_FWD_FLOPS),
    }
    if "bin_count" in stage_ms and "bin_sort" in stage_ms:
        # Binning, count and sort phases together (live stage times of the
        # eager steps): this build's bytes against HBM, and the reference's
        # emit + 64-bit key sort bytes as a rate of reference work.
        bin_ms = stage_ms["bin_count"] + stage_ms["bin_sort"]
        own = binning_bytes(n, visible, segments, intersections, num_tiles)
        gbs = own / (bin_ms * 1e-3) / 1e9
        ref = REF_BIN_BYTES_PER_GAUSSIAN * n + REF_BIN_BYTES_PER_INTERSECTION * intersections
        rooflines["binning"] = {
            "bound": "latency", "achieved": gbs, "peak": hbm_peak, "unit": "GB/s",
            "frac": gbs / hbm_peak, "ms": bin_ms, "algorithmic_bytes": own,
            "segments": segments,
            "reference_work": {"basis": "the reference's emit of 64-bit keys and their 6-pass "
                                        "radix sort: 32 B per Gaussian + 164 B per intersection",
                               "bytes": ref, "achieved": ref / (bin_ms * 1e-3) / 1e9,
                               "unit": "GB/s"},
            "note": "count + sort phases (5 + 7 launches, latency-bound: their bytes are few); "
                    f"peak: {peak_kind} hbm_gbs (MEASURED_PEAKS.json)"}
    if backward:
        rooflines["project_bwd"] = hbm("project_bwd", n * project_bwd_bytes(k))
        rooflines["composite_bwd"] = issue("composite_bwd", pairs * COMPOSITE_BWD_FLOPS)
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
        "config": workload_config(args.config, scene),
        "run": {"views_per_step": views_per_step, "views_per_rank_per_step": per_view,
                "parallelism": (f"view-parallel x{world}" + (
                    (", sharded peer exchange: each rank copies its shard's screen-space "
                     "gradient rows from every rank (symmetric memory, NVLink), sums the "
                     "projection backward of its shard over all ranks' views, and copies the "
                     "other shards' parameter gradients" if transport == "p2p-shard" and peers
                     else ", projection backward summed over all ranks' views, reading their "
                     "screen-space gradients from peer memory (symmetric memory, NVLink)"
                     if peers else
                     ", NCCL all-gather of screen-space gradients + projection backward "
                     "summed over all ranks' views" if screen else
                     ", NCCL all-reduce of gradients") if backward else ", no collective"))
                if world > 1 else "single GPU",
                "step": "CUDA-graph replay of the captured training step (same kernels; "
                        "eager_ms_per_step is the step launched from Python)" if graphed
                else "launched from Python"},
        "stage_ms": stage_ms, "kernel_ms": kernel_ms, "dominant_kernel": dominant,
        "view": {"visible": visible, "intersections": intersections, "tiles": num_tiles,
                 "segments": segments, "active_pairs": n_contrib, "reference_pairs": pairs},
        "roofline": main_roof, "rooflines": rooflines, "optimizer": optimizer,
        "e2e": {"value": views_per_step * 1000.0 / e2e_ms, "unit": UNIT, "ms_per_step": e2e_ms,
                "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h},
        "gpu_launches": (launches_per_view(tiles_w, num_tiles // tiles_w, backward, peers,
                                           peers and transport == "p2p-shard") * per_view
                         if not batched else
                         (launches_per_view(tiles_w, num_tiles // tiles_w, False) - 1) * per_view
                         + -(-per_view // BATCH_VIEWS)) * args.steps,
        "clocks": clock,
        "rank_ms_per_step": headline_rank_ms,
        "rank_view_ms": rank_view_ms,
        "parity": parity,
    }
    if world == 1 and rank == 0 and not args.no_cpu_baseline:
        O, threads = load_oracle(host_cores())
        cpu_view = ReferenceView(O, load_scene(args.config, args.points), args.config)
        cpu_view.run()  # warm-up
        cpu_s = [cpu_view.run() for _ in range(CPU_BASELINE_VIEWS)]
        line["cpu_baseline"] = {
            "value": CPU_BASELINE_VIEWS / sum(cpu_s), "unit": UNIT, "cores": threads,
            "kind": "port",
            "sample": f"{CPU_BASELINE_VIEWS} whole views of the config's first camera "
                      f"({cpu_view.what}) after one warm-up view, CPU restatement of the "
                      f"reference's kernels on {threads} host threads"}
    if rank == 0:
        print(json.dumps(line), flush=True)
    if world > 1:
        view_parallel.release_arenas()
        torch.distributed.destroy_process_group()
    if parity is not None and not parity["ok"]:
        sys.exit(f"multi-GPU gradients outside rtol {PARITY_RTOL} / atol {PARITY_ATOL} of the "
                 f"plain all-reduce: {parity}")


if __name__ == "__main__":
    main()
