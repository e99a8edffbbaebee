"""Python driver for the CPU oracle -- TEST INFRASTRUCTURE ONLY.

Loads ``oracle/_build/libgs_oracle.so`` (built from ``gs_oracle.c`` by
``oracle/Makefile``) and exposes the reference rasterizer's stages on numpy
arrays. Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU
baseline use this module; the product never imports it.

Scalar folding follows the reference: ``lim_x``/``lim_y``, the ellipsoid
extent and cutoff are computed in Python double and rounded to float32 where
the kernels consume them (project.py:158-159,308; composite.py:226;
project_bwd.py:376-377).
"""

from __future__ import annotations

import ctypes
import math
import os
import subprocess
from dataclasses import dataclass

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIBRARY = os.path.join(HERE, "_build", "libgs_oracle.so")

_f32p = np.ctypeslib.ndpointer(dtype=np.float32, flags="C_CONTIGUOUS")
_i32p = np.ctypeslib.ndpointer(dtype=np.int32, flags="C_CONTIGUOUS")
_i64p = np.ctypeslib.ndpointer(dtype=np.int64, flags="C_CONTIGUOUS")


class Params(ctypes.Structure):
    _fields_ = [
        ("fx", ctypes.c_float), ("fy", ctypes.c_float), ("cx", ctypes.c_float),
        ("cy", ctypes.c_float), ("width", ctypes.c_int32), ("height", ctypes.c_int32),
        ("tile_size", ctypes.c_int32), ("gaussian_mode", ctypes.c_int32),
        ("near_plane", ctypes.c_float), ("far_plane", ctypes.c_float),
        ("lim_x", ctypes.c_float), ("lim_y", ctypes.c_float),
        ("bwd_lim_x", ctypes.c_float), ("bwd_lim_y", ctypes.c_float),
        ("extent", ctypes.c_float), ("cutoff", ctypes.c_float),
        ("opacity_threshold", ctypes.c_float),
    ]


def build() -> str:
    """Compile the oracle library if it is missing or older than its sources."""
    sources = [os.path.join(HERE, f) for f in ("gs_oracle.c", "detmath.h", "Makefile")]
    if not os.path.exists(LIBRARY) or os.path.getmtime(LIBRARY) < max(map(os.path.getmtime, sources)):
        subprocess.run(["make", "-s", "-C", HERE], check=True)
    return LIBRARY


_lib = None


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        _lib = ctypes.CDLL(build())
        P = ctypes.POINTER(Params)
        i64, i32 = ctypes.c_int64, ctypes.c_int32
        _lib.gso_project.argtypes = [i64, _f32p, _f32p, _f32p, _f32p, _f32p, i32, _f32p, _f32p, P,
                                     _f32p, _f32p, _f32p, _f32p, _i32p, _i32p]
        _lib.gso_set_threads.argtypes = [i32]
        _lib.gso_max_threads.restype = i32
        _lib.gso_total.argtypes = [i64, _i32p]
        _lib.gso_total.restype = i64
        _lib.gso_bin.argtypes = [i64, _i32p, _f32p, _i32p, i32, i32, ctypes.c_void_p,
                                 ctypes.c_void_p, _i32p, ctypes.c_void_p, _i64p]
        _lib.gso_composite.argtypes = [_f32p, _f32p, _f32p, _f32p, _i32p, _i64p, P,
                                       ctypes.c_void_p, i32, _f32p, _f32p, _i32p]
        _lib.gso_composite_bwd.argtypes = [i64, _f32p, _f32p, _f32p, _f32p, _i32p, _i64p, i64,
                                           _f32p, _f32p, _i32p, P, ctypes.c_void_p, i32, _f32p]
        _lib.gso_project_bwd.argtypes = [i64, _f32p, _f32p, _f32p, _f32p, _f32p, i32, _f32p, _f32p,
                                         _f32p, _f32p, _i32p, P, _f32p, _f32p, _f32p, _f32p,
                                         _f32p]
        ptr5 = ctypes.c_void_p * 5
        _lib.gso_adam_step.argtypes = [i64, i32, ptr5, ptr5, ptr5, ptr5,
                                       ctypes.POINTER(AdamParams), ctypes.c_void_p]
        _lib.gso_relocate.argtypes = [i64, i64, i32, ctypes.c_void_p, i64, ctypes.c_void_p, i64,
                                      _f32p, _f32p, _f32p, _f32p, _f32p, ctypes.c_void_p,
                                      ctypes.c_void_p * 10]
        _lib.gso_relocate.restype = ctypes.c_int
        _lib.gso_exp_array.argtypes = [i64, _f32p, _f32p]
        _lib.gso_log_array.argtypes = [i64, _f32p, _f32p]
    return _lib


class AdamParams(ctypes.Structure):
    """gso_adam_params: torch Adam's step scalars, folded as torch folds them."""
    _fields_ = [(name, ctypes.c_float) for name in
                ("lerp_weight", "beta2", "sq_weight", "eps")] + \
               [("neg_step_size", ctypes.c_float * 5), ("bias2_sqrt", ctypes.c_float * 5),
                ("noise_lr", ctypes.c_float), ("position_lr", ctypes.c_float)]


@dataclass
class Settings:
    fx: float
    fy: float
    cx: float
    cy: float
    width: int
    height: int
    tile_size: int = 16
    opacity_threshold: float = 0.999
    near: float = 0.2
    far: float = 100.0
    rendering_mode: str = "gaussian"
    confidence: float = 0.95

    @property
    def tiles_w(self) -> int:
        return self.width // self.tile_size

    @property
    def num_tiles(self) -> int:
        return (self.width // self.tile_size) * (self.height // self.tile_size)

    def params(self) -> Params:
        tiles_w = self.width // self.tile_size
        tiles_h = self.height // self.tile_size
        ellipsoid = self.rendering_mode == "ellipsoid"
        return Params(
            fx=self.fx, fy=self.fy, cx=self.cx, cy=self.cy,
            width=self.width, height=self.height, tile_size=self.tile_size,
            gaussian_mode=0 if ellipsoid else 1,
            near_plane=self.near, far_plane=self.far,
            lim_x=1.3 * tiles_w * self.tile_size / (2.0 * self.fx),
            lim_y=1.3 * tiles_h * self.tile_size / (2.0 * self.fy),
            bwd_lim_x=1.3 * self.width / (2.0 * self.fx),
            bwd_lim_y=1.3 * self.height / (2.0 * self.fy),
            extent=math.sqrt(-2 * math.log1p(-self.confidence)) if ellipsoid else 3.0,
            cutoff=-2.0 * math.log1p(-self.confidence),
            opacity_threshold=self.opacity_threshold,
        )


def set_threads(threads: int) -> int:
    """Run the parallel loops on ``threads`` host threads (whatever
    OMP_NUM_THREADS says); returns the thread count now in effect."""
    lib().gso_set_threads(int(threads))
    return int(lib().gso_max_threads())


def _c(a, dtype=np.float32):
    return np.ascontiguousarray(a, dtype=dtype)


def project(mean, rotation, scale, opacity, color, camera_rotation, camera_translation,
            s: Settings) -> dict:
    n = mean.shape[0]
    num_sh = color.shape[1]
    out = dict(
        projected_mean=np.empty((n, 3), np.float32),
        inverse_covariance=np.empty((n, 2, 2), np.float32),
        projected_color=np.empty((n, 3), np.float32),
        projected_opacity=np.empty((n, 1), np.float32),
        bounds=np.empty((n, 2, 2), np.int32),
        counts=np.empty((n,), np.int32),
    )
    p = s.params()
    lib().gso_project(n, _c(mean), _c(rotation), _c(scale), _c(opacity), _c(color), num_sh,
                      _c(camera_rotation), _c(camera_translation), ctypes.byref(p),
                      out["projected_mean"], out["inverse_covariance"], out["projected_color"],
                      out["projected_opacity"], out["bounds"], out["counts"])
    return out


def bin(bounds, depths, counts, s: Settings, with_keys: bool = False) -> dict:
    bounds, depths, counts = _c(bounds, np.int32), _c(depths), _c(counts, np.int32)
    n = counts.shape[0]
    total = lib().gso_total(n, counts)
    sorted_ids = np.empty((total,), np.int32)
    ranges = np.empty((s.num_tiles, 2), np.int64)
    keys = np.empty((total,), np.int64) if with_keys else None
    ids = np.empty((total,), np.int32) if with_keys else None
    sorted_keys = np.empty((total,), np.int64) if with_keys else None
    ptr = lambda a: a.ctypes.data if a is not None else None  # noqa: E731
    lib().gso_bin(n, bounds, depths, counts, s.tiles_w, s.num_tiles, ptr(keys), ptr(ids),
                  sorted_ids, ptr(sorted_keys), ranges)
    out = dict(gaussian_ids=sorted_ids, ranges=ranges)
    if with_keys:
        out.update(keys=keys, ids=ids, sorted_keys=sorted_keys)
    return out


def composite(projected_mean, inverse_covariance, projected_color, projected_opacity,
              gaussian_ids, ranges, s: Settings, tiles=None) -> dict:
    h, w = s.height, s.width
    image = np.zeros((h, w, 3), np.float32)
    final_t = np.ones((h, w), np.float32)
    n_contrib = np.zeros((h, w), np.int32)
    tiles_arr = None if tiles is None else _c(tiles, np.int32)
    p = s.params()
    lib().gso_composite(_c(projected_mean), _c(inverse_covariance), _c(projected_color),
                        _c(projected_opacity), _c(gaussian_ids, np.int32), _c(ranges, np.int64),
                        ctypes.byref(p), None if tiles_arr is None else tiles_arr.ctypes.data,
                        0 if tiles_arr is None else len(tiles_arr), image, final_t, n_contrib)
    return dict(image=image, final_transmittance=final_t, n_contributors=n_contrib)


def rasterize(mean, rotation, scale, opacity, color, camera_rotation, camera_translation,
              s: Settings) -> dict:
    """All ten outputs of the ``gaussian_splats::rasterize`` op, plus bounds."""
    out = project(mean, rotation, scale, opacity, color, camera_rotation, camera_translation, s)
    out.update(bin(out["bounds"], out["projected_mean"][:, 2], out["counts"], s))
    out.update(composite(out["projected_mean"], out["inverse_covariance"],
                         out["projected_color"], out["projected_opacity"],
                         out["gaussian_ids"], out["ranges"], s))
    return out


def composite_bwd(fwd: dict, grad_image, s: Settings, tiles=None) -> np.ndarray:
    """grad_projected [N, 9]. With ``tiles``, only those tiles are walked; the
    caller must pass a grad_image that is zero on every other tile."""
    n = fwd["projected_mean"].shape[0]
    grad = np.empty((n, 9), np.float32)
    p = s.params()
    tiles_arr = None if tiles is None else _c(tiles, np.int32)
    lib().gso_composite_bwd(n, _c(fwd["projected_mean"]), _c(fwd["inverse_covariance"]),
                            _c(fwd["projected_color"]), _c(fwd["projected_opacity"]),
                            _c(fwd["gaussian_ids"], np.int32), _c(fwd["ranges"], np.int64),
                            len(fwd["gaussian_ids"]), _c(grad_image),
                            _c(fwd["final_transmittance"]), _c(fwd["n_contributors"], np.int32),
                            ctypes.byref(p), None if tiles_arr is None else tiles_arr.ctypes.data,
                            0 if tiles_arr is None else len(tiles_arr), grad)
    return grad


def project_bwd(mean, rotation, scale, opacity, color, camera_rotation, camera_translation,
                inverse_covariance, grad_projected, counts, s: Settings) -> dict:
    n = mean.shape[0]
    num_sh = color.shape[1]
    out = dict(mean=np.empty((n, 3), np.float32), rotation=np.empty((n, 4), np.float32),
               scale=np.empty((n, 3), np.float32), opacity=np.empty((n, 1), np.float32),
               color=np.empty((n, num_sh, 3), np.float32))
    p = s.params()
    lib().gso_project_bwd(n, _c(mean), _c(rotation), _c(scale), _c(opacity), _c(color), num_sh,
                          _c(camera_rotation), _c(camera_translation), _c(inverse_covariance),
                          _c(grad_projected), _c(counts, np.int32), ctypes.byref(p),
                          out["mean"], out["rotation"], out["scale"], out["opacity"],
                          out["color"])
    return out


def backward(inputs: dict, fwd: dict, grad_image, s: Settings, tiles=None) -> dict:
    """Parameter gradients for ``grad_image`` (interface.py:176-239)."""
    grad_projected = composite_bwd(fwd, grad_image, s, tiles)
    grads = project_bwd(inputs["mean"], inputs["rotation"], inputs["scale"], inputs["opacity"],
                        inputs["color"], inputs["camera_rotation"], inputs["camera_translation"],
                        fwd["inverse_covariance"], grad_projected, fwd["counts"], s)
    grads["grad_projected"] = grad_projected
    return grads


def exp(x) -> np.ndarray:
    x = _c(x)
    y = np.empty_like(x)
    lib().gso_exp_array(x.size, x, y)
    return y


def log(x) -> np.ndarray:
    x = _c(x)
    y = np.empty_like(x)
    lib().gso_log_array(x.size, x, y)
    return y


def load_golden(path: str) -> tuple[dict, Settings, dict]:
    """Inputs, settings and recorded reference outputs of a golden ``.npz``."""
    d = np.load(path)
    inputs = {k[3:]: d[k] for k in d.files if k.startswith("in_")}
    fx, fy, cx, cy = (float(v) for v in inputs["intrinsics"])
    w, h = (int(v) for v in inputs["image_size"])
    near, far = (float(v) for v in inputs["near_far"])
    s = Settings(fx=fx, fy=fy, cx=cx, cy=cy, width=w, height=h,
                 tile_size=int(inputs["tile_size"]),
                 opacity_threshold=float(inputs["opacity_threshold"]), near=near, far=far,
                 rendering_mode=str(inputs["rendering_mode"]),
                 confidence=float(inputs["confidence"]))
    expected = {k: d[k] for k in d.files if not k.startswith("in_")}
    return inputs, s, expected


def scene_inputs(scene, view: int = 0) -> tuple[dict, Settings]:
    """Numpy inputs and settings for one camera of a scene object (duck-typed:
    ``tensors()``, ``cameras``, ``settings`` as in the package's scenes)."""
    camera = scene.cameras[view]
    fx, fy = camera.focal_length
    cx, cy = camera.principal_point
    w, h = camera.image_size
    st = scene.settings
    names = ("mean", "rotation", "scale", "opacity", "color")
    inputs = {k: t.detach().cpu().numpy() for k, t in zip(names, scene.tensors())}
    inputs["camera_rotation"] = camera.rotation_matrix.cpu().numpy()
    inputs["camera_translation"] = camera.translation.cpu().numpy()
    settings = Settings(fx=fx, fy=fy, cx=cx, cy=cy, width=w, height=h, tile_size=st.tile_size,
                        opacity_threshold=st.opacity_threshold, near=st.near, far=st.far,
                        rendering_mode=st.rendering_mode, confidence=st.confidence)
    return inputs, settings


ADAM_NAMES = ("mean", "rotation", "scale", "opacity", "color")


def adam_scalars(step: int, lrs, betas=(0.9, 0.999), eps=1e-15, noise_lr=0.0,
                 position_lr=0.0) -> AdamParams:
    """Scalars of Adam step ``step`` (1-based; an int for all five groups or
    one per group) folded in double like torch.optim.Adam's foreach path
    (torch/optim/adam.py: bias corrections 1 - beta^step, step size
    -(lr / bc1), sqrt(bc2))."""
    beta1, beta2 = betas
    steps = [step] * 5 if isinstance(step, int) else list(step)
    h = AdamParams()
    h.lerp_weight, h.beta2, h.sq_weight, h.eps = 1 - beta1, beta2, 1 - beta2, eps
    for k, (t, lr) in enumerate(zip(steps, lrs)):
        bc1 = 1 - beta1 ** t
        bc2 = 1 - beta2 ** t
        h.neg_step_size[k] = (lr / bc1) * -1
        h.bias2_sqrt[k] = bc2 ** 0.5
    h.noise_lr, h.position_lr = noise_lr, position_lr
    return h


def adam_step(params: dict, grads: dict, exp_avg: dict, exp_avg_sq: dict, hyper: AdamParams,
              randn=None) -> dict:
    """One Adam step (+ position noise when ``randn`` [N,3] is given) on copies
    of the float32 arrays; returns {"params", "exp_avg", "exp_avg_sq"} keyed by
    ADAM_NAMES. A missing gradient skips that parameter."""
    out = {key: {k: np.array(src[k], dtype=np.float32, copy=True) for k in ADAM_NAMES}
           for key, src in (("params", params), ("exp_avg", exp_avg),
                            ("exp_avg_sq", exp_avg_sq))}
    g = {k: (_c(grads[k]) if grads.get(k) is not None else None) for k in ADAM_NAMES}
    ptr5 = ctypes.c_void_p * 5
    addr = lambda d: ptr5(*(None if d[k] is None else d[k].ctypes.data for k in ADAM_NAMES))  # noqa: E731
    n = out["params"]["mean"].shape[0]
    num_sh = out["params"]["color"].shape[1]
    r = None if randn is None else _c(randn)
    lib().gso_adam_step(n, num_sh, addr(out["params"]), addr(g), addr(out["exp_avg"]),
                        addr(out["exp_avg_sq"]), ctypes.byref(hyper),
                        None if r is None else r.ctypes.data)
    return out


def relocate(state: dict, counts, output_indices=None, output_base: int = 0,
             exp_avg: dict | None = None, exp_avg_sq: dict | None = None) -> dict:
    """copy_splats + normalize_copies + the moment reset of relocate_splats
    (training/utils.py:94-101,120-145,187-193) on copies of the float32 arrays.

    ``state`` holds mean, rotation, scale, opacity, color and optionally
    normals (all rows, including the output rows); ``counts`` [n_src] int64;
    output slot j writes row ``output_indices[j]`` or ``output_base + j``.
    Returns {"state", "exp_avg", "exp_avg_sq", "error"} (error bits as
    gso_relocate returns them)."""
    out = {k: np.array(v, dtype=np.float32, copy=True) for k, v in state.items()}
    moments = [None if m is None else {k: np.array(v, dtype=np.float32, copy=True)
                                       for k, v in m.items()} for m in (exp_avg, exp_avg_sq)]
    counts = np.ascontiguousarray(counts, dtype=np.int64)
    rows = out["mean"].shape[0]
    idx = None if output_indices is None else np.ascontiguousarray(output_indices, np.int64)
    num_outputs = int(np.maximum(counts, 0).sum()) if idx is None else len(idx)
    ptrs = (ctypes.c_void_p * 10)(*(
        None if m is None or m.get(k) is None else m[k].ctypes.data
        for m in moments for k in ADAM_NAMES))
    normals = out.get("normals")
    error = lib().gso_relocate(
        len(counts), rows, out["color"].shape[1], counts.ctypes.data, num_outputs,
        None if idx is None else idx.ctypes.data, output_base, out["mean"], out["rotation"],
        out["scale"], out["opacity"], out["color"],
        None if normals is None else normals.ctypes.data, ptrs)
    return {"state": out, "exp_avg": moments[0], "exp_avg_sq": moments[1], "error": error}
