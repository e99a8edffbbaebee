"""Gaussian splats in PLY files, in the reference's field layout.

Same fields, order and conventions as the reference's ``splats/ply.py:12-89``
(which writes through ``plyfile``, not available here): one ``vertex``
element of float32 properties

    x y z  nx ny nz  f_dc_0..2  f_rest_0..3(K-1)-1  opacity  scale_0..2  rot_0..3

where ``f_rest`` holds the SH coefficients 1..K-1 channel-major (all of red,
then green, then blue), opacity is the logit, scale the log sigma and rot the
(w, x, y, z) quaternion. Files are written binary little-endian; the reader
also takes big-endian and ASCII files, any scalar property types, extra
properties, and further elements after ``vertex`` (as plyfile does). Missing
normals read as zeros.
"""

from __future__ import annotations

from pathlib import Path

import numpy as np
import torch

# PLY scalar type names (both spellings of the spec) -> numpy type codes.
PLY_TYPES = {
    "char": "i1", "int8": "i1", "uchar": "u1", "uint8": "u1",
    "short": "i2", "int16": "i2", "ushort": "u2", "uint16": "u2",
    "int": "i4", "int32": "i4", "uint": "u4", "uint32": "u4",
    "float": "f4", "float32": "f4", "double": "f8", "float64": "f8",
}


def ply_fields(num_sh: int) -> list[str]:
    """Vertex property names for K = ``num_sh`` SH coefficients per channel."""
    return (["x", "y", "z", "nx", "ny", "nz"] + [f"f_dc_{i}" for i in range(3)]
            + [f"f_rest_{i}" for i in range((num_sh - 1) * 3)] + ["opacity"]
            + [f"scale_{i}" for i in range(3)] + [f"rot_{i}" for i in range(4)])


def save_ply(state: dict[str, torch.Tensor], path: str | Path) -> None:
    """Write a splat state dict (mean, rotation, scale, opacity, color and
    optionally normals) as a binary little-endian PLY (splats/ply.py:12-52)."""
    path = Path(path)
    mean, rotation, scale, opacity, color = (
        state[k].detach().cpu().numpy().astype(np.float32)
        for k in ("mean", "rotation", "scale", "opacity", "color"))
    normals = state.get("normals")
    normals = (np.zeros_like(mean) if normals is None
               else normals.detach().cpu().numpy().astype(np.float32))
    n, k, c = color.shape
    if c != 3 or int(k ** 0.5) ** 2 != k:
        raise ValueError(f"Invalid color shape {color.shape}. Expected [N, (degree + 1) ** 2, 3]")
    values = np.concatenate(
        (mean, normals, color[:, 0], color[:, 1:].transpose(0, 2, 1).reshape(n, (k - 1) * 3),
         opacity.reshape(n, 1), scale, rotation), axis=1)
    fields = ply_fields(k)
    header = ["ply", "format binary_little_endian 1.0", f"element vertex {n}"]
    header += [f"property float {name}" for name in fields] + ["end_header"]
    path.parent.mkdir(parents=True, exist_ok=True)
    with open(path, "wb") as f:
        f.write(("\n".join(header) + "\n").encode("ascii"))
        f.write(np.ascontiguousarray(values, dtype="<f4").tobytes())


def _read_header(f):
    if f.readline().strip() != b"ply":
        raise ValueError("not a PLY file")
    fmt, elements = None, []
    while True:
        line = f.readline()
        if not line:
            raise ValueError("PLY header has no end_header")
        words = line.decode("ascii").split()
        if not words or words[0] in ("comment", "obj_info"):
            continue
        if words[0] == "end_header":
            return fmt, elements
        if words[0] == "format":
            fmt = words[1]
        elif words[0] == "element":
            elements.append((words[1], int(words[2]), []))
        elif words[0] == "property":
            if not elements:
                raise ValueError("PLY property before any element")
            if words[1] == "list":
                elements[-1][2].append((words[4], None))
            else:
                if words[1] not in PLY_TYPES:
                    raise ValueError(f"unknown PLY property type {words[1]!r}")
                elements[-1][2].append((words[2], PLY_TYPES[words[1]]))


def _read_vertices(path) -> np.ndarray:
    with open(path, "rb") as f:
        fmt, elements = _read_header(f)
        if fmt not in ("ascii", "binary_little_endian", "binary_big_endian"):
            raise ValueError(f"unknown PLY format {fmt!r}")
        for name, count, props in elements:
            if any(code is None for _, code in props):
                if name == "vertex":
                    raise ValueError("list properties in the vertex element are not supported")
                raise ValueError(f"cannot skip element {name!r} with list properties before "
                                 "the vertices")
            if fmt == "ascii":
                rows = [f.readline() for _ in range(count)]
                if name != "vertex":
                    continue
                dtype = np.dtype([(p, code) for p, code in props])
                table = np.loadtxt(rows, dtype=np.float64, ndmin=2) if count else \
                    np.zeros((0, len(props)))
                out = np.empty(count, dtype=dtype)
                for i, (p, _) in enumerate(props):
                    out[p] = table[:, i]
                return out
            order = "<" if fmt == "binary_little_endian" else ">"
            dtype = np.dtype([(p, order + code) for p, code in props])
            data = f.read(dtype.itemsize * count)
            if len(data) != dtype.itemsize * count:
                raise ValueError(f"PLY element {name!r} is truncated")
            if name == "vertex":
                return np.frombuffer(data, dtype=dtype)
    raise ValueError("PLY file has no vertex element")


def load_ply(path: str | Path) -> dict[str, torch.Tensor]:
    """Read a splat PLY into the state dict ``save_ply`` writes
    (splats/ply.py:55-89): float32 mean, normals (zeros if absent), rotation,
    scale, opacity [N,1] and color [N,K,3]."""
    path = Path(path)
    if path.suffix.lower() != ".ply":
        raise ValueError(f"Only .ply files are supported. Got {path}")
    vertex = _read_vertices(path)
    names = vertex.dtype.names or ()

    def columns(fields):
        return np.stack([vertex[name].astype(np.float32) for name in fields], axis=1) \
            if len(vertex) else np.zeros((0, len(fields)), np.float32)

    mean = columns(["x", "y", "z"])
    normals = columns(["nx", "ny", "nz"]) if all(n in names for n in ("nx", "ny", "nz")) \
        else np.zeros_like(mean)
    rest = len([name for name in names if name.startswith("f_rest_")])
    if rest % 3:
        raise ValueError(f"{rest} f_rest properties is not a multiple of 3")
    dc = columns([f"f_dc_{i}" for i in range(3)])
    sh = (columns([f"f_rest_{i}" for i in range(rest)]).reshape(len(vertex), 3, -1)
          .transpose(0, 2, 1) if rest else np.empty((len(vertex), 0, 3), np.float32))
    return {
        "mean": torch.from_numpy(np.ascontiguousarray(mean)),
        "normals": torch.from_numpy(np.ascontiguousarray(normals)),
        "rotation": torch.from_numpy(columns([f"rot_{i}" for i in range(4)])),
        "scale": torch.from_numpy(columns([f"scale_{i}" for i in range(3)])),
        "opacity": torch.from_numpy(np.ascontiguousarray(columns(["opacity"]))),
        "color": torch.from_numpy(np.ascontiguousarray(
            np.concatenate((dc[:, None], sh), axis=1))),
    }
