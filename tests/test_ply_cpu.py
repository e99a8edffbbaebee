"""PLY I/O in the reference's field layout (splats/ply.py:12-89): round trips,
the exact header and byte layout, channel-major SH, and reading the variants
plyfile accepts (big-endian, ASCII, doubles, extra properties and elements)."""

import numpy as np
import pytest
import torch

from gaussian_splats_b200.ply import load_ply, ply_fields, save_ply
from gaussian_splats_b200.splats import GaussianSplat


def _state(n=7, k=16, seed=0):
    g = torch.Generator().manual_seed(seed)
    return {"mean": torch.randn(n, 3, generator=g), "rotation": torch.randn(n, 4, generator=g),
            "scale": torch.randn(n, 3, generator=g), "opacity": torch.randn(n, 1, generator=g),
            "color": torch.randn(n, k, 3, generator=g), "normals": torch.randn(n, 3, generator=g)}


@pytest.mark.parametrize("k", [1, 4, 9, 16, 25])
def test_round_trip(tmp_path, k):
    state = _state(k=k)
    save_ply(state, tmp_path / "a.ply")
    back = load_ply(tmp_path / "a.ply")
    for key, value in state.items():
        assert back[key].dtype == torch.float32
        torch.testing.assert_close(back[key], value, rtol=0, atol=0)


def test_header_and_layout(tmp_path):
    state = _state(n=2, k=4)
    save_ply(state, tmp_path / "b.ply")
    raw = (tmp_path / "b.ply").read_bytes()
    header, body = raw.split(b"end_header\n", 1)
    lines = header.decode().splitlines()
    assert lines[:3] == ["ply", "format binary_little_endian 1.0", "element vertex 2"]
    assert [line.split()[2] for line in lines[3:]] == ply_fields(4)
    assert all(line.split()[1] == "float" for line in lines[3:])
    rows = np.frombuffer(body, dtype="<f4").reshape(2, -1)
    assert rows.shape[1] == 6 + 3 + 9 + 1 + 3 + 4
    color = state["color"].numpy()
    # f_rest is channel-major: the red coefficients 1..3, then green, then blue
    np.testing.assert_array_equal(rows[:, 9:18], color[:, 1:].transpose(0, 2, 1).reshape(2, 9))
    np.testing.assert_array_equal(rows[:, 6:9], color[:, 0])
    np.testing.assert_array_equal(rows[:, 18], state["opacity"].numpy()[:, 0])
    np.testing.assert_array_equal(rows[:, -4:], state["rotation"].numpy())


def test_missing_normals_and_checkpoint_conversion(tmp_path):
    state = _state(n=5, k=9)
    del state["normals"]
    save_ply(state, tmp_path / "c.ply")
    back = load_ply(tmp_path / "c.ply")
    assert torch.count_nonzero(back["normals"]) == 0
    splats = GaussianSplat.from_tensors(**back)  # convert.py: ply-to-pt
    torch.testing.assert_close(splats.color.detach(), state["color"])


def _write(path, fmt, props, rows, extra=b""):
    header = ["ply", f"format {fmt} 1.0", "comment made by a test", f"element vertex {len(rows)}"]
    header += [f"property {t} {name}" for t, name in props]
    header += ["element face 1", "property list uchar int vertex_indices", "end_header"]
    with open(path, "wb") as f:
        f.write(("\n".join(header) + "\n").encode())
        if fmt == "ascii":
            f.write("".join(" ".join(repr(float(v)) for v in r) + "\n" for r in rows).encode())
        else:
            order = "<" if fmt == "binary_little_endian" else ">"
            dtype = np.dtype([(name, order + {"float": "f4", "double": "f8", "uchar": "u1"}[t])
                              for t, name in props])
            data = np.empty(len(rows), dtype)
            for i, (_, name) in enumerate(props):
                data[name] = [r[i] for r in rows]
            f.write(data.tobytes())
        f.write(extra)


@pytest.mark.parametrize("fmt", ["ascii", "binary_little_endian", "binary_big_endian"])
def test_reads_other_writers(tmp_path, fmt):
    names = ["x", "y", "z", "f_dc_0", "f_dc_1", "f_dc_2", "opacity", "scale_0", "scale_1",
             "scale_2", "rot_0", "rot_1", "rot_2", "rot_3"]
    props = [("double", n) for n in names] + [("uchar", "red")]
    rows = [[float(i + j) / 8 for j in range(len(names))] + [200] for i in range(3)]
    _write(tmp_path / "d.ply", fmt, props, rows, extra=b"" if fmt == "ascii" else b"\x03")
    back = load_ply(tmp_path / "d.ply")
    assert back["color"].shape == (3, 1, 3) and back["normals"].abs().sum() == 0
    np.testing.assert_allclose(back["mean"].numpy(), np.array(rows)[:, :3], rtol=1e-7)
    np.testing.assert_allclose(back["rotation"].numpy(), np.array(rows)[:, 10:14], rtol=1e-7)


def test_rejects_bad_files(tmp_path):
    (tmp_path / "x.txt").write_text("ply\n")
    with pytest.raises(ValueError):
        load_ply(tmp_path / "x.txt")
    (tmp_path / "y.ply").write_bytes(b"not a ply\n")
    with pytest.raises(ValueError):
        load_ply(tmp_path / "y.ply")
    with pytest.raises(ValueError):
        save_ply(dict(_state(), color=torch.zeros(7, 5, 3)), tmp_path / "z.ply")


def test_convert_round_trip(tmp_path):
    from gaussian_splats_b200.convert import ply_to_pt, pt_to_ply

    splats = GaussianSplat(11, sh_degree=2)
    splats.save_checkpoint(tmp_path / "s.pt")
    ply = pt_to_ply(tmp_path / "s.pt")
    assert ply == tmp_path / "s.ply" and ply.exists()
    back = GaussianSplat.from_checkpoint(ply_to_pt(ply, tmp_path / "t.pt"))
    for name in ("mean", "rotation", "scale", "opacity", "color", "normals"):
        torch.testing.assert_close(getattr(back, name), getattr(splats, name), rtol=0, atol=0)
